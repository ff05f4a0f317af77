"""Row sharding of the RBF forward + backward across the GPUs of one node.

No reference counterpart (the reference runs on one GPU).  The split:
  * X, G and K are partitioned by rows: rank r owns rows ``row_range(N, world, r)``;
  * Y is replicated;
  * forward: K_r = rbf(X_r, Y) is local, no communication;
  * backward: dX_r is local and complete; dY is linear in the rows, so each rank computes the
    partial dY over its rows and ONE all-reduce (sum) over the process group completes it.
One process per GPU; the collective is ``torch.distributed.all_reduce`` on the NCCL backend on
GPUs (NVLink / NVSwitch), gloo on CPU in the tests.  The compute is pluggable so that the same
driver runs with the sm_100a kernels (``native``) or with a CPU implementation in tests.
"""
import torch
import torch.distributed as dist


def row_range(n_rows, world, rank):
    """Balanced contiguous [start, stop) of ``n_rows`` for ``rank`` of ``world``."""
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class NativeShardCompute:
    """The sm_100a kernels through the C ABI: forward (filling the workspace) and the
    prepared shard backward."""

    def forward(self, X, Y, gamma):
        from cases.rbf import native
        return native.forward_with_workspace(X, Y, gamma)

    def backward(self, X, Y, G, K, gamma, state):
        from cases.rbf import native
        return native.rbf_backward(X, Y, G, K, gamma, workspace=state)


def forward_backward_shard(X_local, Y, G_local, gamma, compute=None, group=None,
                           reduce_dy=True):
    """One forward + backward of this rank's rows.  Returns (K_local, dX_local, dY) where dY is
    the full gradient (all-reduced over ``group``) when ``reduce_dy`` and the process group is
    initialised, else this rank's partial sum."""
    compute = compute or NativeShardCompute()
    K_local, state = compute.forward(X_local, Y, gamma)
    dX_local, dY = compute.backward(X_local, Y, G_local, K_local, gamma, state)
    if reduce_dy and dist.is_available() and dist.is_initialized():
        dist.all_reduce(dY, op=dist.ReduceOp.SUM, group=group)
    return K_local, dX_local, dY


def shard_inputs(X, G, world, rank):
    """Views of the rows of X and G this rank owns."""
    a, b = row_range(X.shape[0], world, rank)
    return X[a:b], G[a:b]


def max_over_ranks(value, device=None, group=None):
    """Max of a scalar over the process group (identity when not distributed)."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
