"""Row sharding of the RBF forward + backward across the GPUs of one node.

No reference counterpart (the reference runs on one GPU).  The split:
  * X, G and K are partitioned by rows: rank r owns rows ``row_range(N, world, r)``;
  * Y is replicated;
  * forward: K_r = rbf(X_r, Y) is local, no communication;
  * backward: dX_r is local and complete; dY is linear in the rows, so each rank computes the
    partial dY over its rows and ONE all-reduce (sum) over the process group completes it.
One process per GPU; the collective is either ``torch.distributed.all_reduce`` (NCCL on GPUs,
gloo on CPU in the tests) or, with ``RoutedDy``, fused into the backward over peer memory.  The
compute is pluggable so that the same driver runs with the sm_100a kernels (``native``) or with
a CPU implementation in tests.
"""
import os

import torch
import torch.distributed as dist

RBF_ERR_TIMEOUT = 7


def check_status_default():
    """RBF_CHECK_STATUS=1 makes the production paths read the device status word after every
    step (one host synchronisation per step) and raise on a timed-out device wait."""
    return os.environ.get("RBF_CHECK_STATUS", "0") not in ("", "0")


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

    def forward_backward(self, X, Y, G, gamma):
        """Both passes in one library call (rbf_sm100_forward_backward: one split pass, which
        also zeroes the backward's accumulation targets).  Returns (K, dX, dY, state)."""
        from cases.rbf import native
        return tuple(native.rbf_forward_backward(X, Y, G, gamma, return_workspace=True))

    def status(self, state):
        """Device status word of the step's workspace (0 ok, 7 a bounded wait ran out)."""
        from cases.rbf import native
        return native.read_status(state)


class RoutedDy:
    """Peer-memory buffers of the fused dY reduction (no NCCL on the data path).

    Every rank holds, in CUDA symmetric memory, two M x D fp32 slots and an int[world] signal
    array; the backward accumulates this rank's dY partial into slot ``step % 2``, and
    ``native.dy_exchange`` completes dY over NVLink peer loads: barrier, each 128-row j-block
    summed by its owner (j-block % world), barrier, gather from the owners.  ``counters`` (this
    rank's device ints: step, two tickets) drive the slot choice on the device, so a captured
    CUDA graph of the step can be replayed.  Build it on every rank of ``group`` (collective).
    """

    def __init__(self, M, D, device, group=None):
        import ctypes
        import torch.distributed._symmetric_memory as symm_mem
        group = group or dist.group.WORLD
        self.M, self.D, self.device = int(M), int(D), torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise RuntimeError("the fused dY reduction supports 1..8 ranks")
        if self.D % 4:
            raise RuntimeError("the fused dY reduction needs D % 4 == 0")
        slot_bytes = 2 * self.M * self.D * 4
        self.flags_offset = (slot_bytes + 255) // 256 * 256
        nbytes = self.flags_offset + 256
        with torch.cuda.device(self.device):
            self.buffer = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            self.buffer.zero_()
            self.counters = torch.zeros(4, dtype=torch.int32, device=self.device)
            torch.cuda.synchronize()
        self.handle = symm_mem.rendezvous(self.buffer, group)
        # counters: [step, ticket 0, ticket 1, sticky failure flag] (rbf_sm100_dy_exchange)
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.dy_ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*[p + self.flags_offset for p in ptrs])
        dist.barrier(group=group)  # every rank's slots and flags are zero before the first step

    def failed(self):
        """True once an exchange on these buffers timed out (a peer never arrived): every later
        exchange skips its work, and the buffers must be built again.  Synchronizes."""
        return int(self.counters[3].item()) != 0


def _raise_on_status(st, where):
    if st != 0:
        raise RuntimeError(f"{where}: device status {st}"
                           + (" (a bounded device-side wait timed out; K, dX or dY are incomplete)"
                              if st == RBF_ERR_TIMEOUT else ""))


def forward_backward_shard(X_local, Y, G_local, gamma, compute=None, group=None,
                           reduce_dy=True, route=None, check_status=None):
    """One forward + backward of this rank's rows.  Returns (K_local, dX_local, dY) where dY is
    the full gradient when ``reduce_dy`` and the process group is initialised (all-reduced over
    ``group`` with NCCL, or -- with ``route``, a ``RoutedDy`` -- reduced inside the backward
    over peer memory), else this rank's partial sum.

    ``check_status`` (default: RBF_CHECK_STATUS=1): after the step, read the device status word
    (one synchronisation) and raise RuntimeError if a bounded device wait ran out -- in the
    forward, the backward or the dY exchange (whose timeout is sticky: later steps on the same
    ``route`` raise too, until it is built again)."""
    compute = compute or NativeShardCompute()
    if check_status is None:
        check_status = check_status_default()
    if route is not None:
        from cases.rbf import native
        K_local, ws = native.forward_with_workspace(X_local, Y, gamma)
        dX_local = native.rbf_backward_shard_routed(X_local, Y, G_local, K_local, gamma, ws, route)
        dY = native.dy_exchange(route, ws)
        if check_status:
            _raise_on_status(native.read_status(ws), "routed row-sharded step")
        return K_local, dX_local, dY
    if hasattr(compute, "forward_backward"):
        K_local, dX_local, dY, state = compute.forward_backward(X_local, Y, G_local, gamma)
    else:
        K_local, state = compute.forward(X_local, Y, gamma)
        dX_local, dY = compute.backward(X_local, Y, G_local, K_local, gamma, state)
    if check_status and hasattr(compute, "status"):
        _raise_on_status(compute.status(state), "row-sharded step")
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
