"""The row-sharded forward + backward driver (cases/rbf/shard.py) on two CPU ranks (gloo).

The compute is the fp64 oracle on each rank's rows; the test checks that the sharded K and dX
rows and the all-reduced dY equal the unsharded oracle result, which exercises the partition
and the single dY collective without a GPU.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases.rbf import shard


class OracleCompute:
    """CPU stand-in for NativeShardCompute with the same call shapes."""

    def forward(self, X, Y, gamma):
        from oracle import oracle
        K = oracle.forward(X.numpy(), Y.numpy(), gamma)
        return torch.from_numpy(K.astype(np.float32)), None

    def backward(self, X, Y, G, K, gamma, state):
        from oracle import oracle
        dX, dY = oracle.backward(X.numpy(), Y.numpy(), G.numpy(), gamma)
        return torch.from_numpy(dX.astype(np.float32)), torch.from_numpy(dY.astype(np.float32))


class OneCallOracleCompute(OracleCompute):
    """Stand-in with the one-call entry of NativeShardCompute (forward_backward): the driver must
    use it, not the two calls."""

    def forward(self, X, Y, gamma):
        raise AssertionError("the one-call entry should have been used")

    def forward_backward(self, X, Y, G, gamma):
        K, _ = OracleCompute.forward(self, X, Y, gamma)
        dX, dY = OracleCompute.backward(self, X, Y, G, K, gamma, None)
        return K, dX, dY, None


def _worker(rank, world, port, N, M, D, gamma, out_dir, one_call=False):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "nl2cuda-kernel-agent_b200"), root):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(5)
    X = torch.randn(N, D, generator=g)
    Y = torch.randn(M, D, generator=g)
    G = torch.randn(N, M, generator=g)
    Xl, Gl = shard.shard_inputs(X, G, world, rank)
    compute = OneCallOracleCompute() if one_call else OracleCompute()
    K, dX, dY = shard.forward_backward_shard(Xl, Y, Gl, gamma, compute=compute)
    a, b = shard.row_range(N, world, rank)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), K=K.numpy(), dX=dX.numpy(), dY=dY.numpy(),
             a=a, b=b)
    t = shard.max_over_ranks(float(rank) + 0.5)
    assert t == world - 0.5
    dist.barrier()
    dist.destroy_process_group()


def test_row_range_partitions():
    for n in (0, 1, 7, 4096, 4097):
        for w in (1, 2, 3, 8):
            ranges = [shard.row_range(n, w, r) for r in range(w)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(ranges[r][1] == ranges[r + 1][0] for r in range(w - 1))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world,one_call", [(2, False), (2, True)])
def test_two_rank_shard_matches_unsharded(tmp_path, world, one_call):
    N, M, D, gamma = 37, 29, 6, 0.15
    port = 29500 + (os.getpid() % 1000) + (7 if one_call else 0)
    mp.spawn(_worker, args=(world, port, N, M, D, gamma, str(tmp_path), one_call), nprocs=world,
             join=True)
    from oracle import oracle
    g = torch.Generator().manual_seed(5)
    X = torch.randn(N, D, generator=g)
    Y = torch.randn(M, D, generator=g)
    G = torch.randn(N, M, generator=g)
    K = oracle.forward(X.numpy(), Y.numpy(), gamma)
    dX, dY = oracle.backward(X.numpy(), Y.numpy(), G.numpy(), gamma)
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        a, b = int(z["a"]), int(z["b"])
        np.testing.assert_allclose(z["K"], K[a:b], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(z["dX"], dX[a:b], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(z["dY"], dY, rtol=1e-5, atol=1e-6)


class TimedOutCompute(OracleCompute):
    """The native compute's status hook, faked: rank 1's device wait ran out (status 7)."""

    def __init__(self, rank):
        self.rank = rank

    def status(self, state):
        return 7 if self.rank == 1 else 0


def _status_worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "nl2cuda-kernel-agent_b200"), root):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    X, Y, G = torch.randn(6, 3), torch.randn(5, 3), torch.randn(6, 5)
    Xl, Gl = shard.shard_inputs(X, G, world, rank)
    outcome = "ok"
    try:
        # The status is read before the dY collective: the failing rank raises and never joins
        # it, so the check must not be left to a collective that would wait for it.
        shard.forward_backward_shard(Xl, Y, Gl, 0.1, compute=TimedOutCompute(rank),
                                     reduce_dy=False, check_status=True)
    except RuntimeError as e:
        outcome = "raised: " + str(e)
    with open(os.path.join(out_dir, f"status{rank}.txt"), "w") as f:
        f.write(outcome)
    dist.destroy_process_group()


def test_status_check_raises_on_the_rank_whose_wait_timed_out(tmp_path):
    port = 30500 + (os.getpid() % 1000)
    mp.spawn(_status_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "status0.txt").read_text() == "ok"
    r1 = (tmp_path / "status1.txt").read_text()
    assert r1.startswith("raised:") and "timed out" in r1


def test_status_check_is_opt_in(monkeypatch):
    monkeypatch.delenv("RBF_CHECK_STATUS", raising=False)
    assert shard.check_status_default() is False
    monkeypatch.setenv("RBF_CHECK_STATUS", "1")
    assert shard.check_status_default() is True
