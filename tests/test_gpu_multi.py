"""Row-sharded forward + backward on 2 GPUs (skipped with fewer): the dY reduction fused into the
backward over peer memory (shard.RoutedDy) against the NCCL all-reduce path and the oracle,
CUDA-graph replays of the routed step, and the bounded cross-GPU wait running out when one rank
never joins (no GPU fault: the waiting kernel returns RBF_ERR_TIMEOUT, the failure is sticky on
those buffers, and the status-checking step raises)."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N_PER, M, D, GAMMA = 300, 516, 48, 0.02


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    r = np.random.default_rng(42)
    X = r.standard_normal((2 * N_PER, D)).astype(np.float32)
    Y = r.standard_normal((M, D)).astype(np.float32)
    G = r.standard_normal((2 * N_PER, M)).astype(np.float32)
    return X, Y, G


def _worker(rank, world, port, out_dir, one_phase_max):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "nl2cuda-kernel-agent_b200"), root):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from cases.rbf import native, shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      RBF_XCHG_ONE_PHASE_MAX=str(one_phase_max))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        X, Y, G = _inputs()
        a, b = shard.row_range(X.shape[0], world, rank)
        Xd = torch.from_numpy(X[a:b]).to(dev)
        Yd = torch.from_numpy(Y).to(dev)
        Gd = torch.from_numpy(G[a:b]).to(dev)
        K0, dX0, dY0 = shard.forward_backward_shard(Xd, Yd, Gd, GAMMA)  # NCCL all-reduce
        route = shard.RoutedDy(M, D, dev)
        for _ in range(4):  # eager steps: the slot rotates through all three
            K1, dX1, dY1 = shard.forward_backward_shard(Xd, Yd, Gd, GAMMA, route=route)
            torch.testing.assert_close(dY1, dY0, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(dX1, dX0, rtol=1e-5, atol=1e-6)
            assert torch.equal(K1, K0)
        # CUDA graph of the routed step, replayed: the slot comes from device memory.
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                Kg, dXg, dYg = shard.forward_backward_shard(Xd, Yd, Gd, GAMMA, route=route)
        torch.cuda.current_stream(dev).wait_stream(s)
        for _ in range(5):
            g.replay()
            torch.cuda.synchronize(dev)
            torch.testing.assert_close(dYg, dY0, rtol=1e-5, atol=1e-6)
        np.save(os.path.join(out_dir, f"dY_{rank}.npy"), dYg.cpu().numpy())
        np.save(os.path.join(out_dir, f"dX_{rank}.npy"), dXg.cpu().numpy())
        del g
        dist.barrier()

        # Bounded wait: rank 1 never joins this exchange; rank 0's wait runs out (100 ms).
        route2 = shard.RoutedDy(M, D, dev)
        K, ws = native.forward_with_workspace(Xd, Yd, GAMMA)
        native.rbf_backward_shard_routed(Xd, Yd, Gd, K, GAMMA, ws, route2)
        if rank == 0:
            os.environ["RBF_WAIT_TIMEOUT_MS"] = "100"
            native.dy_exchange(route2, ws)
            torch.cuda.synchronize(dev)
            assert native.read_status(ws) == 7
            os.environ.pop("RBF_WAIT_TIMEOUT_MS")
            # The timeout is sticky: the counter did not advance, and the next exchange on the
            # same buffers skips its work and reports the timeout at once.
            assert route2.failed()
            assert int(route2.counters[0].item()) == 0
            native.dy_exchange(route2, ws)
            assert native.read_status(ws) == 7
            with pytest.raises(RuntimeError, match="timed out"):
                shard.forward_backward_shard(Xd, Yd, Gd, GAMMA, route=route2, check_status=True)
            # the context is still usable
            assert torch.isfinite(native.rbf_forward(Xd, Yd, GAMMA)).all()
        torch.cuda.synchronize(dev)
        dist.barrier()  # rank 1 keeps its peer memory alive until rank 0 is done with it
        with open(os.path.join(out_dir, f"ok_{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("one_phase_max", [8, 0])
def test_two_gpu_routed_dy(tmp_path, one_phase_max):
    """one_phase_max 8: one barrier, every rank sums all partials (the default);
    0: owners reduce, second barrier, gather."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), one_phase_max), nprocs=2, join=True)
    assert all((tmp_path / f"ok_{r}").exists() for r in range(2))
    from oracle import oracle
    X, Y, G = _inputs()
    dXr, dYr = oracle.backward(X, Y, G, GAMMA)
    from gpu_util import assert_gate
    for r in range(2):
        assert_gate(f"dY rank {r}", np.load(tmp_path / f"dY_{r}.npy"), dYr)
    dX = np.concatenate([np.load(tmp_path / f"dX_{r}.npy") for r in range(2)])
    assert_gate("dX", dX, dXr)
