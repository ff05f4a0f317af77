"""TEST / BASELINE INFRASTRUCTURE ONLY -- the reference's CPU implementation of the RBF path.

The reference's own CPU path is ``cases/rbf/reference.py:14-20``: the broadcast forward
``exp(-gamma * ((X[:,None]-Y[None])**2).sum(-1))`` with its backward from torch autograd.  That
file cannot travel to the GPU box, so this module restates it (same torch ops, same order) and
runs it over blocks of X rows so that the [rows, M, D] intermediate fits host memory; dY is
summed over the blocks.  bench.py times it as the CPU baseline ("kind": "port") and as the
``--impl reference`` arm.
"""
import time

import torch


def forward_backward_block(Xb, Y, Gb, gamma):
    """Reference forward + autograd backward on one block of X rows -> (K, dX, dY_partial)."""
    Xb = Xb.detach().clone().requires_grad_(True)
    Yl = Y.detach().clone().requires_grad_(True)
    diff = Xb.unsqueeze(1) - Yl.unsqueeze(0)
    K = torch.exp(-gamma * diff.pow(2).sum(dim=-1))
    K.backward(Gb)
    return K.detach(), Xb.grad, Yl.grad


def forward_backward(X, Y, G, gamma, block_rows=256):
    """Full forward + backward over row blocks -> (K, dX, dY)."""
    N = X.shape[0]
    K = torch.empty(N, Y.shape[0], dtype=X.dtype)
    dX = torch.empty_like(X)
    dY = torch.zeros_like(Y)
    for a in range(0, N, block_rows):
        b = min(N, a + block_rows)
        Kb, dXb, dYb = forward_backward_block(X[a:b], Y, G[a:b], gamma)
        K[a:b] = Kb
        dX[a:b] = dXb
        dY += dYb
    return K, dX, dY


def time_sample(N, M, D, gamma, sample_rows, threads, seed=0, block_rows=256, min_seconds=0.0):
    """Seconds for the reference forward + backward of ``sample_rows`` rows of X against all M
    rows of Y (inputs iid N(0,1)), using ``threads`` intra-op threads.  Returns (seconds,
    rows_done)."""
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    rows = max(1, min(sample_rows, N))
    X = torch.randn(rows, D, generator=g)
    Y = torch.randn(M, D, generator=g)
    G = torch.randn(rows, M, generator=g)
    forward_backward_block(X[:min(rows, 8)], Y, G[:min(rows, 8)], gamma)  # warm-up
    t0 = time.perf_counter()
    done = 0
    while True:
        forward_backward(X, Y, G, gamma, block_rows=block_rows)
        done += rows
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return el, done


# ---- cosine similarity: the reference's cases/cosine_sim/reference.py:14-21 + autograd ------

def cos_forward_backward_block(Ab, B, dSb, eps):
    """Reference forward + autograd backward on one block of A rows -> (S, dA, dB_partial)."""
    Ab = Ab.detach().clone().requires_grad_(True)
    Bl = B.detach().clone().requires_grad_(True)
    Ah = Ab / (Ab.norm(dim=-1, keepdim=True) + eps)
    Bh = Bl / (Bl.norm(dim=-1, keepdim=True) + eps)
    S = (Ah.unsqueeze(1) * Bh.unsqueeze(0)).sum(dim=-1)
    S.backward(dSb)
    return S.detach(), Ab.grad, Bl.grad


def cos_time_sample(N, M, D, eps, sample_rows, threads, seed=0, block_rows=256, min_seconds=0.0):
    """Seconds for the reference cosine forward + backward of ``sample_rows`` rows of A against
    all M rows of B, using ``threads`` intra-op threads.  Returns (seconds, rows_done)."""
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    rows = max(1, min(sample_rows, N))
    A = torch.randn(rows, D, generator=g)
    B = torch.randn(M, D, generator=g)
    dS = torch.randn(rows, M, generator=g)
    cos_forward_backward_block(A[:min(rows, 8)], B, dS[:min(rows, 8)], eps)  # warm-up
    t0 = time.perf_counter()
    done = 0
    while True:
        for a in range(0, rows, block_rows):
            b = min(rows, a + block_rows)
            cos_forward_backward_block(A[a:b], B, dS[a:b], eps)
        done += rows
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return el, done
