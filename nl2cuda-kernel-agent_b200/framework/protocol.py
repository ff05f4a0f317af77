"""Tolerance and timing protocol (reference ``framework/protocol.py:12-36``).

The values are the reference's: allclose atol = rtol = 1e-2 over seeds 0-4; 10 warm-up and 100
timed iterations, 3 repeats, re-measure while the coefficient of variation exceeds 5% (at most
4 retries); a candidate passes the speed gate at >= 1.05x over ``torch.compile``.
``parity_tol`` is this build's stricter gate (max abs / rel error 1e-3 against the reference).
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Protocol:
    atol: float = 1e-2
    rtol: float = 1e-2
    seeds: tuple = (0, 1, 2, 3, 4)
    warmup: int = 10
    iters: int = 100
    repeats: int = 3
    cv_threshold: float = 0.05
    max_retries: int = 4
    speedup_target: float = 1.05
    parity_tol: float = 1e-3


PROTOCOL = Protocol()


def dtype_of(name):
    import torch
    table = {"float32": torch.float32, "float64": torch.float64, "float16": torch.float16}
    return table[name]
