"""The Case protocol: the one interface between the harness and an algorithm.

Same fields as the reference's ``framework/case.py:13-35`` (``Case`` dataclass): ``name``,
``description``, ``params``, ``grad_inputs``, ``dtype``, ``make_inputs`` and
``reference_forward``.
"""
from dataclasses import dataclass
from typing import Callable


@dataclass
class Case:
    """One algorithm: its scalar parameters, which inputs receive gradients, the acceptance
    dtype, a seeded input generator ``(seed, dtype, device, requires_grad) -> dict`` and the
    PyTorch forward that defines correctness ``(inputs, params) -> Tensor`` (its backward comes
    from autograd)."""
    name: str
    description: str
    params: dict
    grad_inputs: list
    dtype: str
    make_inputs: Callable
    reference_forward: Callable
