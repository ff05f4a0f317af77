"""Cosine-similarity case: exposes ``CASE`` for the harness (reference
``cases/cosine_sim/__init__.py:16-24``)."""
import os

from framework.case import Case
from cases.cosine_sim import config
from cases.cosine_sim.reference import make_inputs, reference_forward


def _description():
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "description.md"),
              encoding="utf-8") as f:
        return f.read()


CASE = Case(
    name="cosine_sim",
    description=_description(),
    params={"eps": config.EPS},
    grad_inputs=["A", "B"],
    dtype=config.DTYPE,
    make_inputs=make_inputs,
    reference_forward=reference_forward,
)
