"""RBF case: exposes ``CASE`` for the harness (reference ``cases/rbf/__init__.py:16-24``)."""
import os

from framework.case import Case
from cases.rbf import config
from cases.rbf.reference import make_inputs, reference_forward


def _description():
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "description.md"),
              encoding="utf-8") as f:
        return f.read()


CASE = Case(
    name="rbf",
    description=_description(),
    params={"gamma": config.GAMMA},
    grad_inputs=["X", "Y"],
    dtype=config.DTYPE,
    make_inputs=make_inputs,
    reference_forward=reference_forward,
)
