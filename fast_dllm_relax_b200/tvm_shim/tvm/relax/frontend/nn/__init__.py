"""tvm.relax.frontend.nn stand-in.

Only the names that fast_dllm_relax/model/cuda.py and model/metal.py reference at import time are
defined.  Building a graph from them raises: the sm_100a library is the compiled module.
"""

from __future__ import annotations

from . import core  # noqa: F401
from ...._inert import _Inert


class Module:
    """Base class placeholder; constructing a reference model class raises."""

    def __init__(self, *args, **kwargs):
        raise NotImplementedError("Relax graph construction is not available with the sm_100a library")


class Tensor:
    """Placeholder for nn.Tensor (only used in annotations at import time)."""

    @staticmethod
    def from_scalar(*_args, **_kwargs):
        raise NotImplementedError("Relax graph construction is not available with the sm_100a library")

    @staticmethod
    def placeholder(*_args, **_kwargs):
        raise NotImplementedError("Relax graph construction is not available with the sm_100a library")


class ExternModule:
    pass


Parameter = _Inert("tvm.relax.frontend.nn.Parameter")
Linear = _Inert("tvm.relax.frontend.nn.Linear")
Embedding = _Inert("tvm.relax.frontend.nn.Embedding")
ModuleList = _Inert("tvm.relax.frontend.nn.ModuleList")
op = _Inert("tvm.relax.frontend.nn.op")
spec = _Inert("tvm.relax.frontend.nn.spec")
