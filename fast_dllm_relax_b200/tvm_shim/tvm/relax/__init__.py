"""tvm.relax stand-in: the VirtualMachine that dispatches vm[name] to a backend."""

from __future__ import annotations

from .._inert import _Inert
from . import frontend  # noqa: F401
from .. import transform  # noqa: F401

_PIPELINES: dict = {}


class VirtualMachine:
    """`relax.VirtualMachine(executable, device)`; `vm[name]` returns a callable entry point.

    `executable` is any object with `create_backend(device)`; the backend exposes
    `function(name)`, which raises for names the module does not export (the reference probes
    optional entries with try/except, runtime.py:113-151, runners.py:628-632).
    """

    def __init__(self, executable, device, memory_cfg=None, profile: bool = False):
        if isinstance(device, (list, tuple)):
            device = device[0]
        self.module = executable
        self.device = device
        self._backend = executable.create_backend(device)
        self._fns: dict = {}

    def __getitem__(self, name: str):
        fn = self._fns.get(name)
        if fn is None:
            fn = self._backend.function(name)
            self._fns[name] = fn
        return fn

    def __contains__(self, name: str) -> bool:
        try:
            self[name]
        except Exception:  # noqa: BLE001
            return False
        return True

    @property
    def backend(self):
        return self._backend


def register_pipeline(name: str):
    def _decorator(fn):
        _PIPELINES[name] = fn
        return fn

    return _decorator


def get_pipeline(name: str = "default", **kwargs):
    if name not in _PIPELINES:
        raise ValueError(f"unknown pipeline {name}")
    return _PIPELINES[name](**kwargs)


op = _Inert("tvm.relax.op")
const = _Inert("tvm.relax.const")
PrimValue = _Inert("tvm.relax.PrimValue")
ShapeExpr = _Inert("tvm.relax.ShapeExpr")
TensorStructInfo = _Inert("tvm.relax.TensorStructInfo")
backend = _Inert("tvm.relax.backend")
