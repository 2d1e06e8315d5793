"""TVM stand-in for the sm_100a library (fast_dllm_relax_b200).

The reference's runtime and runners (fast_dllm_relax/runtime.py, runners.py) drive a compiled
TVM Relax module through a small slice of TVM's Python API.  This package provides exactly that
slice over PyTorch-owned tensors, so those files run unchanged on top of the sm_100a library:

* tvm.runtime: tensor / empty / from_dlpack / ShapeTuple / load_module, Tensor.copyfrom / numpy
  (runtime.py:246-255, 321-343; runners.py:68-76, 614)
* tvm.relax.VirtualMachine, vm[name](...)          (runners.py:615, runtime.py:169-176, 322-433)
* tvm.register_global_func / get_global_func       (runtime.py:63-80, runners.py:640, common.py:45)
* tvm.device / tvm.cuda / Device.sync              (runners.py:975-993, 1008-1013)
* inert definitions that let fast_dllm_relax/model/cuda.py import (its graph is never built here)

Put the directory that holds this package first on sys.path (or call
`fast_dllm_relax_b200.install_tvm_shim()`) before importing fast_dllm_relax.
"""

from __future__ import annotations

from . import runtime  # noqa: F401
from . import relax  # noqa: F401
from . import s_tir  # noqa: F401
from . import target  # noqa: F401
from . import transform  # noqa: F401
from .runtime import Device, cpu, cuda, device, metal  # noqa: F401

__version__ = "0.0.0+fdllm_sm100_shim"
IS_FDLLM_SHIM = True

_GLOBAL_FUNCS: dict = {
    "vm.builtin.reshape": runtime._reshape,
    "vm.builtin.memory_manager.clear": lambda: None,
}


def register_global_func(func_name, f=None, override: bool = False):
    """Register a Python function under a global name (decorator form supported)."""

    def _register(fn):
        if func_name in _GLOBAL_FUNCS and not override:
            raise ValueError(f"global function {func_name} is already registered")
        _GLOBAL_FUNCS[func_name] = fn
        return fn

    if f is not None:
        return _register(f)
    return _register


def get_global_func(name: str, allow_missing: bool = False):
    fn = _GLOBAL_FUNCS.get(name)
    if fn is None and not allow_missing:
        raise ValueError(f"global function {name} is not registered")
    return fn


def compile(*_args, **_kwargs):  # noqa: A001 -- TVM's name
    raise NotImplementedError(
        "graph compilation is not available: the sm_100a library replaces the compiled Relax module; "
        "export an artifact with fast_dllm_relax_b200.artifacts.write_artifact instead")
