"""sm_100a (B200) library for Fast-dLLM v2 block-diffusion decoding.

    fast_dllm_relax_b200.engine.Engine     the nine entry points + fused extensions over torch tensors
    fast_dllm_relax_b200.artifacts         artifact directories (npz params, names, dtype, manifests)
    fast_dllm_relax_b200.vm_backend        vm[name] entry points for the TVM stand-in
    fast_dllm_relax_b200/tvm_shim/tvm      the TVM stand-in the reference's runtime imports
    include/fdllm_sm100.h                  the C ABI (lib/libfdllm_sm100.so)
"""

from __future__ import annotations

import sys
from pathlib import Path

TVM_SHIM_DIR = Path(__file__).resolve().parent / "tvm_shim"


def install_tvm_shim() -> None:
    """Put the TVM stand-in first on sys.path, so `import tvm` (and the reference's
    fast_dllm_relax.runtime / runners, which import it) resolve to it."""
    p = str(TVM_SHIM_DIR)
    if p in sys.path:
        sys.path.remove(p)
    sys.path.insert(0, p)
    mod = sys.modules.get("tvm")
    if mod is not None and not getattr(mod, "IS_FDLLM_SHIM", False):
        raise RuntimeError("another `tvm` package is already imported; call install_tvm_shim() before importing it")
