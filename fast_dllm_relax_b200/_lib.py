"""ctypes binding of the C ABI in include/fdllm_sm100.h (lib/libfdllm_sm100.so).

The library is required: there is no CPU or eager fallback.  If it has not been built,
`load()` raises with the build command.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libfdllm_sm100.so"

FDLLM_OK = 0
FDLLM_ERR_INVALID = -1
FDLLM_ERR_CUDA = -2
FDLLM_ERR_UNBOUND = -3
FDLLM_ERR_UNSUPPORTED = -4
FDLLM_ERR_DEVICE = -5

DEVICE_ERRORS = {
    0: "none", 1: "TMA producer wait expired", 2: "MMA issuer wait expired", 3: "epilogue wait expired",
    4: "token id outside the vocabulary", 5: "RoPE position outside the table", 6: "KV write outside the cache",
    7: "bounded-wait self test expired", 8: "(no longer raised)",
    9: "device refinement loop exceeded its iteration limit",
}


class FdllmConfig(ctypes.Structure):
    _fields_ = [
        ("vocab_size", ctypes.c_int32), ("hidden_size", ctypes.c_int32), ("intermediate_size", ctypes.c_int32),
        ("num_hidden_layers", ctypes.c_int32), ("num_attention_heads", ctypes.c_int32),
        ("num_key_value_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("tie_word_embeddings", ctypes.c_int32), ("bd_size", ctypes.c_int32),
        ("max_positions", ctypes.c_int32), ("dtype", ctypes.c_int32),
    ]


class FdllmRequest(ctypes.Structure):
    _fields_ = [
        ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("cap", ctypes.c_int32),
        ("rows", ctypes.c_int32), ("prefix_len", ctypes.c_int32), ("write_rel", ctypes.c_int32),
        ("attend_rel", ctypes.c_int32), ("cache_offset_host", ctypes.c_int32),
        ("cache_offset_dev", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
SIGNATURES: dict[str, tuple] = {
    "fdllm_abi_version": (ctypes.c_int, []),
    "fdllm_last_error": (ctypes.c_char_p, []),
    "fdllm_create": (_I, [ctypes.POINTER(FdllmConfig), _I, ctypes.POINTER(_P)]),
    "fdllm_destroy": (_I, [_P]),
    "fdllm_bind_params": (_I, [_P, ctypes.POINTER(_P), _I]),
    "fdllm_embed": (_I, [_P, _P, _I, _P, _P]),
    "fdllm_forward_hidden": (_I, [_P, _P, _P, _I, _P, _P]),
    "fdllm_get_logits": (_I, [_P, _P, _I, _P, _P]),
    "fdllm_build_prefix_cache": (_I, [_P, _P, _P, _I, _P, _P, _I, _P]),
    "fdllm_forward_cached": (_I, [_P, _P, _I, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "fdllm_forward_cached_batch": (_I, [_P, ctypes.POINTER(FdllmRequest), _I, _P, _P, _P]),
    "fdllm_build_prefix_cache_batch": (_I, [_P, ctypes.POINTER(FdllmRequest), _I, _P, _P]),
    "fdllm_confidence": (_I, [_P, _P, _I, _P, _P, _P]),
    "fdllm_confidence_from_logits": (_I, [_P, _P, _I, _P, _P, _P]),
    "fdllm_confidence_static": (_I, [_P, _P, _I, _P, _P, _P]),
    "fdllm_kernel_trace_enable": (_I, [_P, _I]),
    "fdllm_kernel_trace_read": (_I, [_P, _P, _P, _I, ctypes.POINTER(_I)]),
    "fdllm_unmask": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I, ctypes.c_double, _P, _P, _P, _P, _P]),
    "fdllm_token_logprob": (_I, [_P, _P, _I, _P, _P, _P]),
    "fdllm_unmask_batch": (_I, [_P, _P, _P, _P, _I, ctypes.c_double, _P, _P]),
    "fdllm_generate": (_I, [_P, _P, _I, _I, _I, _I, ctypes.c_double, _I, _I, _I, _P, ctypes.POINTER(_I), _P, _P, _P]),
    "fdllm_kernel_launches": (ctypes.c_longlong, []),
    "fdllm_profile_enable": (_I, [_P, _I]),
    "fdllm_profile_read": (_I, [_P, ctypes.POINTER(ctypes.c_double)]),
    "fdllm_device_error": (_I, [_P, ctypes.POINTER(_I)]),
    "fdllm_device_error_detail": (_I, [_P, _P]),
    "fdllm_wait_selftest": (_I, [_P, ctypes.c_ulonglong, ctypes.POINTER(_I)]),
    "fdllm_workspace_bytes": (ctypes.c_longlong, [_P]),
}

_lib = None
_lock = threading.Lock()


class FdllmError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load (once) and type the library; raises if it is missing or has another ABI version."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(f"{p} is missing: build the sm_100a library with `python -m fast_dllm_relax_b200.build`")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.fdllm_abi_version()
        if ver != 1:
            raise ImportError(f"{p} has ABI version {ver}, expected 1")
        if path is None:
            _lib = lib
        return lib


def check(rc: int) -> None:
    """Raise for a non-zero status: ValueError for invalid arguments (the reference's error type
    for bad cache windows, runtime.py:56-57, 69-70, 258-263), FdllmError otherwise."""
    if rc == FDLLM_OK:
        return
    msg = (load().fdllm_last_error() or b"").decode(errors="replace")
    if rc == FDLLM_ERR_INVALID:
        raise ValueError(msg)
    raise FdllmError(rc, msg)
