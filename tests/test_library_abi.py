"""CPU checks of the C ABI boundary: the library loads without a GPU, exports every function that
include/fdllm_sm100.h declares, and the ctypes signatures cover exactly that set."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from fast_dllm_relax_b200 import _lib

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "fdllm_sm100.h"


def header_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^FDLLM_API\s+[\w\s\*]+?\b(fdllm_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_nine_entry_point_replacements():
    names = header_functions()
    for fn in ("fdllm_embed", "fdllm_forward_hidden", "fdllm_get_logits", "fdllm_build_prefix_cache",
               "fdllm_forward_cached"):
        assert fn in names


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from fast_dllm_relax_b200 import build
        build.build()
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = header_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in header_functions():
        assert hasattr(lib, name)


def test_ctypes_signatures_match_header(lib):
    assert set(_lib.SIGNATURES) == header_functions()


def test_abi_version_without_gpu(lib):
    assert lib.fdllm_abi_version() == 1


def test_build_targets_sm100a_only():
    from fast_dllm_relax_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(ImportError, match="build"):
        _lib.load(tmp_path / "nope.so")


def _zero(t):
    if t in (ctypes.c_int, ctypes.c_int32, ctypes.c_longlong, ctypes.c_ulonglong):
        return 0
    if t in (ctypes.c_double, ctypes.c_float):
        return 0.0
    return None


def test_every_handle_call_rejects_a_null_handle_without_a_gpu(lib):
    """Errors cross the ABI as a status and a message, never as a crash: every entry point that
    takes a handle returns FDLLM_ERR_INVALID for a null one before touching a device."""
    checked = 0
    for name, (res, args) in _lib.SIGNATURES.items():
        if not args or args[0] is not ctypes.c_void_p or name == "fdllm_destroy":
            continue
        rc = getattr(lib, name)(*[_zero(a) for a in args])
        if name == "fdllm_workspace_bytes":
            assert rc == 0
        else:
            assert rc == _lib.FDLLM_ERR_INVALID, name
            assert lib.fdllm_last_error().decode() in ("null handle", "null argument"), name
        checked += 1
    assert checked >= 20
    assert lib.fdllm_destroy(None) == _lib.FDLLM_OK


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_create_without_a_device_returns_a_cuda_error(lib):
    from fast_dllm_relax_b200.config import TINY
    c = _lib.FdllmConfig(TINY.vocab_size, TINY.hidden_size, TINY.intermediate_size, TINY.num_hidden_layers,
                         TINY.num_attention_heads, TINY.num_key_value_heads, TINY.head_dim, TINY.rms_norm_eps,
                         TINY.rope_theta, 1, TINY.bd_size, 4096, 0)
    h = ctypes.c_void_p()
    assert lib.fdllm_create(ctypes.byref(c), 0, ctypes.byref(h)) == _lib.FDLLM_ERR_CUDA
    assert h.value is None
    assert lib.fdllm_last_error()
    with pytest.raises(_lib.FdllmError):
        _lib.check(_lib.FDLLM_ERR_CUDA)


def test_tuning_overrides_are_parsed_before_any_device_use(monkeypatch):
    """FDLLM_TUNING ("key=value,...") sets the per-handle kernel-plan parameters at fdllm_create;
    an unknown key or a value out of range is refused with FDLLM_ERR_INVALID before the device is
    touched, so it fails the same way with or without a GPU."""
    lib = _lib.load()
    c = _lib.FdllmConfig(1024, 256, 512, 2, 4, 2, 64, 1e-6, 1e6, 1, 32, 4096, 1)
    h = ctypes.c_void_p()
    for spec, needle in (("bogus=1", "unknown tuning key"), ("nt_max=96", "out of range"),
                         ("split_max", "without '='"), ("attn_splits=x", "bad tuning value"),
                         ("persist_conf_t=2", "out of range"), ("short_split_max=17", "out of range")):
        monkeypatch.setenv("FDLLM_TUNING", spec)
        assert lib.fdllm_create(ctypes.byref(c), 0, ctypes.byref(h)) == _lib.FDLLM_ERR_INVALID, spec
        assert needle in lib.fdllm_last_error().decode(), spec
    monkeypatch.setenv("FDLLM_TUNING", "nt_max=128,split_max=8,persist_min_rows=0,block_graph=0,persist_conf_t=0")
    rc = lib.fdllm_create(ctypes.byref(c), 0, ctypes.byref(h))
    assert rc != _lib.FDLLM_ERR_INVALID  # a valid spec passes parsing (then needs a device)
    if rc == _lib.FDLLM_OK:
        lib.fdllm_destroy(h)
