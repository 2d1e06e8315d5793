"""CPU checks of the C ABI boundary: the library loads without a GPU, exports every function that
include/fdllm_sm100.h declares, and the ctypes signatures cover exactly that set."""

import re
import subprocess
from pathlib import Path

import pytest

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
