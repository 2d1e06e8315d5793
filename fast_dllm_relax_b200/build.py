"""Build the sm_100a library in-tree: fast_dllm_relax_b200/lib/libfdllm_sm100.so.

    python -m fast_dllm_relax_b200.build [--force] [--jobs N]

Each csrc/*.cu is compiled for sm_100a with nvcc (objects in fast_dllm_relax_b200/_build/), then
linked into one shared library with the CUDA runtime linked statically, so the library does not
depend on which libcudart the host process has loaded.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libfdllm_sm100.so"
INCLUDE = PKG.parent / "include"

SOURCES = ["gemm_tc.cu", "gemm_simt.cu", "attention.cu", "attention_tc.cu", "attention_tc_long.cu", "elementwise.cu", "model.cu", "decode.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    extra = list(extra or [])
    stamp = BUILD / "flags"  # objects built with other extra flags are rebuilt
    key = " ".join(extra)
    if not stamp.exists() or stamp.read_text() != key:
        force = True
    hdr = _headers_mtime()
    todo, objs = [], []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda t: _compile(t[0], t[1], extra), todo):
                if verbose and log.strip():
                    print(log, file=sys.stderr)
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    stamp.write_text(key)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / spill / smem usage")
    ap.add_argument("--ktrace", action="store_true",
                    help="compile in the per-launch phase stamps of fdllm_kernel_trace_* (diagnostics; slower)")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else []
    if args.ktrace:
        extra.append("-DFDLLM_KTRACE")
    print(build(force=args.force or args.ptxas_v, jobs=args.jobs, verbose=args.verbose or args.ptxas_v, extra=extra))


if __name__ == "__main__":
    main()
