"""Artifact directories: the files the reference's Relax runner opens, written and read here.

The reference's runner (fast_dllm_relax/runners.py:570-640, 925-972) loads an artifact directory
holding

    fast_dllm_relax_nn.so               the compiled module          (runners.py:933)
    fast_dllm_relax_nn_params.npz       arr_0 .. arr_{n-1}           (runners.py:934, 947-966)
    fast_dllm_relax_nn_param_names.txt  one parameter name per line  (runners.py:935, 638)
    fast_dllm_relax_nn_dtype.txt        "bfloat16" | "float32" ...   (runners.py:948-949)
    fast_dllm_relax_nn_kv_cache.json    KV-cache contract + dims     (export_utils.py:19-34, runners.py:819-834)

bf16 parameters are stored as their uint16 bit patterns (export_utils.py:54-65; read back by
runners.py:68-76).  This library adds one file, fast_dllm_relax_nn_config.json, with the
architecture (the reference bakes it into the compiled module); for a directory exported by the
reference itself, which lacks it, `read_config` infers the architecture from the parameter
shapes and takes rms_norm_eps / rope_theta / context window from the Qwen2.5 defaults unless
overridden.  `fast_dllm_relax_nn.so` in a directory written here is a copy of this package's
sm_100a library; `tvm.runtime.load_module` of the TVM stand-in only uses its location.
"""

from __future__ import annotations

import dataclasses
import json
import shutil
from pathlib import Path
from typing import Sequence

import numpy as np
import torch

from .config import ModelConfig, param_names, param_shapes

LIBRARY = "fast_dllm_relax_nn.so"
PARAMS = "fast_dllm_relax_nn_params.npz"
PARAM_NAMES = "fast_dllm_relax_nn_param_names.txt"
DTYPE = "fast_dllm_relax_nn_dtype.txt"
KV_CACHE_MANIFEST = "fast_dllm_relax_nn_kv_cache.json"
KV_CACHE_CONTRACT = "inplace_bsnh_v1"
CONFIG = "fast_dllm_relax_nn_config.json"

_DTYPES = ("float32", "bfloat16")


def _to_numpy(t: torch.Tensor, dtype: str) -> np.ndarray:
    t = t.detach().to("cpu")
    if dtype == "bfloat16":
        return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.to(torch.float32).contiguous().numpy()


def write_artifact(out_dir: str | Path, cfg: ModelConfig, params: Sequence[torch.Tensor], dtype: str,
                   library: str | Path | None = None) -> Path:
    """Write an artifact directory the reference's runner (through the TVM stand-in) and
    `fast_dllm_relax_b200.vm_backend` load.  `params` in `param_names(cfg)` order."""
    if dtype not in _DTYPES:
        raise ValueError(f"unsupported artifact dtype {dtype!r}")
    names, shapes = param_names(cfg), param_shapes(cfg)
    if len(params) != len(names):
        raise ValueError(f"expected {len(names)} params, got {len(params)}")
    for i, (p, s) in enumerate(zip(params, shapes)):
        if tuple(p.shape) != s:
            raise ValueError(f"param {i} ({names[i]}): shape {tuple(p.shape)}, expected {s}")
    d = Path(out_dir)
    d.mkdir(parents=True, exist_ok=True)
    np.savez(d / PARAMS, *[_to_numpy(p, dtype) for p in params])
    (d / PARAM_NAMES).write_text("\n".join(names) + "\n", encoding="utf-8")
    (d / DTYPE).write_text(dtype + "\n", encoding="utf-8")
    manifest = {"kv_cache": KV_CACHE_CONTRACT, "num_layers": cfg.num_hidden_layers,
                "num_kv_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim, "dtype": dtype}
    (d / KV_CACHE_MANIFEST).write_text(json.dumps(manifest, indent=2) + "\n", encoding="utf-8")
    (d / CONFIG).write_text(cfg.to_json() + "\n", encoding="utf-8")
    if library is None:
        from . import _lib  # noqa: PLC0415
        library = _lib.LIB_PATH
    library = Path(library)
    if library.exists():
        shutil.copyfile(library, d / LIBRARY)
    else:  # the runner only checks that the file exists; the package's library is what runs
        (d / LIBRARY).write_bytes(b"")
    return d


def read_dtype(d: str | Path) -> str:
    p = Path(d) / DTYPE
    dtype = p.read_text(encoding="utf-8").strip() if p.exists() else "float16"  # runners.py:948-949
    if dtype not in _DTYPES:
        raise ValueError(f"artifact dtype {dtype!r} is not supported by the sm_100a library (float32, bfloat16)")
    return dtype


def read_kv_manifest(d: str | Path) -> dict:
    """The KV-cache manifest; refuses another contract, as runners.py:819-834 does."""
    p = Path(d) / KV_CACHE_MANIFEST
    m = json.loads(p.read_text(encoding="utf-8")) if p.exists() else {}
    if m.get("kv_cache") != KV_CACHE_CONTRACT:
        raise RuntimeError(f"artifact {d} does not use the in-place KV cache "
                           f"(no {KV_CACHE_MANIFEST} with kv_cache={KV_CACHE_CONTRACT!r})")
    return m


def _npz_shapes(d: Path, n: int) -> list[tuple[int, ...]]:
    with np.load(d / PARAMS) as z:
        return [tuple(z[f"arr_{i}"].shape) for i in range(n)]


def read_config(d: str | Path, **overrides) -> ModelConfig:
    """The architecture of an artifact: fast_dllm_relax_nn_config.json when present, else inferred
    from the parameter names and shapes plus the KV manifest (head_dim, KV heads)."""
    d = Path(d)
    if (d / CONFIG).exists():
        cfg = ModelConfig.from_file(d / CONFIG)
        return dataclasses.replace(cfg, **overrides) if overrides else cfg
    names = (d / PARAM_NAMES).read_text(encoding="utf-8").splitlines()
    m = read_kv_manifest(d)
    shapes = _npz_shapes(d, len(names))
    by_name = dict(zip(names, shapes))
    vocab, hidden = by_name["model.embed_tokens.weight"]
    layers = int(m["num_layers"])
    hkv, hd = int(m["num_kv_heads"]), int(m["head_dim"])
    qkv_rows = by_name["model.layers.0.self_attn.qkv_proj.weight"][0]
    inter = by_name["model.layers.0.mlp.gate_up_proj.weight"][0] // 2
    kw = dict(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
              num_attention_heads=qkv_rows // hd - 2 * hkv, num_key_value_heads=hkv, head_dim=hd,
              tie_word_embeddings="lm_head.weight" not in by_name)
    kw.update(overrides)
    return ModelConfig(**kw)


def load_params(d: str | Path, device: torch.device | str, cfg: ModelConfig | None = None) -> list[torch.Tensor]:
    """The artifact's parameters as contiguous torch tensors on `device` (bf16 rebuilt from its
    uint16 bits), in file order, checked against the names and shapes `cfg` implies."""
    d = Path(d)
    dtype = read_dtype(d)
    names = (d / PARAM_NAMES).read_text(encoding="utf-8").splitlines()
    if cfg is not None:
        want = param_names(cfg)
        if names != want:
            raise ValueError("parameter names do not match the configuration's layout")
    out = []
    with np.load(d / PARAMS) as z:
        missing = [f"arr_{i}" for i in range(len(names)) if f"arr_{i}" not in z]
        if missing:
            raise ValueError(f"Parameter archive is missing expected arrays: {', '.join(missing[:10])}")
        for i in range(len(names)):
            a = z[f"arr_{i}"]
            if dtype == "bfloat16":
                t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
            else:
                t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            out.append(t.to(device).contiguous())
    if cfg is not None:
        for i, (t, s) in enumerate(zip(out, param_shapes(cfg))):
            if tuple(t.shape) != s:
                raise ValueError(f"param {i} ({names[i]}): shape {tuple(t.shape)}, expected {s}")
    return out
