"""Artifact directories and the TVM stand-in's module loading, on the CPU.

The file set, the bf16-as-uint16 storage and the KV-cache manifest follow the reference's export
and runner (fast_dllm_relax/export_utils.py:19-65, runners.py:68-76, 819-834, 925-972).
"""

import dataclasses
import json

import numpy as np
import pytest
import torch

from fast_dllm_relax_b200 import artifacts, install_tvm_shim
from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params, param_names

install_tvm_shim()
import tvm  # noqa: E402


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_write_then_load_round_trip(tmp_path, dtype):
    params = make_synthetic_params(TINY, seed=0, dtype=dtype, mask_id=TINY_MASK_ID)
    d = artifacts.write_artifact(tmp_path / "a", TINY, params, dtype)
    for f in (artifacts.LIBRARY, artifacts.PARAMS, artifacts.PARAM_NAMES, artifacts.DTYPE,
              artifacts.KV_CACHE_MANIFEST, artifacts.CONFIG):
        assert (d / f).exists(), f
    assert (d / artifacts.PARAM_NAMES).read_text().splitlines() == param_names(TINY)
    assert artifacts.read_dtype(d) == dtype
    assert artifacts.read_config(d) == TINY
    back = artifacts.load_params(d, "cpu", TINY)
    assert len(back) == len(params)
    for a, b in zip(params, back):
        assert a.dtype == b.dtype and torch.equal(a, b)
    with np.load(d / artifacts.PARAMS) as z:  # bf16 travels as its uint16 bit pattern
        assert z["arr_0"].dtype == (np.uint16 if dtype == "bfloat16" else np.float32)


def test_manifest_matches_reference_contract(tmp_path):
    d = artifacts.write_artifact(tmp_path, TINY, make_synthetic_params(TINY, seed=0), "float32")
    m = json.loads((d / artifacts.KV_CACHE_MANIFEST).read_text())
    assert m == {"kv_cache": "inplace_bsnh_v1", "num_layers": 2, "num_kv_heads": 2, "head_dim": 64,
                 "dtype": "float32"}
    (d / artifacts.KV_CACHE_MANIFEST).write_text(json.dumps(dict(m, kv_cache="stacked_bhsd")))
    with pytest.raises(RuntimeError, match="in-place KV cache"):
        artifacts.read_kv_manifest(d)


def test_config_inferred_without_config_file(tmp_path):
    """A directory the reference exported has no config file: the architecture comes from the
    parameter shapes and the manifest; eps / theta take the Qwen2.5 defaults or overrides."""
    untied = dataclasses.replace(TINY, tie_word_embeddings=False, context_window_size=32768)
    d = artifacts.write_artifact(tmp_path, untied, make_synthetic_params(untied, seed=0), "float32")
    (d / artifacts.CONFIG).unlink()
    assert artifacts.read_config(d) == untied
    assert artifacts.read_config(d, rope_theta=1e4).rope_theta == 1e4


def test_missing_array_and_bad_dtype_are_refused(tmp_path):
    d = artifacts.write_artifact(tmp_path, TINY, make_synthetic_params(TINY, seed=0), "float32")
    (d / artifacts.DTYPE).write_text("float16\n")
    with pytest.raises(ValueError, match="not supported"):
        artifacts.read_dtype(d)
    (d / artifacts.DTYPE).write_text("float32\n")
    with np.load(d / artifacts.PARAMS) as z:
        arrs = {k: z[k] for k in z.files if k != "arr_3"}
    np.savez(d / artifacts.PARAMS, **arrs)
    with pytest.raises(ValueError, match="arr_3"):
        artifacts.load_params(d, "cpu")


def test_load_module_through_the_stand_in(tmp_path):
    d = artifacts.write_artifact(tmp_path, TINY, make_synthetic_params(TINY, seed=0), "float32")
    assert getattr(tvm, "IS_FDLLM_SHIM", False)
    ex = tvm.runtime.load_module(str(d / artifacts.LIBRARY))
    assert ex.cfg == TINY and ex.dtype == "float32"
    # no CPU path: a VirtualMachine on the host refuses instead of falling back
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        tvm.relax.VirtualMachine(ex, tvm.cpu(0))


def test_runner_style_param_loading(tmp_path):
    """runners.py:68-76: bf16 params rebuilt by empty(..., "bfloat16").copyfrom(uint16 array)."""
    params = make_synthetic_params(TINY, seed=0, dtype="bfloat16")
    d = artifacts.write_artifact(tmp_path, TINY, params, "bfloat16")
    with np.load(d / artifacts.PARAMS) as z:
        arr = z["arr_1"]
        t = tvm.runtime.empty(arr.shape, "bfloat16", tvm.cpu(0)).copyfrom(arr)
    assert torch.equal(t.torch, params[1])


def test_writer_matches_the_reference_exporter_byte_for_byte(tmp_path, golden_dir):
    """tests/golden/artifact_format.json describes what the reference's own exporter writes for
    the tiny bf16 weights (export_utils.remap_params fusing q/k/v and gate/up, np.savez in the
    model's parameter order, the names, the dtype, write_kv_cache_manifest).  This package's
    writer produces the same files, texts and arrays; the loader reads them back without the
    config file the reference does not write."""
    import hashlib
    import json

    import numpy as np

    want = json.loads((golden_dir / "artifact_format.json").read_text())
    params = make_synthetic_params(TINY, seed=0, dtype="bfloat16", mask_id=TINY_MASK_ID)
    d = artifacts.write_artifact(tmp_path / "a", TINY, params, "bfloat16", library=tmp_path / "missing.so")
    for f in ("fast_dllm_relax_nn_kv_cache.json", "fast_dllm_relax_nn_param_names.txt", "fast_dllm_relax_nn_dtype.txt"):
        assert (d / f).read_text(encoding="utf-8") == want[f], f
    with np.load(d / artifacts.PARAMS) as z:
        got = [dict(name=k, shape=list(z[k].shape), dtype=str(z[k].dtype),
                    sha256=hashlib.sha256(np.ascontiguousarray(z[k]).tobytes()).hexdigest()) for k in z.files]
    assert got == want["arrays"]
    assert set(want["files"]) <= {p.name for p in d.iterdir()}
    (d / artifacts.CONFIG).unlink()  # as the reference exports it
    cfg = artifacts.read_config(d)
    assert (cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads,
            cfg.head_dim, cfg.vocab_size) == (2, 256, 4, 2, 64, 1024)
    loaded = artifacts.load_params(d, "cpu", cfg)
    assert all(torch.equal(a, b) for a, b in zip(loaded, params))


def test_param_lists_match_the_reference_model_tied_and_untied(golden_dir):
    """param_names / param_shapes against the parameter list the reference's own model class
    exports (tests/golden/artifact_format.json), for a tied and an untied lm_head."""
    from fast_dllm_relax_b200.config import param_shapes

    want = json.loads((golden_dir / "artifact_format.json").read_text())["param_lists"]
    for tied in (True, False):
        cfg = dataclasses.replace(TINY, tie_word_embeddings=tied)
        got = [[n, list(s)] for n, s in zip(param_names(cfg), param_shapes(cfg))]
        assert got == want["tied" if tied else "untied"]
