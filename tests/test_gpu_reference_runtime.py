"""The reference's OWN runtime driving this library on the GPU.

`fast_dllm_relax.runtime` is imported, unmodified, from the reference package installed under
baseline/_ref (`pip install --no-deps --target baseline/_ref <reference checkout>`; TVM itself is
not installable here, so `import tvm` resolves to this repository's stand-in).  Its
`relax_greedy_generate` and `score_masked_continuation` then call `vm[name](..., params)` on a
VirtualMachine over an artifact directory, which this library serves (vm_backend.B200Backend).

The goldens were recorded by the same runtime.py (its sha256 is checked against the one the
fixtures name) over the oracle's entry points (tiny_*.json / .npz) and over
the reference's own model graph (model_decode.json).  In fp32 this test must reproduce them
exactly: tokens, step statistics and the sequence of entry-point calls, and scoring logits within
1e-4.  Each decode case runs twice: with the runtime's host confidence path
(FAST_DLLM_DISABLE_GPU_CONFIDENCE=1, the path the goldens took) and with the device confidence
entry get_confidence_m{R} the backend offers (runtime.py:131-174), where the calls match after
renaming get_confidence_m{R} to get_logits.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from fast_dllm_relax_b200 import artifacts, install_tvm_shim
from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from tests._oracle_util import PIN_MASK_ID, pin_config, pin_params

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
if not (REF_DIR / "fast_dllm_relax" / "runtime.py").exists():
    pytest.skip("the reference package is not installed under baseline/_ref", allow_module_level=True)

install_tvm_shim()
import tvm  # noqa: E402  (the stand-in)

if str(REF_DIR) not in sys.path:
    sys.path.insert(1, str(REF_DIR))
import fast_dllm_relax.runtime as ref_rt  # noqa: E402


def _scalar(t) -> int:
    return int(t.torch.item()) if hasattr(t, "torch") else int(np.asarray(t.numpy()))


def _calls_key(name: str) -> str:
    return "get_logits" if name.startswith("get_confidence_m") else name


class LoggingVM:
    """vm[name] with every call logged in the goldens' format [name, rows, cache_offset, prefix_len]."""

    def __init__(self, vm):
        self.vm = vm
        self.calls: list[list] = []

    def __getitem__(self, name):
        fn = self.vm[name]  # KeyError for names the artifact lacks, as the runtime's probes expect

        def call(*args):
            if name == "embed":
                self.calls.append([name, int(args[0].shape[0]), -1, -1])
            elif name in ("forward_hidden", "get_logits", "build_prefix_cache") or name.startswith("get_confidence_m"):
                self.calls.append([_calls_key(name), int(args[0].shape[1]), -1, -1])
            else:  # forward_cached / forward_block_partial_rp*: (x, k, v, cache_offset, ShapeTuple([P]), params)
                self.calls.append([name, int(args[0].shape[1]), _scalar(args[3]), int(args[4][0])])
            return fn(*args)
        return call

    def __contains__(self, name):
        return name in self.vm


def _vm(cfg, params_cpu, tmp):
    d = artifacts.write_artifact(tmp, cfg, params_cpu, "float32")
    dev = tvm.cuda(0)
    vm = tvm.relax.VirtualMachine(tvm.runtime.load_module(str(d / artifacts.LIBRARY)), dev)
    with np.load(d / artifacts.PARAMS) as z:  # the runner's parameter load (runners.py:947-966)
        vparams = [tvm.runtime.tensor(z[f"arr_{i}"], device=dev) for i in range(len(params_cpu))]
    spec = ref_rt.CacheSpec(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim, "float32")
    return vm, vparams, dev, spec


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    return _vm(TINY, make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID),
               tmp_path_factory.mktemp("tiny"))


@pytest.fixture(scope="module")
def pinned(tmp_path_factory):
    return _vm(pin_config(), pin_params("float32", PIN_MASK_ID), tmp_path_factory.mktemp("pin"))


def test_installed_runtime_is_the_one_that_recorded_the_goldens(golden_dir):
    golden = json.loads((golden_dir / "tiny_decode.json").read_text())
    got = hashlib.sha256((REF_DIR / "fast_dllm_relax" / "runtime.py").read_bytes()).hexdigest()
    assert got == golden["reference_runtime_sha256"]


def _generate(setup, case, mask_id, cfg, device_confidence: bool):
    vm, vparams, dev, spec = setup
    old = os.environ.get("FAST_DLLM_DISABLE_GPU_CONFIDENCE")
    os.environ["FAST_DLLM_DISABLE_GPU_CONFIDENCE"] = "0" if device_confidence else "1"
    ref_rt._confidence_fn_cache.clear()  # the runtime reads the switch once per VM and row count
    try:
        lvm = LoggingVM(vm)
        toks, stats = ref_rt.relax_greedy_generate(
            lvm, vparams, dev, tvm.get_global_func("vm.builtin.reshape"), None, list(case["prompt"]),
            num_attention_heads=cfg.num_attention_heads, max_new_tokens=case["max_new_tokens"], block_size=32,
            small_block_size=8, threshold=case.get("threshold", 0.9), temperature=0.0, top_p=0.95,
            use_block_cache=case["use_block_cache"], mask_id=mask_id, stop_token=case.get("stop_token"),
            cache_spec=spec, chunked_prefill=case.get("chunked_prefill", False))
    finally:
        if old is None:
            os.environ.pop("FAST_DLLM_DISABLE_GPU_CONFIDENCE", None)
        else:
            os.environ["FAST_DLLM_DISABLE_GPU_CONFIDENCE"] = old
        ref_rt._confidence_fn_cache.clear()
    return [int(t) for t in toks], stats, lvm.calls


def _check(case, got):
    toks, stats, calls = got
    assert toks == case["tokens"]
    assert {k: stats[k] for k in case["stats"]} == case["stats"]
    assert calls == case["calls"]


TINY_CASES = ["cfg0_nocache", "cfg0_blockcache", "short_prompt_stateless", "one_block_prompt", "unaligned_prompt",
              "low_threshold", "chunked_prefill", "stop_token"]


@pytest.mark.parametrize("device_confidence", [False, True], ids=["host-conf", "device-conf"])
@pytest.mark.parametrize("name", TINY_CASES)
def test_reference_runtime_decodes_tiny_goldens(tiny, golden_dir, name, device_confidence):
    golden = json.loads((golden_dir / "tiny_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    _check(case, _generate(tiny, case, golden["mask_id"], TINY, device_confidence))


@pytest.mark.parametrize("name", ["zero_new_tokens", "one_new_token_aligned", "cut_mid_block",
                                  "cut_mid_block_nocache", "stop_on_first_token"])
def test_reference_runtime_decodes_edge_goldens(tiny, golden_dir, name):
    golden = json.loads((golden_dir / "tiny_decode_edges.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    _check(case, _generate(tiny, case, golden["mask_id"], TINY, True))


@pytest.mark.parametrize("device_confidence", [False, True], ids=["host-conf", "device-conf"])
@pytest.mark.parametrize("name", ["aligned_nocache", "aligned_blockcache", "unaligned_blockcache",
                                  "short_prompt_stateless", "chunked_prefill", "stop_token", "low_threshold"])
def test_reference_runtime_decodes_model_graph_goldens(pinned, golden_dir, name, device_confidence):
    """The whole reference stack's runs (its runtime over its own model graph) reproduced with
    this library in place of the compiled module."""
    golden = json.loads((golden_dir / "model_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    _check(case, _generate(pinned, case, golden["mask_id"], pin_config(), device_confidence))


@pytest.mark.parametrize("name", ["ctx70_cont5", "ctx20_cont4", "ctx64_cont40", "ctx96_cont16"])
def test_reference_runtime_scores_tiny_goldens(tiny, golden_dir, name):
    vm, vparams, dev, spec = tiny
    g = np.load(golden_dir / "tiny_scoring.npz")
    ctx, cont = g[f"{name}/context"].tolist(), g[f"{name}/continuation"].tolist()
    logits, _ = ref_rt.score_masked_continuation(
        vm, vparams, dev, tvm.get_global_func("vm.builtin.reshape"), ctx, cont,
        num_attention_heads=TINY.num_attention_heads, block_size=32, mask_id=TINY_MASK_ID, cache_spec=spec,
        eos_token_id=1022)
    np.testing.assert_allclose(np.asarray(logits), g[f"{name}/logits"], rtol=1e-4, atol=1e-4)


def test_reference_runtime_choice_scoring_reuses_the_prefix_cache(tiny, golden_dir):
    """Answer choices against one context (runtime.py:546-548): the runtime reuses and grows the
    library-written cache; logits, log-likelihoods and the call sequence match the goldens."""
    vm, vparams, dev, spec = tiny
    g = np.load(golden_dir / "tiny_choices.npz")
    lvm = LoggingVM(vm)
    cached = None
    for i in range(int(g["n_choices"])):
        ctx, cont = g[f"choice{i}/context"].tolist(), g[f"choice{i}/continuation"].tolist()
        logits, cached = ref_rt.score_masked_continuation(
            lvm, vparams, dev, tvm.get_global_func("vm.builtin.reshape"), ctx, cont,
            num_attention_heads=TINY.num_attention_heads, block_size=32, mask_id=TINY_MASK_ID, cache_spec=spec,
            eos_token_id=1022, cached_prefix=cached)
        np.testing.assert_allclose(np.asarray(logits), g[f"choice{i}/logits"], rtol=1e-4, atol=1e-4)
        lp = torch.log_softmax(torch.from_numpy(np.asarray(logits, dtype=np.float32)), dim=-1)
        ll = float(lp.gather(-1, torch.tensor(cont)[:, None]).sum())
        assert ll == pytest.approx(float(g[f"choice{i}/loglik"]), rel=1e-4, abs=1e-4)
    assert lvm.calls == json.loads(str(g["calls"]))


def test_reference_runtime_scores_model_graph_goldens(pinned, golden_dir):
    vm, vparams, dev, spec = pinned
    golden = json.loads((golden_dir / "model_decode.json").read_text())["scoring"]
    lvm = LoggingVM(vm)
    cached = None
    for ch in golden["choices"]:
        logits, cached = ref_rt.score_masked_continuation(
            lvm, vparams, dev, tvm.get_global_func("vm.builtin.reshape"), golden["context"], ch["continuation"],
            num_attention_heads=pin_config().num_attention_heads, block_size=32, mask_id=PIN_MASK_ID,
            cache_spec=spec, eos_token_id=PIN_MASK_ID - 1, cached_prefix=cached)
        lp = torch.log_softmax(torch.from_numpy(np.asarray(logits, dtype=np.float32)), dim=-1)
        assert float(lp.gather(-1, torch.tensor(ch["continuation"])[:, None]).sum()) == pytest.approx(
            ch["loglik"], rel=1e-4, abs=1e-4)
        assert [int(i) for i in np.asarray(logits).argmax(-1)] == ch["argmax"]
    assert lvm.calls == golden["calls"]
