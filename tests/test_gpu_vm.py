"""The reference's calling convention end to end: an artifact directory loaded through the TVM
stand-in (`tvm.runtime.load_module` + `relax.VirtualMachine` + `vm[name](..., params)`), driven by
the decode loop and scorer of runtime.py (restated in oracle/decode.py, pinned to the reference by
tests/golden), must reproduce the reference runtime's tokens, statistics, call sequence and
scoring logits in fp32.
"""

import json

import numpy as np
import pytest
import torch

from fast_dllm_relax_b200 import artifacts, install_tvm_shim
from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from oracle import decode as od
from oracle.model import confidence as oracle_confidence
from tests._oracle_util import make_oracle, score_choices

install_tvm_shim()
import tvm  # noqa: E402

pytestmark = pytest.mark.gpu


class VmModel:
    """The oracle decode loop's model interface over vm[name] calls with the reference's argument
    conventions (runtime.py:312-343, 413-436): [1, n, H] activations, a 0-d int32 device
    cache_offset, a host ShapeTuple prefix length, caches written in place.  The decode loop keeps
    its caches on the host; each call runs on device copies and writes them back."""

    def __init__(self, vm, params, dev, cfg):
        self.vm, self.params, self.dev, self.cfg = vm, params, dev, cfg
        self.dtype = torch.float32
        self.calls: list[list] = []

    def _t(self, x):
        return tvm.runtime.Tensor(x.to(self.dev.torch_device).contiguous())

    def embed(self, ids):
        self.calls.append(["embed", int(ids.shape[0]), -1, -1])
        tok = tvm.runtime.tensor(np.asarray(ids, dtype="int32"), device=self.dev)
        return self.vm["embed"](tok, self.params).torch.cpu()

    def forward_hidden(self, x, bias):
        self.calls.append(["forward_hidden", int(x.shape[1]), -1, -1])
        return self.vm["forward_hidden"](self._t(x), self._t(bias), self.params).torch.cpu()

    def get_logits(self, h):
        self.calls.append(["get_logits", int(h.shape[1]), -1, -1])
        return self.vm["get_logits"](self._t(h), self.params).torch.cpu()

    def build_prefix_cache(self, x, bias, k, v):
        self.calls.append(["build_prefix_cache", int(x.shape[1]), -1, -1])
        kd, vd = self._t(k), self._t(v)
        rk, rv = self.vm["build_prefix_cache"](self._t(x), self._t(bias), kd, vd, self.params)
        assert rk is kd and rv is vd  # the caches come back as aliases
        k.copy_(kd.torch.cpu())
        v.copy_(vd.torch.cpu())

    def _cached(self, name, x, k, v, off, plen):
        self.calls.append([name, int(x.shape[1]), int(off), int(plen)])
        kd, vd = self._t(k), self._t(v)
        offt = tvm.runtime.tensor(np.asarray(int(off), dtype="int32"), device=self.dev)
        out = self.vm[name](self._t(x), kd, vd, offt, tvm.runtime.ShapeTuple([int(plen)]), self.params)
        k.copy_(kd.torch.cpu())
        v.copy_(vd.torch.cpu())
        return out.torch.cpu()

    def forward_cached(self, x, k, v, off, plen, write_rel=0, attend_rel=None):
        assert write_rel == 0 and attend_rel in (None, int(x.shape[1]))
        return self._cached("forward_cached", x, k, v, off, plen)

    def forward_block_partial(self, x, k, v, off, plen, rp):
        return self._cached(f"forward_block_partial_rp{rp}", x, k, v, off, plen)


@pytest.fixture(scope="module")
def vm_fp32(tmp_path_factory):
    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    d = artifacts.write_artifact(tmp_path_factory.mktemp("artifact"), TINY, params, "float32")
    dev = tvm.cuda(0)
    ex = tvm.runtime.load_module(str(d / artifacts.LIBRARY))
    vm = tvm.relax.VirtualMachine(ex, dev)
    # parameters as the runner loads them (runners.py:947-966)
    with np.load(d / artifacts.PARAMS) as z:
        vparams = [tvm.runtime.tensor(z[f"arr_{i}"], device=dev) for i in range(len(params))]
    return vm, vparams, dev, params


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "tiny_decode.json").read_text())


@pytest.mark.parametrize("name", ["cfg0_nocache", "cfg0_blockcache", "short_prompt_stateless",
                                  "one_block_prompt", "unaligned_prompt", "low_threshold",
                                  "chunked_prefill", "stop_token"])
def test_vm_decode_matches_reference_runtime(name, vm_fp32, golden):
    vm, vparams, dev, _ = vm_fp32
    case = next(c for c in golden["cases"] if c["name"] == name)
    m = VmModel(vm, vparams, dev, TINY)
    toks, stats = od.relax_greedy_generate(
        m, case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
        threshold=case.get("threshold", 0.9), use_block_cache=case["use_block_cache"],
        mask_id=golden["mask_id"], stop_token=case.get("stop_token"),
        chunked_prefill=case.get("chunked_prefill", False))
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert m.calls == case["calls"]


@pytest.mark.parametrize("name", ["ctx70_cont5", "ctx20_cont4", "ctx64_cont40", "ctx96_cont16"])
def test_vm_scoring_matches_reference_runtime(name, vm_fp32, golden_dir):
    vm, vparams, dev, _ = vm_fp32
    g = np.load(golden_dir / "tiny_scoring.npz")
    ctx, cont = g[f"{name}/context"].tolist(), g[f"{name}/continuation"].tolist()
    logits, _ = od.score_masked_continuation(VmModel(vm, vparams, dev, TINY), ctx, cont, block_size=32,
                                             mask_id=TINY_MASK_ID, eos_token_id=1022)
    np.testing.assert_allclose(logits, g[f"{name}/logits"], rtol=1e-4, atol=1e-4)
    assert od.loglikelihood(logits, cont) == pytest.approx(float(g[f"{name}/loglik"]), rel=1e-4, abs=1e-4)


def test_vm_choice_scoring_reuses_the_prefix_cache(vm_fp32, golden_dir):
    """Answer choices scored one after another against one context through vm[name]: one prefix
    build per context, the cached prefix reused (and grown for a 36-row tail), the reference
    runtime's logits and call sequence (runtime.py:546-548)."""
    vm, vparams, dev, _ = vm_fp32
    g = np.load(golden_dir / "tiny_choices.npz")
    m = VmModel(vm, vparams, dev, TINY)
    res = score_choices(m, g, TINY_MASK_ID)
    for i, (logits, cont, _) in enumerate(res):
        np.testing.assert_allclose(logits, g[f"choice{i}/logits"], rtol=1e-4, atol=1e-4)
        assert od.loglikelihood(logits, cont) == pytest.approx(float(g[f"choice{i}/loglik"]), rel=1e-4, abs=1e-4)
    assert m.calls == json.loads(str(g["calls"]))


@pytest.mark.parametrize("rows", [8, 32])
def test_vm_confidence_entry(rows, vm_fp32):
    """get_confidence_m{rows} (runtime.py:131-174): unshifted first-index argmax and
    1 / sum(exp(logit - max)), as [1, rows] tensors."""
    vm, vparams, dev, params = vm_fp32
    orc = make_oracle(TINY, params, "float32")
    h = torch.randn((1, rows, TINY.hidden_size), generator=torch.Generator().manual_seed(rows))
    ht = tvm.runtime.Tensor(h.to(dev.torch_device))
    ids, maxp = vm[f"get_confidence_m{rows}"](ht, vparams)
    assert tuple(ids.shape) == (1, rows) and ids.dtype == "int32" and maxp.dtype == "float32"
    logits = vm["get_logits"](ht, vparams).torch.cpu()
    torch.testing.assert_close(logits, orc.get_logits(h), rtol=1e-4, atol=1e-4)
    ref_ids, ref_maxp = oracle_confidence(logits[0])  # bit-exact argmax given identical logits
    assert torch.equal(ids.torch.cpu()[0], ref_ids)
    torch.testing.assert_close(maxp.torch.cpu()[0], ref_maxp, rtol=1e-5, atol=0)


def test_vm_rejects_unknown_and_static_siblings(vm_fp32):
    vm = vm_fp32[0]
    for name in ("forward_cached_b32", "get_logits_m8", "forward_block_partial_rp4", "no_such_fn"):
        assert name not in vm
    assert "forward_block_partial_rp24" in vm and "get_confidence_m8" in vm


def test_vm_bad_window_raises_value_error(vm_fp32):
    vm, vparams, dev, _ = vm_fp32
    k = tvm.runtime.empty((2, 1, 64, 2, 64), "float32", dev)
    v = tvm.runtime.empty((2, 1, 64, 2, 64), "float32", dev)
    x = tvm.runtime.Tensor(torch.zeros((1, 32, TINY.hidden_size), device=dev.torch_device))
    off = tvm.runtime.tensor(np.asarray(48, dtype="int32"), device=dev)
    with pytest.raises(ValueError):  # rows [48, 80) past the capacity 64 (runtime.py:56-57)
        vm["forward_cached"](x, k, v, off, tvm.runtime.ShapeTuple([48]), vparams)
