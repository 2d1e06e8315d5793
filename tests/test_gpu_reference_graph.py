"""The product on the GPU against the reference's OWN model graph and decode stack (fixtures of
tests/golden/make_model_golden.py: model/cuda.py run op by op, and runtime.py driving it), on the
small head_dim-128 architecture with 2 query heads per KV head and random norm weights.

Entry points: fp32 within 1e-4, the stated fp32 tolerance.  bf16 at the noise floor of bf16
arithmetic (tests/_oracle_util.assert_within_bf16_noise: no further from the reference than the
oracle with its fp32 sums reordered), against the reference graph's vectors on the dense path and
against the oracle on the cached path (the recorded cached vectors carry a CPU bf16 attention; see
below).  The native decode driver in fp32: identical tokens and step statistics."""

import json

import numpy as np
import pytest
import torch

from oracle.model import build_block_bias
from tests._oracle_util import (PIN_MASK_ID, assert_within_bf16_noise, make_oracle, make_reordered_oracle,
                                pin_config, pin_params)

pytestmark = pytest.mark.gpu

P, B, S, RP = 64, 32, 8, 8


def _dev():
    return torch.device("cuda", 0)


def _get(g, dtype, key) -> torch.Tensor:
    a = g[f"{dtype}/{key}"]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).float()
    return torch.from_numpy(a)


def _oracle_outputs(g, dtype, make) -> dict:
    """An oracle's outputs on the golden's inputs (CPU), keyed like the golden."""
    orc = make(pin_config(), pin_params(dtype), dtype)
    x = orc.embed(torch.from_numpy(g[f"{dtype}/ids"]))[None]
    x8 = orc.embed(torch.from_numpy(g[f"{dtype}/ids8"]))[None]
    h = orc.forward_hidden(x, build_block_bias(0, P + B, B))
    out = {"dense/h": h[0, P:], "dense/logits": orc.get_logits(h[:, P:])[0]}
    shape = (2, 1, P + B, 1, 128)
    k, v = torch.zeros(shape, dtype=orc.dtype), torch.zeros(shape, dtype=orc.dtype)
    orc.build_prefix_cache(x[:, :P], build_block_bias(0, P, B), k, v)
    out["prefill/k"], out["prefill/v"] = k[-1, 0, :P].clone(), v[-1, 0, :P].clone()
    out["cached/h"] = orc.forward_cached(x[:, P:], k, v, P, P)[0]
    out["cached/k"], out["cached/v"] = k[-1, 0, P:P + B].clone(), v[-1, 0, P:P + B].clone()
    out["partial/h"] = orc.forward_block_partial(x8, k, v, P + RP, P, RP)[0]
    out["partial/k"], out["partial/v"] = k[-1, 0, P + RP:P + RP + S].clone(), v[-1, 0, P + RP:P + RP + S].clone()
    return out


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_entry_points_match_the_reference_graph(dtype, golden_dir):
    from fast_dllm_relax_b200.engine import Engine
    g = np.load(golden_dir / "model_graph.npz")
    cfg = pin_config()
    eng = Engine(cfg, [p.to(_dev()) for p in pin_params(dtype)], dtype=dtype)
    x = eng.embed(torch.from_numpy(g[f"{dtype}/ids"]).to(_dev()))[None]
    x8 = eng.embed(torch.from_numpy(g[f"{dtype}/ids8"]).to(_dev()))[None]
    h = eng.forward_hidden(x, build_block_bias(0, P + B, B).to(_dev()))
    mine = {"dense/h": h[0, P:], "dense/logits": eng.get_logits(h[:, P:].contiguous())[0]}
    k, v = eng.new_cache(P + B)
    eng.build_prefix_cache(x[:, :P].contiguous(), None, k, v)
    mine["prefill/k"], mine["prefill/v"] = k[-1, 0, :P].clone(), v[-1, 0, :P].clone()
    mine["cached/h"] = eng.forward_cached(x[:, P:].contiguous(), k, v, P, P)[0]
    mine["cached/k"], mine["cached/v"] = k[-1, 0, P:P + B].clone(), v[-1, 0, P:P + B].clone()
    mine["partial/h"] = eng.forward_block_partial(x8, k, v, P + RP, P, RP)[0]
    mine["partial/k"], mine["partial/v"] = k[-1, 0, P + RP:P + RP + S].clone(), v[-1, 0, P + RP:P + RP + S].clone()
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    orc = _oracle_outputs(g, dtype, make_oracle) if dtype == "bfloat16" else {}
    noise = _oracle_outputs(g, dtype, make_reordered_oracle) if dtype == "bfloat16" else {}
    for key, val in mine.items():
        got, ref = val.float().cpu(), _get(g, dtype, key)
        if dtype == "float32":
            torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4, msg=key)
        elif key.startswith(("dense/", "prefill/")):
            # the reference graph's own vectors, at the noise floor of bf16 arithmetic: the reordered
            # oracle (each projection's fp32 sum split in two) against the same vectors
            assert_within_bf16_noise(got, ref, noise[key], key)
        else:
            # The recorded bf16 cached-path vectors carry the reference callback's attention as it
            # ran where they were made: PyTorch SDPA on the CPU in bf16 (runtime.py:30-48; flash_attn
            # needs a GPU), 0.8% relative error against fp32 softmax.  Element-wise, the cached path
            # is held to the oracle on the same inputs (its dense path is the reference graph bit
            # for bit, and its cached attention is that same fp32 softmax); against the recorded
            # vectors, to a 2e-2 relative error per tensor.
            assert_within_bf16_noise(got, orc[key], noise[key], f"{key} vs oracle")
            rel = float((got - ref).norm() / ref.norm())
            assert rel <= 2e-2, f"{key}: relative error {rel:.4f} against the reference graph"


@pytest.mark.parametrize("name", ["aligned_nocache", "aligned_blockcache", "unaligned_blockcache", "stop_token",
                                  "low_threshold"])
def test_native_decode_matches_the_whole_reference_stack(name, golden_dir):
    from fast_dllm_relax_b200.engine import Engine
    golden = json.loads((golden_dir / "model_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    eng = Engine(pin_config(), [p.to(_dev()) for p in pin_params("float32", PIN_MASK_ID)], dtype="float32")
    toks, stats = eng.generate(case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32,
                               small_block_size=8, threshold=case.get("threshold", 0.9),
                               use_block_cache=case["use_block_cache"], mask_id=golden["mask_id"],
                               stop_token=case.get("stop_token"))
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert eng.device_error() == 0
