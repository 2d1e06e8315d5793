"""The CPU oracle against the reference's OWN model graph (fast_dllm_relax/model/cuda.py) executed
op by op (tests/golden/make_model_golden.py, fixture tests/golden/model_graph.npz): embed ->
forward_hidden -> get_logits, build_prefix_cache, forward_cached and forward_block_partial_rp8,
the cached calls through the reference runtime's own packed callbacks (runtime.py:46-73).

fp32: the oracle reproduces the graph to 1e-5 (bit for bit on the dense path; the cached path's
attention differs only in the summation order of the callback's SDPA).  bf16: the eager graph
rounds after every op (a projection's bias is added after the matmul is rounded), whereas the
compiled module fuses some of them, so the bf16 check is a 2e-2 relative error of each tensor and
identical logit argmax, not a per-element bound.

Decode: the reference's runtime.py driving that graph (tests/golden/model_decode.json) and the
oracle's decode loop over the oracle produce the same tokens, statistics and entry-point calls.
"""

import json

import numpy as np
import pytest
import torch

from oracle import decode as od
from oracle.model import build_block_bias
from tests._oracle_util import PIN_MASK_ID, LoggingOracle, make_oracle, pin_config, pin_params

P, B, S, RP = 64, 32, 8, 8


@pytest.fixture(scope="module")
def graph(golden_dir):
    return np.load(golden_dir / "model_graph.npz")


def _get(g, dtype, key) -> torch.Tensor:
    a = g[f"{dtype}/{key}"]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).float()
    return torch.from_numpy(a)


def _oracle_outputs(dtype: str, g) -> dict[str, torch.Tensor]:
    cfg = pin_config()
    m = make_oracle(cfg, pin_params(dtype), dtype)
    x = m.embed(torch.from_numpy(g[f"{dtype}/ids"]))[None]
    x8 = m.embed(torch.from_numpy(g[f"{dtype}/ids8"]))[None]
    h = m.forward_hidden(x, build_block_bias(0, P + B, B))
    out = {"dense/h": h[0, P:], "dense/logits": m.get_logits(h[:, P:])[0]}
    shape = (cfg.num_hidden_layers, 1, P + B, cfg.num_key_value_heads, cfg.head_dim)
    k, v = torch.zeros(shape, dtype=m.dtype), torch.zeros(shape, dtype=m.dtype)
    m.build_prefix_cache(x[:, :P], build_block_bias(0, P, B), k, v)
    out["prefill/k"], out["prefill/v"] = k[-1, 0, :P].clone(), v[-1, 0, :P].clone()
    out["cached/h"] = m.forward_cached(x[:, P:], k, v, P, P)[0]
    out["cached/k"], out["cached/v"] = k[-1, 0, P:P + B].clone(), v[-1, 0, P:P + B].clone()
    out["partial/h"] = m.forward_block_partial(x8, k, v, P + RP, P, RP)[0]
    out["partial/k"], out["partial/v"] = k[-1, 0, P + RP:P + RP + S].clone(), v[-1, 0, P + RP:P + RP + S].clone()
    return {key: t.float() for key, t in out.items()}


KEYS = ["dense/h", "dense/logits", "prefill/k", "prefill/v", "cached/h", "cached/k", "cached/v", "partial/h",
        "partial/k", "partial/v"]


def test_fp32_oracle_reproduces_the_reference_graph(graph):
    mine = _oracle_outputs("float32", graph)
    for key in KEYS:
        torch.testing.assert_close(mine[key], _get(graph, "float32", key), rtol=1e-5, atol=1e-5, msg=key)


def test_bf16_oracle_agrees_with_the_reference_graph(graph):
    mine = _oracle_outputs("bfloat16", graph)
    for key in KEYS:
        ref = _get(graph, "bfloat16", key)
        rel = float((mine[key] - ref).norm() / ref.norm())
        assert rel <= 2e-2, f"{key}: relative error {rel:.4f}"
    assert torch.equal(mine["dense/logits"].argmax(-1), _get(graph, "bfloat16", "dense/logits").argmax(-1))


def test_fixture_records_which_reference_graph(graph):
    assert len(str(graph["model_cuda_sha256"])) == 64


@pytest.mark.parametrize("name", ["aligned_nocache", "aligned_blockcache", "unaligned_blockcache",
                                  "short_prompt_stateless"])
def test_decode_matches_the_whole_reference_stack(name, golden_dir):
    golden = json.loads((golden_dir / "model_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    m = LoggingOracle(make_oracle(pin_config(), pin_params("float32", PIN_MASK_ID), "float32"))
    toks, stats = od.relax_greedy_generate(m, case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32,
                                           small_block_size=8, threshold=0.9, use_block_cache=case["use_block_cache"],
                                           mask_id=golden["mask_id"])
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert m.calls == case["calls"]


def test_choice_scoring_matches_the_whole_reference_stack(golden_dir):
    """runtime.score_masked_continuation over the reference graph, three choices of one context
    with the prefix cache reused (runtime.py:485-588, 546-548)."""
    sc = json.loads((golden_dir / "model_decode.json").read_text())["scoring"]
    m = LoggingOracle(make_oracle(pin_config(), pin_params("float32", PIN_MASK_ID), "float32"))
    cached = None
    for choice in sc["choices"]:
        logits, cached = od.score_masked_continuation(m, sc["context"], choice["continuation"], block_size=32,
                                                      mask_id=PIN_MASK_ID, eos_token_id=PIN_MASK_ID - 1,
                                                      cached_prefix=cached)
        assert od.loglikelihood(logits, choice["continuation"]) == pytest.approx(choice["loglik"], rel=1e-5, abs=1e-5)
        assert [int(i) for i in logits.argmax(-1)] == choice["argmax"]
    assert m.calls == sc["calls"]
