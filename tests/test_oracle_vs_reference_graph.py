"""The CPU oracle against the reference's OWN model graph (fast_dllm_relax/model/cuda.py) executed
op by op (tests/golden/make_model_golden.py, fixture tests/golden/model_graph.npz): embed ->
forward_hidden -> get_logits, build_prefix_cache, forward_cached and forward_block_partial_rp8,
the cached calls through the reference runtime's own packed callbacks (runtime.py:46-73).

Dense path (forward_hidden, get_logits, build_prefix_cache): the oracle reproduces the graph bit
for bit in fp32 and in bf16 (the stand-in rounds a projection once after its bias, as the
reference's cuBLAS bias epilogue does); the bound checked is one rounding step.  Cached path: the
reference's attention callback runs PyTorch SDPA on the CPU here, which sums in another order in
fp32 (3.6e-6 measured, bound 1e-5) and computes in bf16 for bf16 inputs (0.8% relative error
measured, bound 2e-2 per tensor), where the oracle keeps the softmax in fp32 as the model's dense
path does.

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


DENSE = ["dense/h", "dense/logits", "prefill/k", "prefill/v"]
CACHED = ["cached/h", "cached/k", "cached/v", "partial/h", "partial/k", "partial/v"]


def test_fp32_oracle_reproduces_the_reference_graph(graph):
    mine = _oracle_outputs("float32", graph)
    for key in DENSE:
        torch.testing.assert_close(mine[key], _get(graph, "float32", key), rtol=1e-6, atol=1e-6, msg=key)
    for key in CACHED:
        torch.testing.assert_close(mine[key], _get(graph, "float32", key), rtol=1e-5, atol=1e-5, msg=key)


def test_bf16_oracle_reproduces_the_reference_graph(graph):
    mine = _oracle_outputs("bfloat16", graph)
    for key in DENSE:  # within one bf16 rounding step (bit for bit when measured)
        torch.testing.assert_close(mine[key], _get(graph, "bfloat16", key), rtol=2 ** -7, atol=1e-6, msg=key)
    for key in CACHED:
        ref = _get(graph, "bfloat16", key)
        rel = float((mine[key] - ref).norm() / ref.norm())
        assert rel <= 2e-2, f"{key}: relative error {rel:.4f}"
    assert torch.equal(mine["dense/logits"].argmax(-1), _get(graph, "bfloat16", "dense/logits").argmax(-1))


def test_fixture_records_which_reference_graph(graph):
    assert len(str(graph["model_cuda_sha256"])) == 64


@pytest.mark.parametrize("name", ["aligned_nocache", "aligned_blockcache", "unaligned_blockcache",
                                  "short_prompt_stateless", "chunked_prefill", "stop_token", "low_threshold"])
def test_decode_matches_the_whole_reference_stack(name, golden_dir):
    golden = json.loads((golden_dir / "model_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    m = LoggingOracle(make_oracle(pin_config(), pin_params("float32", PIN_MASK_ID), "float32"))
    toks, stats = od.relax_greedy_generate(m, case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32,
                                           small_block_size=8, threshold=case.get("threshold", 0.9),
                                           use_block_cache=case["use_block_cache"], mask_id=golden["mask_id"],
                                           stop_token=case.get("stop_token"),
                                           chunked_prefill=case.get("chunked_prefill", False))
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
