"""The CPU oracle against the fixtures recorded from the reference's own runtime.py
(tests/golden/make_golden.py): decode tokens, step statistics, the entry-point call sequence,
scoring logits / log-likelihoods, and the bias / shift helpers of model/cuda.py."""

import json

import numpy as np
import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from oracle import decode as od
from oracle.model import build_block_bias
from tests._oracle_util import LoggingOracle, make_oracle, score_choices


@pytest.fixture(scope="module")
def tiny_oracle():
    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    return make_oracle(TINY, params, "float32")


@pytest.fixture(scope="module")
def decode_golden(golden_dir):
    return json.loads((golden_dir / "tiny_decode.json").read_text())


def _case_ids(golden_dir):
    return [c["name"] for c in json.loads((golden_dir / "tiny_decode.json").read_text())["cases"]]


@pytest.mark.parametrize("name", ["cfg0_nocache", "cfg0_blockcache", "short_prompt_stateless",
                                  "one_block_prompt", "unaligned_prompt", "low_threshold",
                                  "chunked_prefill", "stop_token"])
def test_decode_matches_reference_runtime(name, tiny_oracle, decode_golden):
    case = next(c for c in decode_golden["cases"] if c["name"] == name)
    m = LoggingOracle(tiny_oracle)
    toks, stats = od.relax_greedy_generate(
        m, case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
        threshold=case.get("threshold", 0.9), use_block_cache=case["use_block_cache"],
        mask_id=decode_golden["mask_id"], stop_token=case.get("stop_token"),
        chunked_prefill=case.get("chunked_prefill", False))
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert m.calls == case["calls"]


EDGE_CASES = ["zero_new_tokens", "one_new_token_aligned", "cut_mid_block", "cut_mid_block_nocache",
              "stop_on_first_token"]


@pytest.mark.parametrize("name", EDGE_CASES)
def test_decode_edge_cases_match_reference_runtime(name, tiny_oracle, golden_dir):
    """No new tokens, one token after a block-aligned prompt, limits that cut the first block, a
    stop on the first committed token (tests/golden/tiny_decode_edges.json)."""
    golden = json.loads((golden_dir / "tiny_decode_edges.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    m = LoggingOracle(tiny_oracle)
    toks, stats = od.relax_greedy_generate(
        m, case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
        threshold=0.9, use_block_cache=case["use_block_cache"], mask_id=golden["mask_id"],
        stop_token=case.get("stop_token"))
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert m.calls == case["calls"]


@pytest.mark.parametrize("name", ["ctx70_cont5", "ctx20_cont4", "ctx64_cont40", "ctx96_cont16"])
def test_scoring_matches_reference_runtime(name, tiny_oracle, golden_dir):
    g = np.load(golden_dir / "tiny_scoring.npz")
    ctx = g[f"{name}/context"].tolist()
    cont = g[f"{name}/continuation"].tolist()
    logits, _ = od.score_masked_continuation(tiny_oracle, ctx, cont, block_size=32, mask_id=TINY_MASK_ID,
                                             eos_token_id=1022)
    np.testing.assert_array_equal(logits, g[f"{name}/logits"])
    assert od.loglikelihood(logits, cont) == pytest.approx(float(g[f"{name}/loglik"]), abs=0)


def test_choice_scoring_reuses_the_prefix_cache(tiny_oracle, golden_dir):
    """Several answer choices against one context (runtime.py:546-548): the prefix cache is built
    once and reused, grown for a tail longer than a block, and rebuilt for a new context."""
    g = np.load(golden_dir / "tiny_choices.npz")
    m = LoggingOracle(tiny_oracle)
    res = score_choices(m, g, TINY_MASK_ID)
    for i, (logits, cont, _) in enumerate(res):
        np.testing.assert_array_equal(logits, g[f"choice{i}/logits"])
        assert od.loglikelihood(logits, cont) == pytest.approx(float(g[f"choice{i}/loglik"]), abs=0)
    caches = [c for _, _, c in res]
    assert all(c is caches[0] for c in caches[1:4]) and caches[4] is not caches[0]
    assert caches[0].capacity >= 64 + 36  # grown for the 36-row tail
    assert m.calls == json.loads(str(g["calls"]))


def test_bias_helper_matches_reference(golden_dir):
    g = np.load(golden_dir / "helpers.npz")
    for key in [k for k in g.files if k.startswith("bias/")]:
        P, B, bs = key.split("/")[1].split("_")
        got = build_block_bias(int(P), int(B), None if bs == "None" else int(bs)).numpy()
        np.testing.assert_array_equal(got, g[key], err_msg=key)


def test_bias_rejects_bad_sizes():
    with pytest.raises(ValueError):
        build_block_bias(-1, 4)
    with pytest.raises(ValueError):
        build_block_bias(0, 0)
    with pytest.raises(ValueError):
        build_block_bias(0, 4, 0)


def test_confidence_is_first_index_argmax_and_inverse_sum():
    from oracle.model import confidence
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.0], [0.0, 0.0, 0.0, 0.0]])
    ids, maxp = confidence(logits)
    assert ids.tolist() == [1, 0]
    ref = torch.softmax(logits, -1).max(-1).values
    torch.testing.assert_close(maxp, ref, rtol=1e-6, atol=0)
