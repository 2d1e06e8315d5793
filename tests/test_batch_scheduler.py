"""The batched-serving scheduler (fast_dllm_relax_b200.batch_decode) on the CPU: an engine stand-in
backed by the oracle (test infrastructure) runs the tiny fp32 model, and every request must
reproduce the reference runtime's tokens and statistics (tests/golden/tiny_decode.json), alone
and batched with requests in other states.  This pins the scheduler's host logic -- the window
descriptors it hands to the device unmask (shift base, window, masked rows), how it applies the
decisions, block appends, the stateless first block, batched prefix builds -- independently of
the CUDA kernels; the stand-in's unmask_batch restates the device kernel's rule."""

import json

import pytest
import torch

from fast_dllm_relax_b200.batch_decode import generate_batch
from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from oracle.model import build_block_bias, confidence
from tests._oracle_util import make_oracle, unmask_batch_rule

CASES = ["cfg0_nocache", "cfg0_blockcache", "short_prompt_stateless", "one_block_prompt", "unaligned_prompt",
         "low_threshold", "stop_token"]


class OracleEngine:
    """The Engine calls generate_batch makes, computed by the CPU oracle one request at a time."""

    def __init__(self, cfg, params):
        self.cfg = cfg
        self.device = torch.device("cpu")
        self.m = make_oracle(cfg, params, "float32")
        self.calls = {"prefix_batch": 0, "step_batch": 0}

    def new_cache(self, cap):
        shape = (self.cfg.num_hidden_layers, 1, cap, self.cfg.num_key_value_heads, self.cfg.head_dim)
        return torch.zeros(shape), torch.zeros(shape)

    def embed(self, ids):
        return self.m.embed(ids)

    def build_prefix_cache_batch(self, x, caches, rows):
        self.calls["prefix_batch"] += 1
        o = 0
        for (k, v), r in zip(caches, rows):
            self.m.build_prefix_cache(x[o:o + r][None], build_block_bias(0, r, self.cfg.bd_size), k, v)
            o += r

    def forward_cached_batch(self, x, reqs):
        self.calls["step_batch"] += 1
        outs, o = [], 0
        for r in reqs:
            rows = r["rows"]
            off = r.get("cache_offset", r["prefix_len"] + r.get("write_rel", 0))
            outs.append(self.m.forward_cached(x[o:o + rows][None], r["k"], r["v"], off, r["prefix_len"],
                                              r.get("write_rel", 0), r.get("attend_rel", rows))[0])
            o += rows
        return torch.cat(outs)

    def confidence(self, hidden):
        return confidence(self.m.get_logits(hidden[None])[0])

    def unmask_batch(self, ids, maxp, desc, threshold):
        return unmask_batch_rule(ids, maxp, desc, threshold)

    def forward_hidden(self, x, bias):
        assert bias is None  # the scheduler relies on the implicit block-causal mask
        return self.m.forward_hidden(x, build_block_bias(0, x.shape[1], self.cfg.bd_size))

    def get_logits(self, hidden):
        return self.m.get_logits(hidden)


@pytest.fixture(scope="module")
def engine():
    return OracleEngine(TINY, make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID))


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "tiny_decode.json").read_text())


def _kw(case, golden):
    return dict(max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
                threshold=case.get("threshold", 0.9), use_block_cache=case["use_block_cache"],
                mask_id=golden["mask_id"], stop_token=case.get("stop_token"))


@pytest.mark.parametrize("name", CASES)
def test_scheduler_single_request_matches_reference_runtime(name, engine, golden):
    case = next(c for c in golden["cases"] if c["name"] == name)
    toks, stats = generate_batch(engine, [case["prompt"]], **_kw(case, golden))
    assert toks[0] == case["tokens"]
    assert stats[0] == case["stats"]


def test_scheduler_mixed_batch_matches_reference_runtime(engine, golden):
    """Requests of different lengths share the batched prefix builds and step forwards; each
    reproduces its own golden run (the settings of cfg0_blockcache for all)."""
    case = next(c for c in golden["cases"] if c["name"] == "cfg0_blockcache")
    kw = _kw(case, golden)
    prompts = [c["prompt"] for c in golden["cases"] if c["name"] in CASES]
    alone = [generate_batch(engine, [p], **kw) for p in prompts]
    before = dict(engine.calls)
    toks, stats = generate_batch(engine, prompts, **kw)
    for i, (t1, s1) in enumerate(alone):
        assert toks[i] == t1[0], f"request {i}"
        assert stats[i] == s1[0], f"request {i}"
    assert toks[0] == case["tokens"]
    # batched: far fewer step launches than the requests' steps summed
    steps = engine.calls["step_batch"] - before["step_batch"]
    assert steps < sum(s["block_recomputes"] for s in stats)


@pytest.mark.parametrize("name", ["zero_new_tokens", "one_new_token_aligned", "cut_mid_block",
                                  "cut_mid_block_nocache", "stop_on_first_token"])
def test_scheduler_edge_cases_match_reference_runtime(name, engine, golden_dir):
    """The decode loop's edge cases (tests/golden/tiny_decode_edges.json) through the scheduler."""
    golden = json.loads((golden_dir / "tiny_decode_edges.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    toks, stats = generate_batch(engine, [case["prompt"]], max_new_tokens=case["max_new_tokens"], block_size=32,
                                 small_block_size=8, threshold=0.9, use_block_cache=case["use_block_cache"],
                                 mask_id=golden["mask_id"], stop_token=case.get("stop_token"))
    assert toks[0] == case["tokens"]
    assert stats[0] == case["stats"]


@pytest.mark.parametrize("name", ["aligned_nocache", "aligned_blockcache", "unaligned_blockcache",
                                  "short_prompt_stateless", "stop_token", "low_threshold"])
def test_scheduler_matches_the_whole_reference_stack(name, golden_dir):
    """Decode runs of the reference's runtime driving the reference's own model graph
    (tests/golden/model_decode.json), reproduced by the scheduler over the pinned oracle."""
    from tests._oracle_util import PIN_MASK_ID, pin_config, pin_params
    golden = json.loads((golden_dir / "model_decode.json").read_text())
    case = next(c for c in golden["cases"] if c["name"] == name)
    eng = OracleEngine(pin_config(), pin_params("float32", PIN_MASK_ID))
    toks, stats = generate_batch(eng, [case["prompt"]], max_new_tokens=case["max_new_tokens"], block_size=32,
                                 small_block_size=8, threshold=case.get("threshold", 0.9),
                                 use_block_cache=case["use_block_cache"], mask_id=golden["mask_id"],
                                 stop_token=case.get("stop_token"))
    assert toks[0] == case["tokens"]
    assert stats[0] == case["stats"]
