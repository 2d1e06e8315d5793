"""Batched decoding (fast_dllm_relax_b200.batch_decode): every request follows runtime.py's loop;
in fp32 each reproduces the reference runtime's tokens and statistics (tests/golden), alone and
when batched with requests in other states (different prompt lengths, stateless first blocks,
partial steps, appends in the same batched forward)."""

import json

import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params

pytestmark = pytest.mark.gpu

CASES = ["cfg0_nocache", "cfg0_blockcache", "short_prompt_stateless", "one_block_prompt", "unaligned_prompt",
         "low_threshold", "stop_token"]


@pytest.fixture(scope="module")
def engine_fp32():
    from fast_dllm_relax_b200.engine import Engine
    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    return Engine(TINY, [p.cuda() for p in params], dtype="float32")


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "tiny_decode.json").read_text())


def _kw(case, golden):
    return dict(max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
                threshold=case.get("threshold", 0.9), use_block_cache=case["use_block_cache"],
                mask_id=golden["mask_id"], stop_token=case.get("stop_token"))


@pytest.mark.parametrize("name", CASES)
def test_single_request_matches_reference_runtime(name, engine_fp32, golden):
    from fast_dllm_relax_b200.batch_decode import generate_batch
    case = next(c for c in golden["cases"] if c["name"] == name)
    toks, stats = generate_batch(engine_fp32, [case["prompt"]], **_kw(case, golden))
    assert toks[0] == case["tokens"]
    assert stats[0] == case["stats"]


def test_mixed_batch_matches_single_requests(engine_fp32, golden):
    """Requests of different lengths run in the same batched forwards (block-cache settings of
    cfg0_blockcache): each result equals the request run alone."""
    from fast_dllm_relax_b200.batch_decode import generate_batch
    case = next(c for c in golden["cases"] if c["name"] == "cfg0_blockcache")
    kw = _kw(case, golden)
    prompts = [c["prompt"] for c in golden["cases"] if c["name"] in CASES]  # 64, 20, 32, 45 ... tokens
    alone = [generate_batch(engine_fp32, [p], **kw) for p in prompts]
    toks, stats = generate_batch(engine_fp32, prompts, **kw)
    for i, (t1, s1) in enumerate(alone):
        assert toks[i] == t1[0], f"request {i}"
        assert stats[i] == s1[0], f"request {i}"
    assert toks[0] == case["tokens"]


def test_bf16_batch_runs_and_is_deterministic():
    from fast_dllm_relax_b200.batch_decode import generate_batch
    from fast_dllm_relax_b200.config import ModelConfig
    from fast_dllm_relax_b200.engine import Engine
    mid = ModelConfig(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                      num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=4096)
    params = make_synthetic_params(mid, seed=2, dtype="bfloat16", mask_id=4095)
    eng = Engine(mid, [p.cuda() for p in params], dtype="bfloat16")
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 4000, (n,), generator=g).tolist() for n in (64, 96, 40, 128, 33, 70, 64, 100)]
    kw = dict(max_new_tokens=40, mask_id=4095, use_block_cache=True)
    a, sa = generate_batch(eng, prompts, **kw)
    b, sb = generate_batch(eng, prompts, **kw)
    assert a == b and sa == sb
    assert all(len(t) > 0 and 4095 not in t for t in a)
    assert eng.device_error() == 0


def test_unmask_batch_kernel_is_bit_exact():
    """fdllm_unmask_batch against the host restatement of the rule on 200 random batched steps:
    full and partial windows, append rows (win 0), ties, confidences at and around the threshold."""
    from fast_dllm_relax_b200.config import TINY, make_synthetic_params
    from fast_dllm_relax_b200.engine import Engine
    from tests._oracle_util import unmask_batch_rule
    eng = Engine(TINY, [p.cuda() for p in make_synthetic_params(TINY, 0, "float32")], dtype="float32")
    g = torch.Generator().manual_seed(5)
    for case in range(200):
        n = int(torch.randint(1, 40, (1,), generator=g))
        desc, o = [], 0
        for _ in range(n):
            rows = [8, 32][int(torch.randint(0, 2, (1,), generator=g))]
            win = 0 if int(torch.randint(0, 6, (1,), generator=g)) == 0 else 8
            base = 0 if rows == 8 else 8 * int(torch.randint(0, 4, (1,), generator=g))
            bits = int(torch.randint(0, 256, (1,), generator=g)) if win else 0
            desc.append((o, rows, base, win, bits))
            o += rows
        ids = torch.randint(0, 1000, (o,), generator=g, dtype=torch.int32)
        levels = torch.tensor([0.1, 0.5, 0.9, 0.9000001, 0.95, 0.3], dtype=torch.float32)
        maxp = levels[torch.randint(0, len(levels), (o,), generator=g)]
        d = torch.tensor(desc, dtype=torch.int32)
        got = eng.unmask_batch(ids.cuda(), maxp.cuda(), d.cuda(), 0.9).cpu()
        ref = unmask_batch_rule(ids, maxp, d, 0.9)
        for i, (_, _, _, win, _) in enumerate(desc):
            assert torch.equal(got[i, :2 + win], ref[i, :2 + win]), (case, i)
    assert eng.device_error() == 0
