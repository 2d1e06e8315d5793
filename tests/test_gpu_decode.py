"""Native device-resident decode against the fixtures recorded from the reference's runtime.py
(tests/golden/make_golden.py): in fp32 the decoded sequences, step statistics must be identical."""

import json

import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params

pytestmark = pytest.mark.gpu

NATIVE_CASES = ["cfg0_nocache", "cfg0_blockcache", "one_block_prompt", "unaligned_prompt", "low_threshold",
                "stop_token"]


@pytest.fixture(scope="module")
def engine_fp32():
    from fast_dllm_relax_b200.engine import Engine
    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    return Engine(TINY, [p.cuda() for p in params], dtype="float32")


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.loads((golden_dir / "tiny_decode.json").read_text())


@pytest.mark.parametrize("name", NATIVE_CASES)
def test_native_decode_matches_reference_fp32(name, engine_fp32, golden):
    case = next(c for c in golden["cases"] if c["name"] == name)
    toks, stats = engine_fp32.generate(
        case["prompt"], max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
        threshold=case.get("threshold", 0.9), use_block_cache=case["use_block_cache"], mask_id=golden["mask_id"],
        stop_token=case.get("stop_token"))
    assert toks == case["tokens"]
    assert stats == case["stats"]
    assert engine_fp32.device_error() == 0


def test_native_decode_rejects_short_prompt(engine_fp32):
    from fast_dllm_relax_b200._lib import FdllmError
    with pytest.raises(FdllmError, match="stateless"):
        engine_fp32.generate(list(range(20)), max_new_tokens=8, mask_id=TINY_MASK_ID)


def test_native_decode_bf16_runs_and_is_deterministic():
    from fast_dllm_relax_b200.engine import Engine
    params = make_synthetic_params(TINY, seed=0, dtype="bfloat16", mask_id=TINY_MASK_ID)
    eng = Engine(TINY, [p.cuda() for p in params], dtype="bfloat16")
    prompt = list(range(100, 164))
    a = eng.generate(prompt, max_new_tokens=64, use_block_cache=True, mask_id=TINY_MASK_ID)
    b = eng.generate(prompt, max_new_tokens=64, use_block_cache=True, mask_id=TINY_MASK_ID)
    assert a == b
    assert len(a[0]) == 34 and TINY_MASK_ID not in a[0]
    assert eng.device_error() == 0
