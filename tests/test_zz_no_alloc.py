"""fdllm_confidence_static (no device allocation) against fdllm_confidence, through the C ABI.

Collected last (tests/conftest.py sorts test_zz_ files to the end) so it also runs after every
other GPU test has used the library; it passes on its own as well.
"""

import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, ModelConfig, make_synthetic_params

pytestmark = pytest.mark.gpu

MID = ModelConfig(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                  num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=4096)
STATIC_FLOATS = 1 << 20  # the fixed scratch: 4 MiB of fp32


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module", params=[("tiny", "float32"), ("tiny", "bfloat16"), ("mid", "bfloat16")],
                ids=lambda p: f"{p[0]}-{p[1]}")
def engine(request):
    from fast_dllm_relax_b200.engine import Engine
    name, dtype = request.param
    cfg = TINY if name == "tiny" else MID
    params = make_synthetic_params(cfg, seed=3, dtype=dtype, mask_id=TINY_MASK_ID if name == "tiny" else None)
    return Engine(cfg, [p.to(_dev()) for p in params], dtype=dtype)


def _hidden(eng, rows, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((rows, eng.cfg.hidden_size), generator=g).to(eng.dtype).to(_dev())


def test_static_matches_confidence_on_consecutive_calls(engine):
    eng = engine
    for rows, seed in ((33, 1), (7, 2)):  # the second call reads a scratch the first one left dirty
        h = _hidden(eng, rows, seed)
        ids_ref, maxp_ref = eng.confidence(h)
        ids = torch.full((rows,), -1, dtype=torch.int32, device=_dev())
        maxp = torch.full((rows,), -1.0, dtype=torch.float32, device=_dev())
        ws = eng.workspace_bytes()
        eng.confidence_static(h, ids, maxp)
        torch.cuda.synchronize()
        assert eng.workspace_bytes() == ws  # the handle's workspace did not grow
        assert torch.equal(ids.cpu(), ids_ref.cpu()), f"rows={rows}"
        assert torch.equal(maxp.cpu(), maxp_ref.cpu()), f"rows={rows}"


def test_static_rejects_rows_beyond_the_fixed_scratch(engine):
    eng = engine
    max_rows = STATIC_FLOATS // (4 * ((eng.cfg.vocab_size + 127) // 128))
    h = _hidden(eng, max_rows + 1, 5)
    ids = torch.empty(max_rows + 1, dtype=torch.int32, device=_dev())
    maxp = torch.empty(max_rows + 1, dtype=torch.float32, device=_dev())
    with pytest.raises(ValueError, match="fixed 4 MiB scratch"):
        eng.confidence_static(h, ids, maxp)
    # at the limit it runs and still matches the allocating entry point
    h = h[:max_rows]
    eng.confidence_static(h, ids, maxp)
    ids_ref, maxp_ref = eng.confidence(h)
    assert torch.equal(ids[:max_rows].cpu(), ids_ref.cpu())
    assert torch.equal(maxp[:max_rows].cpu(), maxp_ref.cpu())


def test_static_at_the_production_vocabulary():
    """Two layers of the 1.5B shape with its full 151936-token vocabulary (1187 lm_head slabs): the
    fixed scratch holds 220 rows.  A 220-row call equals fdllm_confidence bit for bit, twice in a
    row; a 221-row call is refused before anything is launched."""
    from fast_dllm_relax_b200.engine import Engine
    cfg = ModelConfig(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                      num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=4096)
    params = make_synthetic_params(cfg, seed=4, dtype="bfloat16", mask_id=151665)
    eng = Engine(cfg, [p.to(_dev()) for p in params], dtype="bfloat16")
    max_rows = STATIC_FLOATS // (4 * ((cfg.vocab_size + 127) // 128))
    assert max_rows == 220
    ids = torch.full((max_rows + 1,), -1, dtype=torch.int32, device=_dev())
    maxp = torch.full((max_rows + 1,), -1.0, dtype=torch.float32, device=_dev())
    for seed in (6, 7):
        h = _hidden(eng, max_rows, seed)
        ids_ref, maxp_ref = eng.confidence(h)
        eng.confidence_static(h, ids, maxp)
        torch.cuda.synchronize()
        assert torch.equal(ids[:max_rows].cpu(), ids_ref.cpu())
        assert torch.equal(maxp[:max_rows].cpu(), maxp_ref.cpu())
    with pytest.raises(ValueError, match="rows = 221 exceeds 220"):
        eng.confidence_static(_hidden(eng, max_rows + 1, 8), ids, maxp)
    # outputs the kernel could not write are refused on the host
    with pytest.raises(ValueError, match="ids must be"):
        eng.confidence_static(_hidden(eng, 4, 9), ids.cpu(), maxp)
    with pytest.raises(ValueError, match="at least rows elements"):
        eng.confidence_static(_hidden(eng, 4, 9), ids[:3], maxp)
    assert eng.device_error() == 0
