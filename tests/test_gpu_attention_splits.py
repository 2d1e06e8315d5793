"""The key-split decode attention of csrc/attention.cu at every split count.

A decode-sized cached call splits each (request, 16-token query tile, KV head) over the CTAs of a
thread-block cluster, whose members merge their partial rows by log-sum-exp through distributed
shared memory.  One engine per split count 1..8
(FDLLM_TUNING=attn_splits=S) runs the same cached steps over the same random caches (MID: the
1.5B layer shapes, 2 layers): each must agree with the oracle at the bf16 noise floor
(tests/_oracle_util.assert_within_bf16_noise) and with the unsplit kernel as two GPU plans of the
same arithmetic.  The prefix lengths leave empty splits (100 keys over 8 splits), partial last
tiles and several tiles per split (1000 keys).
"""

import pytest
import torch

from fast_dllm_relax_b200.config import ModelConfig, make_synthetic_params
from tests._oracle_util import assert_within_bf16_noise, bf16_discrepancy, make_oracle, make_reordered_oracle

pytestmark = pytest.mark.gpu

MID = ModelConfig(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                  num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=8192)
SPLITS = range(1, 9)


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def engines():
    import os

    from fast_dllm_relax_b200.engine import Engine
    params = make_synthetic_params(MID, seed=23, dtype="bfloat16", mask_id=4095)
    dev_params = [p.to(_dev()) for p in params]
    old = os.environ.get("FDLLM_TUNING")
    engs = {}
    try:
        for s in SPLITS:
            os.environ["FDLLM_TUNING"] = f"attn_splits={s}"
            engs[s] = Engine(MID, dev_params, dtype="bfloat16")
    finally:
        if old is None:
            os.environ.pop("FDLLM_TUNING", None)
        else:
            os.environ["FDLLM_TUNING"] = old
    return engs, make_oracle(MID, params, "bfloat16"), make_reordered_oracle(MID, params, "bfloat16")


def _caches(P, seed):
    g = torch.Generator().manual_seed(seed)
    shape = (MID.num_hidden_layers, 1, P + 32, MID.num_key_value_heads, MID.head_dim)
    return [(torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16) for _ in range(2)]


def _act(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((1, n, MID.hidden_size), generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("P", [100, 384, 1000])
@pytest.mark.parametrize("rows", [32, 8])
def test_every_split_count_matches_oracle_and_unsplit(engines, P, rows):
    engs, orc, alt = engines
    k0, v0 = _caches(P, P + rows)
    x = _act(rows, 7 * P + rows)
    if rows == 32:
        call = ("forward_cached", (P, P))
    else:
        call = ("forward_block_partial", (P + 8, P, 8))
    kr, vr, ka, va = k0.clone(), v0.clone(), k0.clone(), v0.clone()
    ref = getattr(orc, call[0])(x, kr, vr, *call[1])
    ref_alt = getattr(alt, call[0])(x, ka, va, *call[1])
    outs = {}
    for s, eng in engs.items():
        k, v = k0.to(_dev()), v0.to(_dev())
        outs[s] = getattr(eng, call[0])(x.to(_dev()), k, v, *call[1]).cpu()
        assert eng.device_error() == 0, f"splits={s}"
        assert_within_bf16_noise(outs[s], ref, ref_alt, f"P={P} rows={rows} splits={s} vs oracle")
    for s in SPLITS:
        d = bf16_discrepancy(outs[s], outs[1])
        assert d["out"] <= 1e-3 and d["rel"] <= 1e-2, f"P={P} rows={rows} splits={s} vs unsplit: {d}"
