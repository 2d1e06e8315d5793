"""Projection plans of large calls (csrc/model.cu run_gemm, csrc/gemm_tc.cu).

A 1024-row batched cached step (32 requests x 32 rows, the configs[2] serving step) runs its
projections on the persistent GEMM by default.  Each alternative plan must match the plain
persistent plan as two GPU plans of the same arithmetic, and the oracle at the bf16 noise floor
(tests/_oracle_util.assert_within_bf16_noise).  The plans (FDLLM_TUNING):
  persist_nt96=1    few-slab projections (o, down: 12 weight slabs) on 96-token tiles;
  persist_splitk=2  the long-K projection (down: K = 8960) on 256-token tiles with K split 3 ways
                    (fp32 partials merged in split order by the tile's last split);
  short_k_nt=64     short-K projections (qkv, o: K = 1536) on the per-tile kernel, 64-token tiles;
  persist_merge_all=1  with the split plan, every split of a tile waits for the others and merges
                    every third 32-column chunk (instead of the last split merging them all);
  persist_l2_ahead=8  the persistent producer prefetches weight k blocks 8 ahead into L2.
MID: the 1.5B layer shapes, 2 layers.
"""

import pytest
import torch

from fast_dllm_relax_b200.config import ModelConfig, make_synthetic_params
from tests._oracle_util import assert_within_bf16_noise, bf16_discrepancy, make_oracle, make_reordered_oracle

pytestmark = pytest.mark.gpu

MID = ModelConfig(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                  num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=8192)


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def engines():
    import os

    from fast_dllm_relax_b200.engine import Engine
    params = make_synthetic_params(MID, seed=31, dtype="bfloat16", mask_id=4095)
    dev_params = [p.to(_dev()) for p in params]
    old = os.environ.get("FDLLM_TUNING")
    engs = {}
    try:
        for spec in PLANS:
            os.environ["FDLLM_TUNING"] = spec
            engs[spec] = Engine(MID, dev_params, dtype="bfloat16")
    finally:
        if old is None:
            os.environ.pop("FDLLM_TUNING", None)
        else:
            os.environ["FDLLM_TUNING"] = old
    return engs, make_oracle(MID, params, "bfloat16"), make_reordered_oracle(MID, params, "bfloat16")


PLANS = ["persist_nt96=0,persist_splitk=0,short_k_nt=0,persist_merge_all=0", "persist_nt96=1", "persist_splitk=2",
         "short_k_nt=64", "persist_splitk=2,persist_merge_all=1", "persist_l2_ahead=8"]


@pytest.mark.parametrize("plan", PLANS[1:])
@pytest.mark.parametrize("n_req", [32, 31])
def test_batched_step_plans(engines, plan, n_req):
    """32 x 32 rows (11 tiles of 96, the last one partial) and 31 x 32 rows; caches of different
    prefix lengths."""
    engs, orc, alt = engines
    base, nt96 = engs[PLANS[0]], engs[plan]
    g = torch.Generator().manual_seed(n_req)
    lens = [64 + 16 * i for i in range(n_req)]
    caches0 = []
    for P in lens:
        shape = (MID.num_hidden_layers, 1, P + 32, MID.num_key_value_heads, MID.head_dim)
        caches0.append([(torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16) for _ in range(2)])
    x = torch.randn((n_req * 32, MID.hidden_size), generator=g).to(torch.bfloat16)
    outs = []
    for eng in (base, nt96):
        caches = [(k.to(_dev()), v.to(_dev())) for k, v in caches0]
        reqs = [dict(k=k, v=v, rows=32, prefix_len=P) for (k, v), P in zip(caches, lens)]
        h = eng.forward_cached_batch(x.to(_dev()), reqs).cpu()
        assert eng.device_error() == 0
        outs.append((h, [(k.cpu(), v.cpu()) for k, v in caches]))
    d = bf16_discrepancy(outs[1][0], outs[0][0])
    assert d["out"] <= 1e-3 and d["rel"] <= 1e-2, f"{plan} vs the plain persistent plan: {d}"
    for i in (0, n_req - 1):
        P = lens[i]
        kr, vr = caches0[i][0].clone(), caches0[i][1].clone()
        ka, va = caches0[i][0].clone(), caches0[i][1].clone()
        ref = orc.forward_cached(x[None, 32 * i:32 * i + 32], kr, vr, P, P)
        ref_alt = alt.forward_cached(x[None, 32 * i:32 * i + 32], ka, va, P, P)
        assert_within_bf16_noise(outs[1][0][32 * i:32 * i + 32], ref[0], ref_alt[0], f"{plan} request {i} vs oracle")
        assert_within_bf16_noise(outs[1][1][i][0][:, :, P:P + 32], kr[:, :, P:P + 32], ka[:, :, P:P + 32],
                                 f"{plan} request {i} K rows vs oracle")
