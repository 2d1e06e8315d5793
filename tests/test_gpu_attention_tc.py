"""The tcgen05 attention (csrc/attention_tc.cu; csrc/attention_tc_long.cu for grids of more CTAs
than SMs) against the oracle and against the mma.sync attention it replaces for calls with many
query tokens.

Two engines share one set of MID weights (the 1.5B layer shapes, 2 layers): the default one runs
attention on the tensor cores from 64 query tokens per request; the other has it turned off
(FDLLM_TUNING=attn_tc_min_q=0) and runs the legacy kernel everywhere.  Prefix builds (single and
batched, ragged lengths that leave partial 21-token tiles and partial 64-key tiles), a dense
forward_hidden and a batched cached forward must agree with the oracle at the bf16 noise floor
(tests/_oracle_util.assert_within_bf16_noise) and with each other as two GPU plans of the same
arithmetic.
"""

import pytest
import torch

from fast_dllm_relax_b200.config import ModelConfig, make_synthetic_params
from oracle.model import build_block_bias
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
    params = make_synthetic_params(MID, seed=21, dtype="bfloat16", mask_id=4095)
    dev_params = [p.to(_dev()) for p in params]
    old = os.environ.get("FDLLM_TUNING")
    try:
        os.environ["FDLLM_TUNING"] = ""
        tc = Engine(MID, dev_params, dtype="bfloat16")
        os.environ["FDLLM_TUNING"] = "attn_tc_min_q=0"
        legacy = Engine(MID, dev_params, dtype="bfloat16")
        os.environ["FDLLM_TUNING"] = "attn_lazy_log2=8"
        lazy = Engine(MID, dev_params, dtype="bfloat16")
        os.environ["FDLLM_TUNING"] = "attn_tc_split_min_keys=1024"
        SPLIT.append(Engine(MID, dev_params, dtype="bfloat16"))
    finally:
        if old is None:
            os.environ.pop("FDLLM_TUNING", None)
        else:
            os.environ["FDLLM_TUNING"] = old
    LAZY.append(lazy)
    return tc, legacy, make_oracle(MID, params, "bfloat16"), make_reordered_oracle(MID, params, "bfloat16")


LAZY: list = []  # the engine whose long-prefill kernel moves its exponent base lazily (2^8)
SPLIT: list = []  # the engine that splits long cached key ranges over tcgen05 CTAs (from 1024 keys)


def _act(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((1, n, MID.hidden_size), generator=g).to(torch.bfloat16)


def _consistent(a, b, label):
    d = bf16_discrepancy(a, b)
    assert d["out"] <= 1e-3 and d["rel"] <= 1e-2, f"{label}: {d}"


@pytest.mark.parametrize("P", [64, 96, 200, 1000, 2048])
def test_prefix_build_matches_oracle_and_legacy(engines, P):
    """P = 2048 is 98 query tiles x 2 KV heads = 196 CTAs: the O-in-TMEM kernel of
    attention_tc_long.cu; the others fit one CTA per SM."""
    tc, legacy, orc, alt = engines
    x = _act(P, P)
    caches = []
    for eng in (tc, legacy):
        k, v = eng.new_cache(P + 32)
        eng.build_prefix_cache(x.to(_dev()), None, k, v)
        caches.append((k[:, :, :P].cpu(), v[:, :, :P].cpu()))
    ref = [torch.zeros((2, 1, P + 32, 2, 128), dtype=torch.bfloat16) for _ in range(4)]
    orc.build_prefix_cache(x, build_block_bias(0, P, 32), ref[0], ref[1])
    alt.build_prefix_cache(x, build_block_bias(0, P, 32), ref[2], ref[3])
    for i, name in ((0, "k"), (1, "v")):
        assert_within_bf16_noise(caches[0][i], ref[i][:, :, :P], ref[2 + i][:, :, :P], f"P={P} {name} vs oracle")
        _consistent(caches[0][i], caches[1][i], f"P={P} {name} tcgen05 vs legacy")
    assert tc.device_error() == 0 and legacy.device_error() == 0


def test_forward_hidden_matches_oracle(engines):
    tc, legacy, orc, alt = engines
    T = 160
    x = _act(T, 7)
    bias = build_block_bias(0, T, 32)
    got = tc.forward_hidden(x.to(_dev()), None)
    assert_within_bf16_noise(got, orc.forward_hidden(x, bias), alt.forward_hidden(x, bias), "forward_hidden")
    _consistent(got, legacy.forward_hidden(x.to(_dev()), None), "forward_hidden tcgen05 vs legacy")
    assert tc.device_error() == 0


def test_batched_ragged_prefix_and_cached_forward(engines):
    """Ragged prefixes in one batched build, then one batched cached forward of 96 rows per
    request (the cached path: every row attends the whole window)."""
    tc, legacy, orc, alt = engines
    lens = [70, 130, 64, 200]
    xs = [_act(P, 100 + i) for i, P in enumerate(lens)]
    out = {}
    for name, eng in (("tc", tc), ("legacy", legacy)):
        caches = [eng.new_cache(P + 96) for P in lens]
        eng.build_prefix_cache_batch(torch.cat([x[0] for x in xs]).to(_dev()), caches, lens)
        blocks = [_act(96, 200 + i) for i in range(len(lens))]
        reqs = [dict(k=k, v=v, rows=96, prefix_len=P) for (k, v), P in zip(caches, lens)]
        h = eng.forward_cached_batch(torch.cat([b[0] for b in blocks]).to(_dev()), reqs)
        out[name] = (h.cpu(), [(k.cpu(), v.cpu()) for k, v in caches], blocks)
    h_tc, caches_tc, blocks = out["tc"]
    _consistent(h_tc, out["legacy"][0], "batched cached forward tcgen05 vs legacy")
    o = 0
    for i, P in enumerate(lens):
        kr, vr, ka, va = [torch.zeros((2, 1, P + 96, 2, 128), dtype=torch.bfloat16) for _ in range(4)]
        orc.build_prefix_cache(xs[i], build_block_bias(0, P, 32), kr, vr)
        alt.build_prefix_cache(xs[i], build_block_bias(0, P, 32), ka, va)
        assert_within_bf16_noise(caches_tc[i][0][:, :, :P], kr[:, :, :P], ka[:, :, :P], f"request {i} prefix k")
        hr = orc.forward_cached(blocks[i], kr, vr, P, P)
        ha = alt.forward_cached(blocks[i], ka, va, P, P)
        assert_within_bf16_noise(h_tc[o:o + 96], hr[0], ha[0], f"request {i} cached forward")
        o += 96
    assert tc.device_error() == 0 and legacy.device_error() == 0


def test_long_prefill_with_lazy_base_matches_oracle(engines):
    """attn_lazy_log2=8: the long-prefill kernel moves a row's exponent base only when its maximum
    outgrows it by more than 2^8 -- equal in exact arithmetic, rounded differently; still at the
    bf16 noise floor against the oracle."""
    tc, legacy, orc, alt = engines
    lazy = LAZY[0]
    P = 2048
    x = _act(P, 77)
    k, v = lazy.new_cache(P + 32)
    lazy.build_prefix_cache(x.to(_dev()), None, k, v)
    ref = [torch.zeros((2, 1, P + 32, 2, 128), dtype=torch.bfloat16) for _ in range(4)]
    orc.build_prefix_cache(x, build_block_bias(0, P, 32), ref[0], ref[1])
    alt.build_prefix_cache(x, build_block_bias(0, P, 32), ref[2], ref[3])
    for got, i, name in ((k, 0, "k"), (v, 1, "v")):
        assert_within_bf16_noise(got[:, :, :P].cpu(), ref[i][:, :, :P], ref[2 + i][:, :, :P], f"lazy base {name}")
    assert lazy.device_error() == 0


def _random_caches(P, seed):
    g = torch.Generator().manual_seed(seed)
    shape = (MID.num_hidden_layers, 1, P + 32, MID.num_key_value_heads, MID.head_dim)
    return [(torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16) for _ in range(2)]


def test_cached_key_splits_match_oracle_and_legacy(engines):
    """Long cached key ranges with few CTAs (decode steps over 1100-3000 prefix tokens): the tcgen05
    kernel with the keys split over up to 8 CTAs per (request, KV head, query tile), partials merged
    by log-sum-exp in a second launch -- against the oracle at the bf16 noise floor and against the
    default plan (the mma.sync key-split kernel)."""
    tc, legacy, orc, alt = engines
    split = SPLIT[0]
    lens = [1100, 1500, 2600]
    caches0 = [_random_caches(P, 300 + P) for P in lens]
    x = torch.cat([_act(32, 400 + i)[0] for i in range(len(lens))])
    outs = {}
    for name, eng in (("split", split), ("default", tc)):
        caches = [(k.to(_dev()), v.to(_dev())) for k, v in caches0]
        reqs = [dict(k=k, v=v, rows=32, prefix_len=P) for (k, v), P in zip(caches, lens)]
        outs[name] = eng.forward_cached_batch(x.to(_dev()), reqs).cpu()
        assert eng.device_error() == 0, name
    _consistent(outs["split"], outs["default"], "key-split tcgen05 vs default plan")
    for i, P in enumerate(lens):
        kr, vr = caches0[i][0].clone(), caches0[i][1].clone()
        ka, va = caches0[i][0].clone(), caches0[i][1].clone()
        ref = orc.forward_cached(x[None, 32 * i:32 * i + 32], kr, vr, P, P)
        ref_alt = alt.forward_cached(x[None, 32 * i:32 * i + 32], ka, va, P, P)
        assert_within_bf16_noise(outs["split"][32 * i:32 * i + 32], ref[0], ref_alt[0], f"request {i} (P={P})")
    # one request alone: 4 (KV head, query tile) CTAs, 8 splits
    P = 3000
    k0, v0 = _random_caches(P, 9)
    x1 = _act(32, 10)
    k, v = k0.to(_dev()), v0.to(_dev())
    got = split.forward_cached(x1.to(_dev()), k, v, P, P).cpu()
    ref = orc.forward_cached(x1, k0.clone(), v0.clone(), P, P)
    ref_alt = alt.forward_cached(x1, k0.clone(), v0.clone(), P, P)
    assert_within_bf16_noise(got, ref, ref_alt, "one request, P=3000")
    assert split.device_error() == 0
