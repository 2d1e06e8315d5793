"""GPU parity of the sm_100a library against the CPU oracle, through the C ABI.

Tolerances: hidden states and logits within rtol 2e-2 in bf16 and 1e-4 in
fp32; argmax tokens and unmask decisions bit-exact given identical logits; decoded sequences
identical in fp32.  The reference's own invariants (tests/test_tiny_compile.py:216-329) are
carried over: sentinel write windows, cached == dense, partial == full rows, tied == untied.
"""

import dataclasses

import numpy as np
import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, ModelConfig, make_synthetic_params
from oracle.model import build_block_bias, confidence as oracle_confidence
from tests._oracle_util import make_oracle

pytestmark = pytest.mark.gpu

# 2 layers of the real 1.5B layer shapes (hidden 1536, 12/2 heads of 128, SwiGLU 8960) with a
# 4096-token vocabulary: exercises split-K, the paired gate/up slabs and head_dim 128.
MID = ModelConfig(vocab_size=4096, hidden_size=1536, intermediate_size=8960, num_hidden_layers=2,
                  num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=4096)

TOL = {"float32": dict(rtol=1e-4, atol=1e-4), "bfloat16": dict(rtol=2e-2, atol=2e-2)}


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module", params=[("tiny", "float32"), ("tiny", "bfloat16"), ("mid", "bfloat16")],
                ids=lambda p: f"{p[0]}-{p[1]}")
def setup(request):
    from fast_dllm_relax_b200.engine import Engine
    name, dtype = request.param
    cfg = TINY if name == "tiny" else MID
    params_cpu = make_synthetic_params(cfg, seed=0, dtype=dtype, mask_id=TINY_MASK_ID if name == "tiny" else None)
    eng = Engine(cfg, [p.to(_dev()) for p in params_cpu], dtype=dtype)
    orc = make_oracle(cfg, params_cpu, dtype)
    return cfg, dtype, eng, orc


def _rand_act(cfg, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((1, n, cfg.hidden_size), generator=g).to({"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype])


def _close(a, b, dtype, msg=""):
    torch.testing.assert_close(a.float().cpu(), b.float().cpu(), msg=msg, **TOL[dtype])


def test_embed_is_exact(setup):
    cfg, dtype, eng, orc = setup
    ids = torch.tensor([0, 5, cfg.vocab_size - 1, 17, 5], dtype=torch.int32)
    out = eng.embed(ids.to(_dev()))
    assert torch.equal(out.cpu(), orc.embed(ids))


def test_get_logits_all_row_counts(setup):
    cfg, dtype, eng, orc = setup
    for rows in (1, 5, 8, 16, 17, 32, 33, 64, 100, 256, 300):
        h = _rand_act(cfg, rows, dtype, rows)
        got = eng.get_logits(h.to(_dev())).cpu()
        ref = orc.get_logits(h)
        _close(got, ref, dtype, f"rows={rows}")
        if dtype == "bfloat16":  # same fp32 accumulate, one rounding: nearly all bits agree
            assert (got == ref).float().mean() > 0.97, f"rows={rows}"


def test_forward_hidden_and_prefill(setup):
    cfg, dtype, eng, orc = setup
    T = 96
    x = _rand_act(cfg, T, dtype, 1)
    bias = build_block_bias(0, T, 32)
    _close(eng.forward_hidden(x.to(_dev()), bias.to(_dev())).cpu(), orc.forward_hidden(x, bias), dtype)
    # the implicit block-causal mask (bias=None) equals the explicit bias
    _close(eng.forward_hidden(x.to(_dev()), None).cpu(), orc.forward_hidden(x, bias), dtype)

    k, v = eng.new_cache(T + 32)
    kr, vr = torch.zeros(k.shape, dtype=k.dtype), torch.zeros(v.shape, dtype=v.dtype)
    eng.build_prefix_cache(x.to(_dev()), bias.to(_dev()), k, v)
    orc.build_prefix_cache(x, bias, kr, vr)
    _close(k[:, :, :T].cpu(), kr[:, :, :T], dtype, "k")
    _close(v[:, :, :T].cpu(), vr[:, :, :T], dtype, "v")


def test_forward_cached_and_partials(setup):
    cfg, dtype, eng, orc = setup
    P = 64
    prefix = _rand_act(cfg, P, dtype, 2)
    block = _rand_act(cfg, 32, dtype, 3)
    bias = build_block_bias(0, P, 32)
    k, v = eng.new_cache(P + 64)
    kr, vr = torch.zeros(k.shape, dtype=k.dtype), torch.zeros(v.shape, dtype=v.dtype)
    eng.build_prefix_cache(prefix.to(_dev()), None, k, v)
    orc.build_prefix_cache(prefix, bias, kr, vr)
    off = torch.tensor(P, dtype=torch.int32, device=_dev())
    h = eng.forward_cached(block.to(_dev()), k, v, off, P)
    hr = orc.forward_cached(block, kr, vr, P, P)
    _close(h.cpu(), hr, dtype, "forward_cached")
    _close(k[:, :, :P + 32].cpu(), kr[:, :, :P + 32], dtype, "k rows")
    for rp in (0, 8, 16, 24):
        small = _rand_act(cfg, 8, dtype, 10 + rp)
        hp = eng.forward_block_partial(small.to(_dev()), k, v, P + rp, P, rp)
        hpr = orc.forward_block_partial(small, kr, vr, P + rp, P, rp)
        _close(hp.cpu(), hpr, dtype, f"rp{rp}")
    _close(eng.get_logits(h).cpu(), orc.get_logits(hr), dtype, "logits")


def test_inplace_cache_write_windows(setup):
    """tests/test_tiny_compile.py:216-261: each call writes exactly its own rows."""
    cfg, dtype, eng, orc = setup
    P, CAP = 32, 96
    k, v = eng.new_cache(CAP)
    k.fill_(7.0)
    v.fill_(7.0)
    eng.build_prefix_cache(_rand_act(cfg, P, dtype, 4).to(_dev()), build_block_bias(0, P, 32).to(_dev()), k, v)
    torch.cuda.synchronize()
    for c in (k, v):
        assert not (c[:, :, :P] == 7.0).any(), "build_prefix_cache left prefix rows unwritten"
        assert (c[:, :, P:] == 7.0).all(), "build_prefix_cache wrote past the prefix"
    kp = k[:, :, :P].clone()
    eng.forward_cached(_rand_act(cfg, 32, dtype, 5).to(_dev()), k, v, P, P)
    torch.cuda.synchronize()
    assert torch.equal(k[:, :, :P], kp), "forward_cached modified the committed prefix"
    assert not (k[:, :, P:P + 32] == 7.0).any()
    assert (k[:, :, P + 32:] == 7.0).all(), "forward_cached wrote past the block"
    for rp in (0, 8, 16, 24):
        win = slice(P + rp, P + rp + 8)
        k[:, :, win] = 7.0
        before = k.clone()
        eng.forward_block_partial(_rand_act(cfg, 8, dtype, 20 + rp).to(_dev()), k, v, P + rp, P, rp)
        torch.cuda.synchronize()
        outside = torch.ones(CAP, dtype=torch.bool)
        outside[win] = False
        assert torch.equal(k[:, :, outside], before[:, :, outside]), f"rp{rp} wrote outside its window"
        assert not (k[:, :, win] == 7.0).any(), f"rp{rp} left its window unwritten"


def test_cached_matches_dense_and_partial_matches_full(setup):
    """tests/test_tiny_compile.py:264-290."""
    cfg, dtype, eng, orc = setup
    P = 64
    seq = _rand_act(cfg, P + 32, dtype, 6).to(_dev())
    h_dense = eng.forward_hidden(seq, build_block_bias(0, P + 32, 32).to(_dev()))[:, P:]
    k, v = eng.new_cache(P + 32)
    eng.build_prefix_cache(seq[:, :P].contiguous(), None, k, v)
    h_cached = eng.forward_cached(seq[:, P:].contiguous(), k, v, P, P)
    _close(h_cached, h_dense, dtype, "cached vs dense")
    for rp in (0, 8, 16, 24):
        hp = eng.forward_block_partial(seq[:, P + rp:P + rp + 8].contiguous(), k, v, P + rp, P, rp)
        _close(hp, h_cached[:, rp:rp + 8], dtype, f"rp{rp}")


def test_confidence_fused_matches_logits(setup):
    cfg, dtype, eng, orc = setup
    for rows in (8, 32):
        h = _rand_act(cfg, rows, dtype, 30 + rows).to(_dev())
        logits = eng.get_logits(h)[0]
        ids, maxp = eng.confidence(h)
        ids2, maxp2 = eng.confidence_from_logits(logits)
        assert torch.equal(ids, ids2)
        torch.testing.assert_close(maxp, maxp2, rtol=2e-5, atol=0)
        rid, rmax = oracle_confidence(logits.cpu())
        assert torch.equal(ids2.cpu(), rid)
        torch.testing.assert_close(maxp2.cpu(), torch.softmax(logits.cpu(), -1).max(-1).values, rtol=1e-5, atol=0)


def test_token_logprob_matches_log_softmax(setup):
    cfg, dtype, eng, orc = setup
    h = _rand_act(cfg, 40, dtype, 7).to(_dev())
    tg = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1))
    got = eng.token_logprob(h, tg)
    ref = torch.log_softmax(eng.get_logits(h)[0].cpu(), -1).gather(-1, tg[:, None])[:, 0]
    torch.testing.assert_close(got.cpu(), ref, rtol=1e-4, atol=1e-4)


def _batched_vs_single(setup, cases, seed0):
    """Run `cases` (prefix, rows, write_rel) one by one and as one batch; compare outputs and caches.
    The caches must be bit-identical where the batch and the single request get the same split-K
    plan: K is split over twice as many CTAs at <= 32 token rows, so a request of up to 32 rows
    alone sums its fp32 partials in another order than inside a batch of more rows, and agrees to
    rounding."""
    cfg, dtype, eng, orc = setup
    reqs, xs, singles = [], [], []
    for i, (P, rows, rp) in enumerate(cases):
        k, v = eng.new_cache(P + 32)
        eng.build_prefix_cache(_rand_act(cfg, P, dtype, seed0 + i).to(_dev()), None, k, v)
        if rows == 8:  # partial steps read the block rows a full step wrote
            eng.forward_cached(_rand_act(cfg, 32, dtype, seed0 + 10 + i).to(_dev()), k, v, P, P)
        x = _rand_act(cfg, rows, dtype, seed0 + 20 + i).to(_dev())
        ks, vs = k.clone(), v.clone()
        single = (eng.forward_cached(x, ks, vs, P + rp, P, rp, 32 if rows == 8 else rows)[0], ks, vs)
        singles.append(single)
        xs.append(x[0])
        reqs.append(dict(k=k, v=v, rows=rows, prefix_len=P, write_rel=rp, attend_rel=32 if rows == 8 else rows))
    out = eng.forward_cached_batch(torch.cat(xs), reqs)
    total = sum(r["rows"] for r in reqs)
    o = 0
    for r, (hs, ks, vs) in zip(reqs, singles):
        _close(out[o:o + r["rows"]], hs, dtype, "batched rows")
        if dtype == "float32" or (total <= 32) == (r["rows"] <= 32):
            assert torch.equal(r["k"], ks) and torch.equal(r["v"], vs)
        else:
            _close(r["k"], ks, dtype, "batched K cache")
            _close(r["v"], vs, dtype, "batched V cache")
        o += r["rows"]


def test_batched_forward_matches_single_requests(setup):
    """80 mixed rows in one batched forward, and 16 rows of partial steps (the <= 32-row plan),
    against the same requests run one at a time."""
    _batched_vs_single(setup, ((32, 32, 0), (64, 8, 8), (96, 32, 0), (32, 8, 24)), 40)
    _batched_vs_single(setup, ((64, 8, 8), (32, 8, 24)), 70)


def test_invalid_windows_raise_value_error(setup):
    cfg, dtype, eng, orc = setup
    k, v = eng.new_cache(64)
    x = _rand_act(cfg, 32, dtype, 8).to(_dev())
    with pytest.raises(ValueError, match="outside cache capacity"):
        eng.forward_cached(x, k, v, 48, 48)
    with pytest.raises(ValueError, match="past the attended rows"):
        eng.forward_cached(x[:, :8].contiguous(), k, v, 40, 16, write_rel=30, attend_rel=32)
    with pytest.raises(ValueError, match="capacity"):
        eng.build_prefix_cache(_rand_act(cfg, 96, dtype, 9).to(_dev()), None, k, v)


def test_tied_logits_equal_untied_with_same_array():
    """tests/test_tiny_compile.py:311-329."""
    from fast_dllm_relax_b200.engine import Engine
    for dtype in ("float32", "bfloat16"):
        params = [p.to(_dev()) for p in make_synthetic_params(TINY, 0, dtype)]
        untied_cfg = dataclasses.replace(TINY, tie_word_embeddings=False)
        e_t = Engine(TINY, params, dtype=dtype)
        e_u = Engine(untied_cfg, params + [params[0].clone()], dtype=dtype)
        h = _rand_act(TINY, 32, dtype, 11).to(_dev())
        assert torch.equal(e_t.get_logits(h), e_u.get_logits(h))


def _unmask_rule(ids, maxp, block, s0, sub_len, partial, mask_id, thr):
    """runtime.py:172-173 shift + 794-805 rule, on host numpy (the oracle for the kernel)."""
    ids = np.asarray(ids)
    maxp = np.asarray(maxp, dtype=np.float32)
    sh_ids = np.concatenate([ids[:1], ids[:-1]])
    sh_p = np.concatenate([maxp[:1], maxp[:-1]])
    bid = sh_ids if partial else sh_ids[s0:s0 + sub_len]
    bp = sh_p if partial else sh_p[s0:s0 + sub_len]
    blk = list(block)
    masked = [j for j in range(sub_len) if blk[s0 + j] == mask_id]
    rows = [r for r in masked if bp[r] > thr]
    if masked and not rows:
        rows = [masked[int(np.argmax([bp[r] for r in masked]))]]
    for r in rows:
        blk[s0 + r] = int(bid[r])
    return blk, rows


def test_unmask_kernel_is_bit_exact():
    from fast_dllm_relax_b200.engine import Engine
    eng = Engine(TINY, [p.to(_dev()) for p in make_synthetic_params(TINY, 0, "float32")], dtype="float32")
    rng = np.random.default_rng(0)
    mask = 1023
    for case in range(300):
        partial = bool(case % 2)
        s0 = int(rng.integers(0, 4)) * 8
        rows = 8 if partial else 32
        ids = rng.integers(0, 1000, rows).astype(np.int32)
        maxp = rng.choice(np.array([0.1, 0.5, 0.9, 0.9000001, 0.95, 0.3], dtype=np.float32), rows)
        if case % 5 == 0:
            maxp[:] = np.float32(0.25)  # all tied: first masked position wins
        block = rng.integers(0, 1000, 32).astype(np.int32)
        block[s0:s0 + 8][rng.random(8) < 0.6] = mask
        if not (block[s0:s0 + 8] == mask).any():
            block[s0 + 3] = mask
        exp_blk, exp_rows = _unmask_rule(ids, maxp, block, s0, 8, partial, mask, 0.9)
        blk_d = torch.from_numpy(block.copy()).to(_dev())
        tok, conf, flag, status = eng.unmask(torch.from_numpy(ids).to(_dev()), torch.from_numpy(maxp).to(_dev()),
                                             blk_d, s0, 8, partial, mask, 0.9)
        assert blk_d.cpu().tolist() == exp_blk, case
        assert [j for j in range(8) if flag[j]] == sorted(exp_rows), case
        assert int(status[1]) == len(exp_rows)
        assert int(status[0]) == sum(1 for j in range(8) if exp_blk[s0 + j] == mask)


def test_bounded_wait_expires_and_context_survives():
    """Failure detection on the GPU: a wait on a flag nothing sets gives up after its limit,
    reports its code, and the context stays usable."""
    from fast_dllm_relax_b200.engine import Engine
    eng = Engine(TINY, [p.to(_dev()) for p in make_synthetic_params(TINY, 0, "float32")], dtype="float32")
    assert eng.wait_selftest(50_000_000) == 7
    assert eng.device_error() == 0
    x = eng.embed(torch.tensor([1, 2, 3], dtype=torch.int32, device=_dev()))
    assert x.shape == (3, TINY.hidden_size)


def test_out_of_range_token_sets_device_error_not_fault():
    from fast_dllm_relax_b200.engine import Engine
    eng = Engine(TINY, [p.to(_dev()) for p in make_synthetic_params(TINY, 0, "float32")], dtype="float32")
    out = eng.embed(torch.tensor([1, TINY.vocab_size + 5], dtype=torch.int32, device=_dev()))
    assert eng.device_error() == 4
    assert torch.equal(out[1].cpu(), torch.zeros(TINY.hidden_size))
    assert eng.device_error() == 0
