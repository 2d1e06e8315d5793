"""The reference's own invariants of the cached entry points, checked on the CPU oracle itself
(the GPU tests check the same properties on the product against this oracle).  The properties are
those of the reference's tests/test_tiny_compile.py:216-329, restated here over OracleModel:

* each cache call writes exactly its own row window of the in-place KV cache (:216-263);
* cached forward == dense block-causal forward on the same rows, and a partial forward of a
  sub-block == the full cached step's rows (:266-292);
* growing a prefix cache keeps its committed rows (:295-310);
* tied get_logits == untied get_logits holding the same array, bit for bit (:313-329).
"""

import dataclasses

import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from oracle import decode as od
from oracle.model import build_block_bias
from tests._oracle_util import make_oracle

SENTINEL = 7.0
TOL = {"float32": dict(rtol=1e-4, atol=1e-4), "bfloat16": dict(rtol=2e-2, atol=2e-2)}


@pytest.fixture(scope="module", params=["float32", "bfloat16"])
def model(request):
    params = make_synthetic_params(TINY, seed=0, dtype=request.param, mask_id=TINY_MASK_ID)
    return make_oracle(TINY, params, request.param), request.param


def _rand(rows: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    return torch.randn((1, rows, TINY.hidden_size), generator=torch.Generator().manual_seed(seed)).to(dtype)


def _cache(m, cap: int):
    shape = (TINY.num_hidden_layers, 1, cap, TINY.num_key_value_heads, TINY.head_dim)
    return torch.full(shape, SENTINEL, dtype=m.dtype), torch.full(shape, SENTINEL, dtype=m.dtype)


def test_cache_calls_write_exactly_their_windows(model):
    m, dt = model
    P, B, S, CAP = 32, TINY.bd_size, TINY.bd_size // 4, 96
    k, v = _cache(m, CAP)
    prefix, block = _rand(P, m.dtype, 1), _rand(B, m.dtype, 2)
    m.build_prefix_cache(prefix, build_block_bias(0, P, B), k, v)
    for c in (k, v):
        assert not (c[:, :, :P] == SENTINEL).any(), "prefill left prefix rows unwritten"
        assert (c[:, :, P:] == SENTINEL).all(), "prefill wrote past the prefix"
    k_prefix = k[:, :, :P].clone()
    m.forward_cached(block, k, v, P, P)
    assert torch.equal(k[:, :, :P], k_prefix), "forward_cached modified the committed prefix"
    assert not (k[:, :, P:P + B] == SENTINEL).any(), "forward_cached left block rows unwritten"
    assert (k[:, :, P + B:] == SENTINEL).all(), "forward_cached wrote past the block"
    # layer 0's block rows equal a dense prefill of prefix + block at those rows
    kd, vd = _cache(m, CAP)
    m.build_prefix_cache(torch.cat([prefix, block], dim=1), build_block_bias(0, P + B, B), kd, vd)
    for c, d in ((k, kd), (v, vd)):
        torch.testing.assert_close(c[0, :, P:P + B].float(), d[0, :, P:P + B].float(), **TOL[dt])
    for rp in (0, 8, 16, 24):
        win = slice(P + rp, P + rp + S)
        k[:, :, win] = SENTINEL
        before = k.clone()
        m.forward_block_partial(_rand(S, m.dtype, 10 + rp), k, v, P + rp, P, rp)
        outside = torch.ones(CAP, dtype=torch.bool)
        outside[win] = False
        assert torch.equal(k[:, :, outside], before[:, :, outside]), f"rp{rp} wrote outside its window"
        assert not (k[:, :, win] == SENTINEL).any(), f"rp{rp} left its window unwritten"


def test_cached_matches_dense_and_partial_matches_full(model):
    m, dt = model
    P, B, S = 64, TINY.bd_size, TINY.bd_size // 4
    seq = _rand(P + B, m.dtype, 3)
    h_dense = m.forward_hidden(seq, build_block_bias(0, P + B, B))[:, P:]
    k, v = _cache(m, P + B)
    m.build_prefix_cache(seq[:, :P], build_block_bias(0, P, B), k, v)
    h_cached = m.forward_cached(seq[:, P:], k, v, P, P)
    torch.testing.assert_close(h_cached.float(), h_dense.float(), **TOL[dt])
    for rp in (0, 8, 16, 24):
        h_part = m.forward_block_partial(seq[:, P + rp:P + rp + S], k, v, P + rp, P, rp)
        torch.testing.assert_close(h_part.float(), h_cached[:, rp:rp + S].float(), **TOL[dt], msg=f"rp{rp}")


def test_growing_a_prefix_cache_keeps_the_prefix(model):
    m, _ = model
    cache = od.allocate_prefix_cache(m, 64)
    m.build_prefix_cache(_rand(64, m.dtype, 4), build_block_bias(0, 64, TINY.bd_size), cache.k, cache.v)
    cache.commit(64)
    before = (cache.k.clone(), cache.v.clone())
    cache.ensure_capacity(160, m)
    assert cache.capacity == 160 and cache.prefix_len == 64
    for old, new in zip(before, (cache.k, cache.v)):
        assert torch.equal(new[:, :, :64], old[:, :, :64])


def test_tied_logits_equal_untied_with_the_same_array():
    tied = make_synthetic_params(TINY, seed=5, dtype="float32")
    untied_cfg = dataclasses.replace(TINY, tie_word_embeddings=False)
    untied = list(tied) + [tied[0].clone()]  # lm_head holding the embedding's array
    mt = make_oracle(TINY, tied, "float32")
    mu = make_oracle(untied_cfg, untied, "float32")
    h = _rand(32, torch.float32, 6)
    assert torch.equal(mt.get_logits(h), mu.get_logits(h))


def test_reordered_oracle_is_the_same_graph():
    """The noise-floor model the bf16 GPU parity tests measure against (split-K sums,
    flash-attention arithmetic) computes the same graph: in fp32 it equals the oracle within fp32
    rounding (1e-5) on the dense, prefill and cached paths."""
    import torch

    from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
    from oracle.model import build_block_bias
    from tests._oracle_util import make_oracle, make_reordered_oracle

    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    a, b = make_oracle(TINY, params, "float32"), make_reordered_oracle(TINY, params, "float32")
    x = torch.randn((1, 96, TINY.hidden_size), generator=torch.Generator().manual_seed(1))
    bias = build_block_bias(0, 96, 32)
    torch.testing.assert_close(b.forward_hidden(x, bias), a.forward_hidden(x, bias), rtol=1e-5, atol=1e-5)
    shape = (TINY.num_hidden_layers, 1, 128, TINY.num_key_value_heads, TINY.head_dim)
    (ka, va), (kb, vb) = [(torch.zeros(shape), torch.zeros(shape)) for _ in range(2)]
    a.build_prefix_cache(x[:, :64], build_block_bias(0, 64, 32), ka, va)
    b.build_prefix_cache(x[:, :64], build_block_bias(0, 64, 32), kb, vb)
    torch.testing.assert_close(kb, ka, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(b.forward_cached(x[:, 64:], kb, vb, 64, 64), a.forward_cached(x[:, 64:], ka, va, 64, 64),
                               rtol=1e-5, atol=1e-5)
