"""The lm_head + confidence of batched calls (csrc/gemm_tc.cu, tokens-on-M persistent tiles).

From 65 token rows the fused lm_head + confidence (and the log-softmax-gather of the scorer) runs
on the persistent GEMM with 128 tokens on the MMA's M side against pairs of 128-row vocabulary
slabs, so each epilogue thread reduces one token's slab in registers.  Its per-slab partials must
equal, bit for bit, those of the tokens-on-N tiles (FDLLM_TUNING=persist_conf_t=0, and
persist_splitk=0 so that both accumulate each logit over K in the same order), which reduce across
lanes through shared memory: the same first-index maximum and the same sum order.  So the
argmax ids, maxp and log-probabilities of the two plans are compared with torch.equal, and both
against the oracle's reduction of the GPU's own fp32 logits (model/metal.py:316-374 semantics:
first-index argmax, maxp = 1 / sum exp(l - max)).

Vocabularies: 4224 (33 slabs: the last pair holds one slab) and the production 151936 (1187
slabs).  Row counts: 65 (one partial token tile), 128, 200, and 1000 / 1024 (the 32-request
serving step).
"""

import os

import pytest
import torch

from fast_dllm_relax_b200.config import ModelConfig, make_synthetic_params
from oracle.model import confidence as oracle_confidence

pytestmark = pytest.mark.gpu


def _cfg(vocab):
    return ModelConfig(vocab_size=vocab, hidden_size=1536, intermediate_size=8960, num_hidden_layers=1,
                       num_attention_heads=12, num_key_value_heads=2, head_dim=128, context_window_size=4096)


def _dev():
    return torch.device("cuda", 0)


# (first, duplicate) lm_head rows made identical in the 4224-token vocabulary: across slab pairs,
# inside one slab, across the boundary of two pairs, and in the last pair's lone slab
DUPS = [(5, 300), (129, 130), (255, 256), (4100, 4200)]


def _engines(vocab, seed, dups=()):
    from fast_dllm_relax_b200.engine import Engine
    cfg = _cfg(vocab)
    params = make_synthetic_params(cfg, seed=seed, dtype="bfloat16", mask_id=vocab - 3)
    for lo, hi in dups:  # the tied embedding is the lm_head
        params[0][hi] = params[0][lo]
    params = [p.to(_dev()) for p in params]
    old = os.environ.get("FDLLM_TUNING")
    try:
        os.environ["FDLLM_TUNING"] = "persist_conf_t=1"
        on = Engine(cfg, params, dtype="bfloat16")
        # without split K, so that both plans accumulate each logit over K in one order
        os.environ["FDLLM_TUNING"] = "persist_conf_t=0,persist_splitk=0"
        off = Engine(cfg, params, dtype="bfloat16")
    finally:
        if old is None:
            os.environ.pop("FDLLM_TUNING", None)
        else:
            os.environ["FDLLM_TUNING"] = old
    return cfg, on, off


@pytest.fixture(scope="module")
def odd():
    return _engines(4224, 41, DUPS)


@pytest.fixture(scope="module")
def full():
    return _engines(151936, 43)


def _hidden(rows, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn((rows, 1536), generator=g) * scale).to(torch.bfloat16).to(_dev())


def _check(cfg, on, off, rows, seed, scale=1.0, h=None):
    h = _hidden(rows, seed, scale) if h is None else h
    ids, maxp = on.confidence(h)
    ids0, maxp0 = off.confidence(h)
    assert on.device_error() == 0 and off.device_error() == 0
    assert torch.equal(ids.cpu(), ids0.cpu()), f"rows={rows}: ids differ between the two tile plans"
    assert torch.equal(maxp.cpu(), maxp0.cpu()), f"rows={rows}: maxp differs between the two tile plans"
    logits = off.get_logits(h)[0].cpu()  # the same K order as both confidence plans
    rid, rmax = oracle_confidence(logits)
    assert torch.equal(ids.cpu(), rid), f"rows={rows}: ids vs the oracle's reduction of the GPU logits"
    torch.testing.assert_close(maxp.cpu(), rmax, rtol=1e-5, atol=0)
    tg = torch.randint(0, cfg.vocab_size, (rows,), generator=torch.Generator().manual_seed(seed + 1))
    lp = on.token_logprob(h, tg.to(_dev()))
    lp0 = off.token_logprob(h, tg.to(_dev()))
    assert torch.equal(lp.cpu(), lp0.cpu()), f"rows={rows}: log-probabilities differ between the two tile plans"
    ref = torch.log_softmax(logits.double(), -1).gather(-1, tg[:, None].long())[:, 0].float()
    torch.testing.assert_close(lp.cpu().reshape(-1), ref, rtol=1e-5, atol=1e-5)
    return ids.cpu()


@pytest.mark.parametrize("rows", [65, 128, 200, 1000])
def test_odd_slab_count(odd, rows):
    cfg, on, off = odd
    _check(cfg, on, off, rows, rows)


def test_sharp_rows_and_ties(odd):
    """Large logits (maxp near 1, sums dominated by one term), and rows whose maximum is tied: a
    hidden state along a duplicated lm_head row gives its two copies the same largest logit, and the
    argmax must be the first copy's index."""
    cfg, on, off = odd
    _check(cfg, on, off, 130, 7, scale=40.0)
    w = _lm_rows(cfg)
    rows = [40.0 * w[hi] for _, hi in DUPS] * 20  # 80 rows: the persistent plan
    h = torch.stack(rows).to(torch.bfloat16).to(_dev())
    ids = _check(cfg, on, off, h.shape[0], 9, h=h)
    assert ids.tolist() == [lo for lo, _ in DUPS] * 20


def _lm_rows(cfg):
    params = make_synthetic_params(cfg, seed=41, dtype="bfloat16", mask_id=cfg.vocab_size - 3)
    w = params[0].float()
    for lo, hi in DUPS:
        w[hi] = w[lo]
    return w


@pytest.mark.parametrize("rows", [200, 1024])
def test_production_vocabulary(full, rows):
    cfg, on, off = full
    _check(cfg, on, off, rows, 100 + rows)
