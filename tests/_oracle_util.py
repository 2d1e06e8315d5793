"""Test helpers: oracle construction and a call-logging proxy (test infrastructure)."""

from __future__ import annotations

import torch

from fast_dllm_relax_b200.config import ModelConfig
from oracle.model import OracleConfig, OracleModel


def oracle_config(cfg: ModelConfig) -> OracleConfig:
    return OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                        intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                        num_attention_heads=cfg.num_attention_heads,
                        num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                        rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                        tie_word_embeddings=cfg.tie_word_embeddings, bd_size=cfg.bd_size)


def make_oracle(cfg: ModelConfig, params, dtype: str) -> OracleModel:
    return OracleModel(oracle_config(cfg), params, dtype)


class LoggingOracle:
    """Wraps an OracleModel and logs calls in the golden call-log format
    [name, rows, cache_offset, prefix_len]."""

    def __init__(self, model: OracleModel):
        self.m = model
        self.cfg = model.cfg
        self.dtype = model.dtype
        self.calls: list[list] = []

    def embed(self, ids):
        self.calls.append(["embed", int(ids.shape[0]), -1, -1])
        return self.m.embed(ids)

    def forward_hidden(self, x, bias):
        self.calls.append(["forward_hidden", int(x.shape[1]), -1, -1])
        return self.m.forward_hidden(x, bias)

    def get_logits(self, h):
        self.calls.append(["get_logits", int(h.shape[1]), -1, -1])
        return self.m.get_logits(h)

    def build_prefix_cache(self, x, bias, k, v):
        self.calls.append(["build_prefix_cache", int(x.shape[1]), -1, -1])
        return self.m.build_prefix_cache(x, bias, k, v)

    def forward_cached(self, x, k, v, off, plen, write_rel=0, attend_rel=None):
        self.calls.append(["forward_cached", int(x.shape[1]), int(off), int(plen)])
        return self.m.forward_cached(x, k, v, off, plen, write_rel, attend_rel)

    def forward_block_partial(self, x, k, v, off, plen, rp):
        self.calls.append([f"forward_block_partial_rp{rp}", int(x.shape[1]), int(off), int(plen)])
        return self.m.forward_block_partial(x, k, v, off, plen, rp)


def score_choices(model, g, mask_id: int) -> list[tuple]:
    """Score the multiple-choice plan recorded in tiny_choices.npz in order with the oracle's
    restatement of runtime.score_masked_continuation, each call handed the (aligned prefix, cache)
    pair the previous call returned (runtime.py:546-548).  Returns (logits, continuation, cache)
    per choice."""
    from oracle import decode as od

    out, cached = [], None
    for i in range(int(g["n_choices"])):
        ctx, cont = g[f"choice{i}/context"].tolist(), g[f"choice{i}/continuation"].tolist()
        logits, cached = od.score_masked_continuation(model, ctx, cont, block_size=32, mask_id=mask_id,
                                                      eos_token_id=1022, cached_prefix=cached)
        out.append((logits, cont, cached[1]))
    return out


# The small architecture the oracle is pinned on against the reference's own model graph
# (tests/golden/make_model_golden.py): head_dim 128, because the reference's cached-attention
# callback hard-codes the 1/sqrt(128) softmax scale (runtime.py:27), and 2 query heads per KV head.
def pin_config():
    from fast_dllm_relax_b200.config import ModelConfig
    return ModelConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=2, num_key_value_heads=1, head_dim=128, rms_norm_eps=1e-6,
                       rope_theta=1e6, context_window_size=4096, tie_word_embeddings=True)


PIN_MASK_ID = 511


def pin_params(dtype: str, mask_id: int | None = None):
    """Weights of the reference-graph pin: N(0, 0.05) matrices and biases (seed 11) and RMSNorm
    weights 1 + N(0, 0.1) (seed 12), so that the norms' weight multiply is exercised too.
    `mask_id`: zero that embedding row (decode runs; see make_synthetic_params)."""
    import torch

    from fast_dllm_relax_b200.config import make_synthetic_params, param_names
    cfg = pin_config()
    g = torch.Generator().manual_seed(12)
    out = []
    for name, p in zip(param_names(cfg), make_synthetic_params(cfg, seed=11, dtype="float32", std=0.05,
                                                               mask_id=mask_id)):
        if name.endswith("norm.weight"):
            p = 1.0 + 0.1 * torch.randn(p.shape, generator=g)
        out.append(p.to({"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype]))
    return out


def assert_close_rel(got, ref, rtol: float, msg: str = "") -> None:
    """Element-wise |got - ref| <= rtol * |ref| + rtol * rms(ref): the stated relative tolerance per
    element, with an absolute floor of rtol times the tensor's RMS for elements near zero, where a
    purely relative bound is undefined (a value that rounds to 1e-5 in one order of summation and
    to 2e-5 in another differs by 100% relative)."""
    import torch

    g, r = got.float().cpu(), ref.float().cpu()
    rms = float(r.pow(2).mean().sqrt())
    torch.testing.assert_close(g, r, rtol=rtol, atol=rtol * rms, msg=lambda m: f"{msg}: {m}" if msg else m)


class ReorderedOracle(OracleModel):
    """The reference graph computed the way the reference's own GPU stack computes it, as a second
    legitimate implementation beside the oracle:

    * every projection's fp32 sum taken in another order: the reduction dimension split into 8
      chunks, each accumulated in fp32, the partial sums added in chunk order (a split-K GEMM
      over 8 CTAs, as cuBLAS runs the reference's skinny projections);
    * attention with flash-attention arithmetic (the reference runtime's cached-attention callback
      calls flash_attn_func, runtime.py:30-48): fp32 scores and row maxima, the unnormalised
      probabilities rounded to the model dtype for the P.V product (fp32 accumulation), divided
      by the fp32 row sum at the end.

    Every other op and every bf16 rounding point is the oracle's.  Its distance from the oracle on
    the same inputs is the noise floor of bf16 arithmetic for that computation: two correct
    implementations of the reference graph disagree by this much."""

    chunks = 8

    def _attend(self, q, k, v, bias):
        cfg = self.cfg
        groups = cfg.num_attention_heads // cfg.num_key_value_heads
        qh = q.permute(1, 0, 2).float()
        kh = k.repeat_interleave(groups, dim=1).permute(1, 2, 0).float()
        vh = v.repeat_interleave(groups, dim=1).permute(1, 0, 2).float()
        s = torch.matmul(qh, kh) * torch.tensor(cfg.head_dim ** -0.5, dtype=torch.float32)
        if bias is not None:
            s = s + bias.float()
        p = torch.exp(s - s.max(dim=-1, keepdim=True).values)
        out = torch.matmul(p.to(self.dtype).float(), vh) / p.sum(dim=-1, keepdim=True)
        return self._r(out).permute(1, 0, 2).reshape(q.shape[0], -1)

    def linear(self, x, w, b=None):
        K = x.shape[-1]
        c = -(-K // self.chunks)
        acc = None
        for k0 in range(0, K, c):
            p = x[:, k0:k0 + c].float() @ w[:, k0:k0 + c].float().t()
            acc = p if acc is None else acc + p
        if b is not None:
            acc = acc + b.float()
        return self._r(acc)


def make_reordered_oracle(cfg: ModelConfig, params, dtype: str) -> ReorderedOracle:
    return ReorderedOracle(oracle_config(cfg), params, dtype)


def bf16_discrepancy(got, ref, rtol: float = 2e-2) -> dict:
    """Relative L2 error, the fraction of elements outside the element-wise bf16 tolerance
    (|d| <= rtol |ref| + rtol rms(ref)) and the largest absolute error."""
    g, r = got.float().cpu(), ref.float().cpu()
    rms = float(r.pow(2).mean().sqrt())
    d = (g - r).abs()
    return {"rel": float((g - r).norm() / r.norm().clamp_min(1e-30)),
            "out": float((d > rtol * r.abs() + rtol * rms).float().mean()),
            "max": float(d.max()), "rms": rms}


def assert_within_bf16_noise(got, ref, noise, msg: str = "", rtol: float = 2e-2, slack: float = 1.5) -> dict:
    """bf16 parity of `got` with the oracle's `ref`, held to the noise floor `noise` (the reordered
    oracle's output on the same inputs; see ReorderedOracle).  The element-wise rtol `rtol` is the
    stated tolerance, but in bf16 two correct summation orders already break it on some elements
    once rounding differences have passed through a few layers, so each measure of the discrepancy
    may exceed the floor's by at most `slack` times (plus a small absolute allowance):

    * relative L2 error    <= slack * floor + 2e-3
    * fraction outside the element-wise tolerance  <= slack * floor + 1e-3
    * largest absolute error  <= slack * floor + rtol * rms(ref)
    """
    a, b = bf16_discrepancy(got, ref, rtol), bf16_discrepancy(noise, ref, rtol)
    line = (f"{msg}: gpu rel {a['rel']:.4f} out {a['out']:.4f} max {a['max']:.4f}; "
            f"reordered-oracle floor rel {b['rel']:.4f} out {b['out']:.4f} max {b['max']:.4f}")
    assert a["rel"] <= slack * b["rel"] + 2e-3, line
    assert a["out"] <= slack * b["out"] + 1e-3, line
    assert a["max"] <= slack * b["max"] + rtol * a["rms"], line
    return {"gpu": a, "floor": b}


def unmask_batch_rule(ids, maxp, desc, threshold: float):
    """fdllm_unmask_batch's rule restated on the host (runtime.py:158-181 shift, 796-805 rule): per
    request (desc row: row0, rows, base, win, masked bits), window row j takes shifted row base + j;
    the masked rows above the threshold are unmasked, else the first most confident masked row.
    Returns int32 [n, 34]: unmasked bits, the last row's unshifted id, the window's tokens."""
    ids, maxp = ids.cpu(), maxp.cpu()
    out = torch.zeros((desc.shape[0], 34), dtype=torch.int32)
    for i, (row0, rows, base, win, bits) in enumerate(desc.cpu().tolist()):
        src = [row0 + (base + j - 1 if base + j > 0 else 0) for j in range(win)]
        toks, conf = [int(ids[r]) for r in src], [float(maxp[r]) for r in src]
        masked = [j for j in range(win) if bits >> j & 1]
        take = [j for j in masked if conf[j] > threshold]
        if not take and masked:
            take = [max(masked, key=lambda j: (conf[j], -j))]
        out[i, 0] = sum(1 << j for j in take)
        out[i, 1] = int(ids[row0 + rows - 1])
        out[i, 2:2 + win] = torch.tensor(toks, dtype=torch.int32)
    return out
