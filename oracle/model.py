"""CPU oracle: a PyTorch restatement of the reference's Fast-dLLM v2 Relax graph.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module; only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of `bench.py` use it,
always as the checker or the timed CPU baseline, never as the thing measured on the GPU.

Every op follows the precision order of `fast_dllm_relax/model/cuda.py` in the reference
(longthangvu/fast-dllm-relax), where each bf16 op is computed in fp32 and rounded back to the
model dtype (TVM's bf16 legalisation; PyTorch's opmath convention):

* RMSNorm            model/cuda.py:269-275  fp32 mean-square, rsqrt, cast, THEN x weight
* RoPE tables        model/cuda.py:226-238 (prefill) and 278-300 (offset): inv_freq = exp(-ln(theta)*i/half)
* RoPE apply         model/cuda.py:241-246, 303-316: q*cos + rotate_half(q)*sin, cos/sin cast first
* SiLU               model/cuda.py:319-328: fp32 x*sigmoid(x), cast
* MLP                model/cuda.py:343-347: split(gate_up) -> silu(gate)*up -> down
* dense attention    model/cuda.py:401-430, 432-466: fp32 QK^T * scale + bias, fp32 softmax, fp32 PV
* cached attention   model/cuda.py:468-529 with the callback runtime.py:63-73: write K/V rows
                     [P+write_rel, +rows), attend rows [0, P+attend_rel), no mask
* layer / model      model/cuda.py:545-579, 604-666
* entry points       model/cuda.py:698-788
* get_logits         model/cuda.py:704-711: matmul in the model dtype, then cast to fp32

Documented deviation: the cached attention uses head_dim**-0.5 (as the dense path,
model/cuda.py:362) rather than the callback's hard-coded 1/sqrt(128) (runtime.py:28); the two
agree for the 1.5B model (head_dim 128) and only the former keeps cached == dense for head_dim 64.

Parity of this restatement is pinned against the reference's own model graph: model/cuda.py
executed op by op through an eager stand-in of TVM's nn frontend, with the reference runtime's
packed callbacks for the cached calls (tests/golden/make_model_golden.py).  This module reproduces
its dense path bit for bit in fp32 and bf16, and its cached path within 1e-5 in fp32 (2e-2
relative in bf16, where the callback's CPU attention computes in bf16;
tests/test_oracle_vs_reference_graph.py).  It also
satisfies the reference's invariants (cached == dense, partial == full rows, tied == untied,
sentinel windows; tests/test_oracle_invariants.py) and agrees with transformers'
Qwen2ForCausalLM in fp32 (tests/test_oracle_vs_transformers.py).  The decode-loop restatement in
`oracle/decode.py` is pinned against the reference's own runtime.py (tests/golden/).
"""

from __future__ import annotations

import dataclasses
import math

import torch


@dataclasses.dataclass(frozen=True)
class OracleConfig:
    """Mirror of FastDLLMRelaxConfig (model/cuda.py:15-29)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool = True
    bd_size: int = 32


def _dt(name: str) -> torch.dtype:
    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


class OracleModel:
    """The nine entry points of the compiled module, over CPU torch tensors.

    `params` is the flat list in the artifact's param_names order: embed, then per layer
    (qkv.w, qkv.b, o.w, gate_up.w, down.w, ln1.w, ln2.w), final norm, and lm_head when untied.
    """

    def __init__(self, cfg: OracleConfig, params: list[torch.Tensor], dtype: str):
        self.cfg = cfg
        self.dtype = _dt(dtype)
        n_expected = 1 + 7 * cfg.num_hidden_layers + 1 + (0 if cfg.tie_word_embeddings else 1)
        if len(params) != n_expected:
            raise ValueError(f"expected {n_expected} params, got {len(params)}")
        p = [t.to("cpu", self.dtype) for t in params]
        self.embed_w = p[0]
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            b = 1 + 7 * i
            self.layers.append(dict(qkv_w=p[b], qkv_b=p[b + 1], o_w=p[b + 2], gu_w=p[b + 3],
                                    down_w=p[b + 4], ln1=p[b + 5], ln2=p[b + 6]))
        self.norm_w = p[1 + 7 * cfg.num_hidden_layers]
        self.lm_w = self.embed_w if cfg.tie_word_embeddings else p[-1]

    # ---- elementwise helpers (each op computed in fp32, rounded to the model dtype) ----------
    def _r(self, x: torch.Tensor) -> torch.Tensor:
        return x.to(self.dtype)

    def rms_norm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """model/cuda.py:269-275."""
        xf = x.float()
        var = (xf * xf).mean(dim=-1, keepdim=True)
        xf = xf * torch.rsqrt(var + torch.tensor(self.cfg.rms_norm_eps, dtype=torch.float32))
        xc = self._r(xf)
        return self._r(w.float() * xc.float())

    def linear(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
        """nn.Linear: fp32 accumulate (+ bias), one rounding to the model dtype."""
        acc = x.float() @ w.float().t()
        if b is not None:
            acc = acc + b.float()
        return self._r(acc)

    def rope_tables(self, n: int, offset: int) -> tuple[torch.Tensor, torch.Tensor]:
        """model/cuda.py:278-300 (offset 0 gives model/cuda.py:226-238)."""
        hd = self.cfg.head_dim
        half = hd // 2
        neg_log = torch.tensor(-math.log(self.cfg.rope_theta), dtype=torch.float32)
        exponent = (neg_log * torch.arange(0, half, dtype=torch.float32)) / torch.tensor(float(half))
        inv_freq = torch.exp(exponent)
        pos = torch.arange(0, n, dtype=torch.float32) + torch.tensor(float(offset), dtype=torch.float32)
        freqs = pos[:, None] * inv_freq[None, :]
        emb = torch.cat([freqs, freqs], dim=-1)
        return self._r(torch.cos(emb)), self._r(torch.sin(emb))

    def apply_rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """x: [n, heads, hd]; model/cuda.py:207-209 rotate_half, 244-245 apply."""
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        rot = torch.cat([self._r(x2.float() * -1.0), x1], dim=-1)
        c, s = cos[:, None, :].float(), sin[:, None, :].float()
        a = self._r(x.float() * c)
        b = self._r(rot.float() * s)
        return self._r(a.float() + b.float())

    def _qkv(self, layer: dict, xn: torch.Tensor, offset: int):
        cfg = self.cfg
        n = xn.shape[0]
        qkv = self.linear(xn, layer["qkv_w"], layer["qkv_b"])
        qd = cfg.num_attention_heads * cfg.head_dim
        kd = cfg.num_key_value_heads * cfg.head_dim
        q = qkv[:, :qd].reshape(n, cfg.num_attention_heads, cfg.head_dim)
        k = qkv[:, qd:qd + kd].reshape(n, cfg.num_key_value_heads, cfg.head_dim)
        v = qkv[:, qd + kd:].reshape(n, cfg.num_key_value_heads, cfg.head_dim)
        cos, sin = self.rope_tables(n, offset)
        return self.apply_rope(q, cos, sin), self.apply_rope(k, cos, sin), v

    def _attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                bias: torch.Tensor | None) -> torch.Tensor:
        """q [n, Hq, hd], k/v [L, Hkv, hd] -> [n, Hq*hd] in the model dtype (fp32 math)."""
        cfg = self.cfg
        groups = cfg.num_attention_heads // cfg.num_key_value_heads
        kr = k.repeat_interleave(groups, dim=1)     # model/cuda.py:212-215, repeat on the head axis
        vr = v.repeat_interleave(groups, dim=1)
        qh = q.permute(1, 0, 2).float()             # [Hq, n, hd]
        kh = kr.permute(1, 2, 0).float()            # [Hq, hd, L]
        vh = vr.permute(1, 0, 2).float()            # [Hq, L, hd]
        scores = torch.matmul(qh, kh) * torch.tensor(cfg.head_dim ** -0.5, dtype=torch.float32)
        if bias is not None:
            scores = scores + bias.float()
        probs = torch.softmax(scores, dim=-1)
        out = torch.matmul(probs, vh)               # fp32 through both matmuls
        return self._r(out).permute(1, 0, 2).reshape(q.shape[0], -1)

    def _mlp(self, layer: dict, h: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        xn = self.rms_norm(h, layer["ln2"])
        gu = self.linear(xn, layer["gu_w"])
        gate, up = gu[:, :cfg.intermediate_size], gu[:, cfg.intermediate_size:]
        g = gate.float()
        act = self._r(g * torch.sigmoid(g))
        prod = self._r(act.float() * up.float())
        return self._r(h.float() + self.linear(prod, layer["down_w"]).float())

    # ---- entry points (model/cuda.py:698-788; signatures model/cuda.py:799-842) -------------
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        return self.embed_w[ids.long()]

    def forward_hidden(self, x: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        """x [1, T, H], bias [1, 1, T, T] -> [1, T, H]."""
        h = x[0].to(self.dtype)
        b2 = bias[0, 0]
        for layer in self.layers:
            xn = self.rms_norm(h, layer["ln1"])
            q, k, v = self._qkv(layer, xn, 0)
            attn = self._attend(q, k, v, b2)
            h = self._r(h.float() + self.linear(attn, layer["o_w"]).float())
            h = self._mlp(layer, h)
        return self.rms_norm(h, self.norm_w)[None]

    def get_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """hidden [1, R, H] -> fp32 logits [1, R, V] (matmul rounds to the model dtype first)."""
        return self.linear(hidden[0], self.lm_w).float()[None]

    def build_prefix_cache(self, x: torch.Tensor, bias: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor) -> None:
        """Writes post-RoPE K/V rows [0, P) of every layer in place (model/cuda.py:610-637)."""
        h = x[0].to(self.dtype)
        P = h.shape[0]
        if P > k_cache.shape[2]:
            raise ValueError(f"KV write [0, {P}) outside cache capacity {k_cache.shape[2]}")
        b2 = bias[0, 0]
        for i, layer in enumerate(self.layers):
            xn = self.rms_norm(h, layer["ln1"])
            q, k, v = self._qkv(layer, xn, 0)
            attn = self._attend(q, k, v, b2)
            h = self._r(h.float() + self.linear(attn, layer["o_w"]).float())
            h = self._mlp(layer, h)
            k_cache[i, 0, :P] = k
            v_cache[i, 0, :P] = v

    def forward_cached(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       cache_offset: int, prefix_len: int, write_rel: int = 0,
                       attend_rel: int | None = None) -> torch.Tensor:
        """model/cuda.py:639-666 with the callback semantics of runtime.py:63-73."""
        h = x[0].to(self.dtype)
        rows = h.shape[0]
        if attend_rel is None:
            attend_rel = rows
        write_start = prefix_len + write_rel
        attend_len = prefix_len + attend_rel
        if write_start + rows > attend_len:
            raise ValueError(f"KV write [{write_start}, {write_start + rows}) past the attended rows [0, {attend_len})")
        if write_start < 0 or write_start + rows > k_cache.shape[2]:
            raise ValueError(f"KV write [{write_start}, {write_start + rows}) outside cache capacity {k_cache.shape[2]}")
        for i, layer in enumerate(self.layers):
            xn = self.rms_norm(h, layer["ln1"])
            q, k, v = self._qkv(layer, xn, int(cache_offset))
            k_cache[i, 0, write_start:write_start + rows] = k
            v_cache[i, 0, write_start:write_start + rows] = v
            attn = self._attend(q, k_cache[i, 0, :attend_len], v_cache[i, 0, :attend_len], None)
            h = self._r(h.float() + self.linear(attn, layer["o_w"]).float())
            h = self._mlp(layer, h)
        return self.rms_norm(h, self.norm_w)[None]

    def forward_block_partial(self, x, k_cache, v_cache, cache_offset, prefix_len, replace_position):
        """forward_block_partial_rp{0,8,16,24} (model/cuda.py:740-788)."""
        return self.forward_cached(x, k_cache, v_cache, cache_offset, prefix_len,
                                   write_rel=replace_position, attend_rel=self.cfg.bd_size)


# ---- device-confidence semantics (model/metal.py:316-374, model/metal.py:513-528) -----------
def confidence(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """logits [R, V] fp32 -> (first-index argmax int32 [R], 1/sum(exp(l - max)) fp32 [R])."""
    lf = logits.float()
    mx = lf.max(dim=-1, keepdim=True).values
    ids = (lf == mx).int().argmax(dim=-1).int()     # first index equal to the max
    s = torch.exp(lf - mx).sum(dim=-1)
    return ids, (1.0 / s).float()


def build_block_bias(prefix_len: int, block_len: int, block_size: int | None = None,
                     blocked_value: float = -1e9) -> torch.Tensor:
    """model/cuda.py:148-177: bias [1, 1, T, T], 0 where q//bs >= k//bs else blocked_value."""
    if prefix_len < 0:
        raise ValueError("prefix_len must be non-negative")
    if block_len <= 0:
        raise ValueError("block_len must be positive")
    T = prefix_len + block_len
    bs = block_len if block_size is None else int(block_size)
    if bs <= 0:
        raise ValueError("block_size must be positive when provided")
    pos = torch.arange(T, dtype=torch.int32)
    allowed = (pos[:, None] // bs) >= (pos[None, :] // bs)
    return torch.where(allowed, 0.0, blocked_value).float()[None, None]
