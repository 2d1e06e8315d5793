"""Model configuration, parameter layout and seeded synthetic weights.

The parameter list layout is the reference artifact's: the flat order of
`fast_dllm_relax_nn_param_names.txt`, which is the named-parameter order of
`FastDLLMRelaxForCausalLM` (fast_dllm_relax/model/cuda.py:532-602, 669-684): the embedding, then
per layer the fused qkv_proj weight and bias, o_proj, the fused gate_up_proj, down_proj and the
two RMSNorm weights, then the final norm, then lm_head for untied checkpoints.  Weights are
[out, in] (fast_dllm_relax/export_utils.py:84-104).
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import torch

DTYPE_CODES = {"float32": 0, "bfloat16": 1}


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    """Mirror of FastDLLMRelaxConfig (fast_dllm_relax/model/cuda.py:15-29)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    context_window_size: int = 32768
    tie_word_embeddings: bool = True
    bd_size: int = 32
    pad_token_id: int = 0

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), indent=2)

    @classmethod
    def from_json(cls, text: str) -> "ModelConfig":
        d = json.loads(text)
        fields = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in fields})

    @classmethod
    def from_file(cls, path: str | Path) -> "ModelConfig":
        return cls.from_json(Path(path).read_text(encoding="utf-8"))


# tiny Qwen2-style block-diffusion LM (fp32, seed 0).
TINY = ModelConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                   num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-6,
                   rope_theta=1e6, context_window_size=4096, tie_word_embeddings=True)

# BASELINE configs[1..4]: Fast-dLLM v2 1.5B (Qwen2.5-1.5B shape).
QWEN_1_5B = ModelConfig(vocab_size=151936, hidden_size=1536, intermediate_size=8960,
                        num_hidden_layers=28, num_attention_heads=12, num_key_value_heads=2,
                        head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                        context_window_size=32768, tie_word_embeddings=True)

TINY_MASK_ID = 1023
QWEN_MASK_ID = 151665  # fast_dllm_relax/common.py:30


def param_names(cfg: ModelConfig) -> list[str]:
    names = ["model.embed_tokens.weight"]
    for i in range(cfg.num_hidden_layers):
        a, m = f"model.layers.{i}.self_attn", f"model.layers.{i}.mlp"
        names += [f"{a}.qkv_proj.weight", f"{a}.qkv_proj.bias", f"{a}.o_proj.weight",
                  f"{m}.gate_up_proj.weight", f"{m}.down_proj.weight",
                  f"model.layers.{i}.input_layernorm.weight",
                  f"model.layers.{i}.post_attention_layernorm.weight"]
    names.append("model.norm.weight")
    if not cfg.tie_word_embeddings:
        names.append("lm_head.weight")
    return names


def param_shapes(cfg: ModelConfig) -> list[tuple[int, ...]]:
    H, I, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    qkv = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * hd
    shapes: list[tuple[int, ...]] = [(cfg.vocab_size, H)]
    for _ in range(cfg.num_hidden_layers):
        shapes += [(qkv, H), (qkv,), (H, cfg.num_attention_heads * hd), (2 * I, H), (H, I), (H,), (H,)]
    shapes.append((H,))
    if not cfg.tie_word_embeddings:
        shapes.append((cfg.vocab_size, H))
    return shapes


def make_synthetic_params(cfg: ModelConfig, seed: int, dtype: str = "float32",
                          device: str | torch.device = "cpu", std: float = 0.02,
                          mask_id: int | None = None) -> list[torch.Tensor]:
    """N(0, std) matrices and biases from torch.Generator(seed) on `device`, RMSNorm weights 1.0
    (as the reference's own tests do, tests/test_tiny_compile.py:45-55).  The values depend on the
    generating device type; tests generate on the CPU and upload.

    `mask_id`: zero that token's embedding (and lm_head) row.  Its logit is then exactly 0 while the
    other vocab logits are nonzero, so greedy decoding never predicts the mask token.  Without this,
    random tied weights can make the mask id win an argmax; the decode loop (runtime.py:750-805)
    then writes the mask id back into a masked slot and repeats the identical step forever.
    """
    dt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype]
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    out = []
    for name, shape in zip(param_names(cfg), param_shapes(cfg)):
        if name.endswith("norm.weight"):
            out.append(torch.ones(shape, dtype=dt, device=device))
        else:
            t = torch.randn(shape, generator=gen, dtype=torch.float32, device=device)
            if mask_id is not None and name in ("model.embed_tokens.weight", "lm_head.weight"):
                t[int(mask_id)] = 0.0
            out.append((t * std).to(dt))
    return out
