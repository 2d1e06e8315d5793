"""The oracle's model arithmetic against an independent implementation: transformers'
Qwen2ForCausalLM (the architecture Fast-dLLM v2 builds on), fp32, fed the same weights (qkv and
gate_up split back into q/k/v and gate/up, export_utils.py:84-104 in reverse) and the reference's
block-causal bias as a 4-D additive mask (model/cuda.py:148-177).  The reference's own numerics
(TVM, the checkpoint's remote modeling code) cannot run here; this pins the oracle's op order
(RMSNorm, RoPE, GQA attention, SwiGLU, final norm) to a second implementation."""

import pytest
import torch

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params
from oracle.model import build_block_bias
from tests._oracle_util import make_oracle

transformers = pytest.importorskip("transformers")


def _hf_model(cfg, params):
    hc = transformers.Qwen2Config(
        vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
        num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
        num_key_value_heads=cfg.num_key_value_heads, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
        max_position_embeddings=cfg.context_window_size, tie_word_embeddings=True, attn_implementation="eager")
    m = transformers.Qwen2ForCausalLM(hc).eval()
    hq, hkv, hd, inter = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size
    sd = {"model.embed_tokens.weight": params[0], "lm_head.weight": params[0],
          "model.norm.weight": params[1 + 7 * cfg.num_hidden_layers]}
    for l in range(cfg.num_hidden_layers):
        qkv_w, qkv_b, o_w, gu_w, d_w, ln1, ln2 = params[1 + 7 * l:8 + 7 * l]
        a, mlp = f"model.layers.{l}.self_attn", f"model.layers.{l}.mlp"
        for name, w, b in zip("qkv", qkv_w.split([hq * hd, hkv * hd, hkv * hd]),
                              qkv_b.split([hq * hd, hkv * hd, hkv * hd])):
            sd[f"{a}.{name}_proj.weight"], sd[f"{a}.{name}_proj.bias"] = w, b
        sd[f"{a}.o_proj.weight"] = o_w
        sd[f"{mlp}.gate_proj.weight"], sd[f"{mlp}.up_proj.weight"] = gu_w.split([inter, inter])
        sd[f"{mlp}.down_proj.weight"] = d_w
        sd[f"model.layers.{l}.input_layernorm.weight"] = ln1
        sd[f"model.layers.{l}.post_attention_layernorm.weight"] = ln2
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not missing and not unexpected
    return m


@pytest.mark.parametrize("T", [32, 70, 96])
def test_dense_forward_matches_transformers_qwen2(T):
    params = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    orc = make_oracle(TINY, params, "float32")
    hf = _hf_model(TINY, params)
    ids = torch.randint(0, 1000, (T,), generator=torch.Generator().manual_seed(T), dtype=torch.int32)
    x = orc.embed(ids)[None]
    bias = build_block_bias(0, T, 32)
    ref = orc.forward_hidden(x, bias)
    with torch.no_grad():
        hf_h = hf.model(inputs_embeds=x, attention_mask=bias, use_cache=False).last_hidden_state
        hf_logits = hf.lm_head(hf_h)
    torch.testing.assert_close(ref, hf_h, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(orc.get_logits(ref), hf_logits, rtol=1e-5, atol=1e-5)
