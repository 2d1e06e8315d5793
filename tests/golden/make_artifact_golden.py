"""Record what the reference's own exporter writes for an artifact directory.

Run where a checkout of the reference exists, naming it:

    FDLLM_REFERENCE=<path to the reference checkout> python tests/golden/make_artifact_golden.py

The reference's export (scripts/export_cuda.py:113-168) compiles the model with TVM, which cannot
run here, but the files besides the compiled library come from plain Python that can:
`export_utils.remap_params` fuses the checkpoint's q/k/v and gate/up projections into the model's
parameter layout and stores bf16 as uint16 bits, the parameters are saved with np.savez in the
model's parameter order together with their names and the dtype, and
`export_utils.write_kv_cache_manifest` writes the KV-cache contract.  This script runs those
functions (the parameter order from the reference's own model class, executed through
tests/golden/eager_nn.py) on a checkpoint-style state dict made by splitting the synthetic tiny
bf16 weights, repeats the export script's four write steps, and records a description of the
result (file texts, and per array its name, shape, dtype and sha256) in
tests/golden/artifact_format.json.  Nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if "FDLLM_REFERENCE" not in os.environ:
    raise SystemExit("set FDLLM_REFERENCE to the reference checkout")
REF = Path(os.environ["FDLLM_REFERENCE"])

sys.path.insert(0, str(REPO / "fast_dllm_relax_b200" / "tvm_shim"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))
sys.path.insert(1, str(REF))

import tvm  # noqa: E402  (the stand-in)

import eager_nn  # noqa: E402

eager_nn.install(tvm)
sys.modules["flash_attn"] = None

from fast_dllm_relax import export_utils  # noqa: E402
from fast_dllm_relax.model.cuda import FastDLLMRelaxConfig, FastDLLMRelaxForCausalLM  # noqa: E402

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params, param_names  # noqa: E402


def checkpoint_state_dict(cfg, params) -> dict[str, torch.Tensor]:
    """The fused synthetic weights split back into a Qwen2 checkpoint's separate projections."""
    sd = {}
    q, kv = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    for name, p in zip(param_names(cfg), params):
        if ".qkv_proj." in name:
            base = name.replace("qkv_proj.", "")
            head, kind = base.rsplit(".", 1)
            sd[f"{head}.q_proj.{kind}"], sd[f"{head}.k_proj.{kind}"], sd[f"{head}.v_proj.{kind}"] = \
                p[:q], p[q:q + kv], p[q + kv:]
        elif ".gate_up_proj." in name:
            head = name.replace(".gate_up_proj.weight", "")
            sd[f"{head}.gate_proj.weight"], sd[f"{head}.up_proj.weight"] = \
                p[:cfg.intermediate_size], p[cfg.intermediate_size:]
        else:
            sd[name] = p
    return sd


def describe(d: Path) -> dict:
    out = {"files": sorted(p.name for p in d.iterdir())}
    for f in (export_utils.KV_CACHE_MANIFEST, "fast_dllm_relax_nn_param_names.txt", "fast_dllm_relax_nn_dtype.txt"):
        out[f] = (d / f).read_text(encoding="utf-8")
    with np.load(d / "fast_dllm_relax_nn_params.npz") as z:
        out["arrays"] = [dict(name=k, shape=list(z[k].shape), dtype=str(z[k].dtype),
                              sha256=hashlib.sha256(np.ascontiguousarray(z[k]).tobytes()).hexdigest())
                         for k in z.files]
    return out


def main() -> None:
    cfg, dtype = TINY, "bfloat16"
    params = make_synthetic_params(cfg, seed=0, dtype=dtype, mask_id=TINY_MASK_ID)
    rcfg = FastDLLMRelaxConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                               intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                               num_attention_heads=cfg.num_attention_heads,
                               num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                               rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                               context_window_size=cfg.context_window_size,
                               tie_word_embeddings=cfg.tie_word_embeddings, bd_size=cfg.bd_size,
                               pad_token_id=cfg.pad_token_id)
    model = FastDLLMRelaxForCausalLM(rcfg, dtype=dtype, fused_qkv=True, fused_gate_up=True)
    named_param_dict = dict(model.named_parameters())
    mapped = export_utils.remap_params(checkpoint_state_dict(cfg, params), named_param_dict, rcfg,
                                       torch_dtype=torch.bfloat16, np_dtype=np.uint16)
    with tempfile.TemporaryDirectory() as tmp:
        d = Path(tmp)
        # the export script's write steps (scripts/export_cuda.py:162-168); the compiled library
        # itself (export_library) needs TVM and is not part of the description
        np.savez(d / "fast_dllm_relax_nn_params.npz", *[mapped[n] for n in named_param_dict])
        (d / "fast_dllm_relax_nn_param_names.txt").write_text("\n".join(named_param_dict) + "\n", encoding="utf-8")
        (d / "fast_dllm_relax_nn_dtype.txt").write_text(dtype + "\n", encoding="utf-8")
        export_utils.write_kv_cache_manifest(d, rcfg, dtype)
        desc = describe(d)
    desc["weights"] = "make_synthetic_params(TINY, seed=0, bfloat16, mask_id=1023)"
    # the parameter list the reference's model class exports, tied and untied (the artifact's
    # params.npz order; tests/test_tiny_compile.py:74-84 checks the same split)
    desc["param_lists"] = {}
    for tied in (True, False):
        import dataclasses  # noqa: PLC0415
        m = FastDLLMRelaxForCausalLM(dataclasses.replace(rcfg, tie_word_embeddings=tied), dtype=dtype,
                                     fused_qkv=True, fused_gate_up=True)
        desc["param_lists"]["tied" if tied else "untied"] = [[n, list(p._shape)] for n, p in m.named_parameters()]
    (HERE / "artifact_format.json").write_text(json.dumps(desc, indent=1) + "\n", encoding="utf-8")
    print(len(desc["arrays"]), "arrays;", desc["files"])


if __name__ == "__main__":
    main()
