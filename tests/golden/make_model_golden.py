"""Generate golden vectors of the reference's OWN model graph (fast_dllm_relax/model/cuda.py).

Run where a checkout of the reference exists, naming it:

    FDLLM_REFERENCE=<path to the reference checkout> python tests/golden/make_model_golden.py

TVM cannot be installed here, so the reference's model definition is executed op by op through
tests/golden/eager_nn.py, an eager PyTorch stand-in for the slice of TVM's Relax `nn` frontend it
is written against.  The cached entry points call the reference runtime's own packed callbacks
(`fast_dllm.attn_inplace`, `fast_dllm.kv_write`, runtime.py:46-73; their PyTorch SDPA branch, as
flash_attn cannot run on the CPU).  The model is FastDLLMRelaxForCausalLM with fused qkv and
gate_up projections (the artifact layout), on the small head_dim-128 architecture and weights of
tests/_oracle_util.pin_config / pin_params, in fp32 and bf16.

Recorded per dtype (tests/golden/model_graph.npz; bf16 values stored as uint16 bit patterns):
  dense/h        forward_hidden over 96 rows with the block-causal bias: the last 32 rows
  dense/logits   get_logits of those 32 rows (fp32)
  prefill/k, v   build_prefix_cache over the first 64 rows: the last layer's K/V rows [0, 64)
  cached/h       forward_cached of rows [64, 96) (cache_offset 64, prefix_len 64)
  cached/k, v    the last layer's K/V rows [64, 96) it wrote
  partial/h      forward_block_partial_rp8 of 8 new rows (cache_offset 72, prefix_len 64)
  partial/k, v   the last layer's K/V rows [72, 80) it overwrote

Decode runs of the whole reference stack (tests/golden/model_decode.json): the reference's
runtime.py (`relax_greedy_generate`) drives a VirtualMachine whose entry points are this eager
reference graph, in fp32 on the same architecture (mask id 511, its embedding row zeroed); the
tokens, step statistics and entry-point calls are recorded, and so are the log-likelihoods and
argmax rows of three answer choices scored against one context with the prefix cache reused.
Nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
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

assert getattr(tvm, "IS_FDLLM_SHIM", False), "expected the repository's TVM stand-in"
eager_nn.install(tvm)
sys.modules["flash_attn"] = None  # the runtime's attention callback takes its SDPA branch

import fast_dllm_relax.runtime  # noqa: E402,F401  (registers the packed callbacks)
from fast_dllm_relax.model.cuda import (  # noqa: E402
    FastDLLMRelaxConfig,
    FastDLLMRelaxForCausalLM,
    build_prefix_block_attention_bias,
)

from fast_dllm_relax_b200.config import param_names  # noqa: E402
import fast_dllm_relax.runtime as ref_rt  # noqa: E402
from tests._oracle_util import PIN_MASK_ID, pin_config, pin_params  # noqa: E402

P, B, S, RP = 64, 32, 8, 8


def run(dtype: str) -> dict[str, np.ndarray]:
    cfg = pin_config()
    model = ref_model(dtype)
    T = eager_nn.Tensor
    g = torch.Generator().manual_seed(21)
    ids = torch.randint(0, cfg.vocab_size, (P + B,), generator=g, dtype=torch.int32)
    ids8 = torch.randint(0, cfg.vocab_size, (S,), generator=g, dtype=torch.int32)
    x = model.embed(T(ids))._expr.as_subclass(torch.Tensor).reshape(1, P + B, -1)
    x8 = model.embed(T(ids8))._expr.as_subclass(torch.Tensor).reshape(1, S, -1)
    out = {"ids": ids.numpy(), "ids8": ids8.numpy()}

    bias = torch.from_numpy(build_prefix_block_attention_bias(0, P + B, block_size=B))
    h = model.forward_hidden(T(x), T(bias))._expr.as_subclass(torch.Tensor)
    logits = model.get_logits(T(h[:, P:]))._expr.as_subclass(torch.Tensor)
    out["dense/h"], out["dense/logits"] = h[0, P:], logits[0]

    shape = (cfg.num_hidden_layers, 1, P + B, cfg.num_key_value_heads, cfg.head_dim)
    k = torch.zeros(shape, dtype=x.dtype)
    v = torch.zeros(shape, dtype=x.dtype)
    pbias = torch.from_numpy(build_prefix_block_attention_bias(0, P, block_size=B))
    model.build_prefix_cache(T(x[:, :P].contiguous()), T(pbias), T(k), T(v))
    out["prefill/k"], out["prefill/v"] = k[-1, 0, :P].clone(), v[-1, 0, :P].clone()

    off = T(torch.tensor(P, dtype=torch.int32))
    hc = model.forward_cached(T(x[:, P:].contiguous()), T(k), T(v), off, P)._expr.as_subclass(torch.Tensor)
    out["cached/h"], out["cached/k"], out["cached/v"] = hc[0], k[-1, 0, P:P + B].clone(), v[-1, 0, P:P + B].clone()

    off8 = T(torch.tensor(P + RP, dtype=torch.int32))
    hp = model.forward_block_partial_rp8(T(x8), T(k), T(v), off8, P)._expr.as_subclass(torch.Tensor)
    out["partial/h"] = hp[0]
    out["partial/k"], out["partial/v"] = k[-1, 0, P + RP:P + RP + S].clone(), v[-1, 0, P + RP:P + RP + S].clone()

    res = {}
    for key, val in out.items():
        if isinstance(val, torch.Tensor):
            val = val.detach()
            val = val.view(torch.int16).numpy().view(np.uint16) if val.dtype == torch.bfloat16 else val.numpy()
        res[f"{dtype}/{key}"] = np.ascontiguousarray(val)
    return res


def ref_model(dtype: str, mask_id: int | None = None):
    cfg = pin_config()
    rcfg = FastDLLMRelaxConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                               intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                               num_attention_heads=cfg.num_attention_heads,
                               num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                               rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                               context_window_size=cfg.context_window_size,
                               tie_word_embeddings=cfg.tie_word_embeddings, bd_size=cfg.bd_size,
                               pad_token_id=cfg.pad_token_id)
    model = FastDLLMRelaxForCausalLM(rcfg, dtype=dtype, fused_qkv=True, fused_gate_up=True)
    named = list(model.named_parameters())
    assert [n for n, _ in named] == param_names(cfg), "parameter order differs from the artifact's"
    for (_, p), t in zip(named, pin_params(dtype, mask_id)):
        p.bind(t)
    return model


class RefGraphBackend:
    """vm[name] served by the eager reference graph over the stand-in's tensors; logs every call
    in the golden call-log format [name, rows, cache_offset, prefix_len]."""

    def __init__(self, model):
        self.model = model
        self.calls: list[list] = []

    def function(self, name: str):
        m, E, R = self.model, eager_nn.Tensor, tvm.runtime.Tensor

        def out(t):
            return R(t._expr.as_subclass(torch.Tensor))

        if name == "embed":
            def embed(ids, params):
                self.calls.append(["embed", int(ids.shape[0]), -1, -1])
                return out(m.embed(E(ids.torch)))
            return embed
        if name == "forward_hidden":
            def forward_hidden(x, bias, params):
                self.calls.append(["forward_hidden", int(x.shape[1]), -1, -1])
                return out(m.forward_hidden(E(x.torch), E(bias.torch)))
            return forward_hidden
        if name == "get_logits":
            def get_logits(h, params):
                self.calls.append(["get_logits", int(h.shape[1]), -1, -1])
                return out(m.get_logits(E(h.torch)))
            return get_logits
        if name == "build_prefix_cache":
            def build_prefix_cache(x, bias, k, v, params):
                self.calls.append(["build_prefix_cache", int(x.shape[1]), -1, -1])
                m.build_prefix_cache(E(x.torch), E(bias.torch), E(k.torch), E(v.torch))
                return k, v
            return build_prefix_cache
        if name == "forward_cached" or name.startswith("forward_block_partial_rp"):
            def cached(x, k, v, off, plen, params):
                o, p = int(off.torch.item()), int(plen[0])
                self.calls.append([name, int(x.shape[1]), o, p])
                fn = m.forward_cached if name == "forward_cached" else getattr(m, name)
                return out(fn(E(x.torch), E(k.torch), E(v.torch), E(off.torch), p))
            return cached
        raise KeyError(name)  # no static or confidence siblings: the reference's host path runs


class RefGraphModule:
    def __init__(self, model):
        self.model = model

    def create_backend(self, dev):
        return RefGraphBackend(self.model)


def make_decode() -> None:
    cfg = pin_config()
    model = ref_model("float32", PIN_MASK_ID)
    dev = tvm.cpu(0)
    vm = tvm.relax.VirtualMachine(RefGraphModule(model), dev)
    params = [tvm.runtime.Tensor(t) for t in pin_params("float32", PIN_MASK_ID)]
    reshape = tvm.get_global_func("vm.builtin.reshape")
    spec = ref_rt.CacheSpec(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim, "float32")
    rng = np.random.default_rng(4)
    p64, p45, p20 = (rng.integers(0, 500, n).tolist() for n in (64, 45, 20))
    cases = [dict(name="aligned_nocache", prompt=p64, max_new_tokens=64, use_block_cache=False),
             dict(name="aligned_blockcache", prompt=p64, max_new_tokens=64, use_block_cache=True),
             dict(name="unaligned_blockcache", prompt=p45, max_new_tokens=40, use_block_cache=True),
             dict(name="short_prompt_stateless", prompt=p20, max_new_tokens=20, use_block_cache=True)]
    out = {"mask_id": PIN_MASK_ID, "cases": []}

    def run_case(case):
        vm.backend.calls.clear()
        toks, stats = ref_rt.relax_greedy_generate(
            vm, params, dev, reshape, None, list(case["prompt"]), num_attention_heads=cfg.num_attention_heads,
            max_new_tokens=case["max_new_tokens"], block_size=32, small_block_size=8,
            threshold=case.get("threshold", 0.9), temperature=0.0, top_p=0.95,
            use_block_cache=case["use_block_cache"], mask_id=PIN_MASK_ID, stop_token=case.get("stop_token"),
            cache_spec=spec, chunked_prefill=case.get("chunked_prefill", False))
        print(case["name"], len(toks), stats, flush=True)
        out["cases"].append(dict(case, tokens=[int(t) for t in toks], stats=stats, calls=list(vm.backend.calls)))

    for case in cases:
        run_case(case)
    p96 = rng.integers(0, 500, 96).tolist()
    run_case(dict(name="chunked_prefill", prompt=p96, max_new_tokens=33, use_block_cache=True, chunked_prefill=True))
    first = out["cases"][1]["tokens"]  # stop on the first token that differs from the first one
    run_case(dict(name="stop_token", prompt=p64, max_new_tokens=64, use_block_cache=True,
                  stop_token=next(t for t in first if t != first[0])))
    run_case(dict(name="low_threshold", prompt=p64, max_new_tokens=64, use_block_cache=True, threshold=0.0025))
    # masked-continuation scoring (runtime.py:485-588), the second and third choices reusing the
    # first one's prefix cache (runtime.py:546-548)
    ctx = rng.integers(0, 500, 70).tolist()
    cached, scoring = None, []
    vm.backend.calls.clear()
    for n in (3, 9, 1):
        cont = rng.integers(0, 500, n).tolist()
        logits, cached = ref_rt.score_masked_continuation(
            vm, params, dev, reshape, ctx, cont, num_attention_heads=cfg.num_attention_heads, block_size=32,
            mask_id=PIN_MASK_ID, cache_spec=spec, eos_token_id=PIN_MASK_ID - 1, cached_prefix=cached)
        lp = torch.log_softmax(torch.from_numpy(np.asarray(logits, dtype=np.float32)), dim=-1)
        scoring.append(dict(continuation=cont, loglik=float(lp.gather(-1, torch.tensor(cont)[:, None]).sum()),
                            argmax=[int(i) for i in np.asarray(logits).argmax(-1)]))
    out["scoring"] = dict(context=ctx, choices=scoring, calls=list(vm.backend.calls))
    print("scoring", [c["loglik"] for c in scoring], flush=True)
    (HERE / "model_decode.json").write_text(json.dumps(out, indent=1) + "\n", encoding="utf-8")


def main() -> None:
    torch.set_num_threads(1)  # deterministic CPU reductions
    res = {"model_cuda_sha256": np.asarray(hashlib.sha256((REF / "fast_dllm_relax/model/cuda.py").read_bytes())
                                           .hexdigest())}
    with torch.no_grad():
        for dtype in ("float32", "bfloat16"):
            res.update(run(dtype))
            print(dtype, "ok", flush=True)
        if "--only" not in sys.argv or "graph" in sys.argv:
            np.savez_compressed(HERE / "model_graph.npz", **res)
        if "--only" not in sys.argv or "decode" in sys.argv:
            make_decode()


if __name__ == "__main__":
    main()
