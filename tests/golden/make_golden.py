"""Generate the golden decode/scoring fixtures from the reference's own runtime.

Run where a checkout of the reference exists, naming it:

    FDLLM_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py

It imports the reference's UNMODIFIED `fast_dllm_relax/runtime.py` (and model/cuda.py's bias and
shift helpers) on top of this repository's TVM stand-in, with a VirtualMachine whose nine entry
points are computed by the CPU oracle (oracle/model.py) on the tiny fp32 config (BASELINE
2 layers, hidden 256, 4/2 heads, head_dim 64, vocab 1024, seed-0 N(0, 0.02)
weights).  It records what the reference's decode loop and scorer produce -- generated tokens,
step statistics and the exact sequence of entry-point calls -- so that tests can pin the oracle's
decode restatement (oracle/decode.py) and the product's drivers against the reference's code.

Outputs (committed): tests/golden/tiny_decode.json, tests/golden/tiny_scoring.npz,
tests/golden/helpers.npz, tests/golden/tiny_choices.npz, tests/golden/tiny_decode_edges.json.
Nothing at test time reads the reference checkout.  `--only choices` and `--only edges`
regenerate one of the last two files alone (each draws from its own random stream, so the others
are unaffected).
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
sys.path.insert(1, str(REF))

import tvm  # noqa: E402  (the stand-in)

from fast_dllm_relax_b200.config import TINY, TINY_MASK_ID, make_synthetic_params  # noqa: E402
from oracle.model import OracleConfig, OracleModel  # noqa: E402

assert getattr(tvm, "IS_FDLLM_SHIM", False), "expected the repository's TVM stand-in"
import fast_dllm_relax.runtime as ref_rt  # noqa: E402
from fast_dllm_relax.model.cuda import (  # noqa: E402
    build_prefix_block_attention_bias,
    extract_shifted_block_logits,
)


def oracle_config(cfg) -> OracleConfig:
    return OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                        intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                        num_attention_heads=cfg.num_attention_heads,
                        num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                        rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
                        tie_word_embeddings=cfg.tie_word_embeddings, bd_size=cfg.bd_size)


class OracleBackend:
    """The nine entry points over shim tensors, computed by the CPU oracle; logs every call."""

    def __init__(self, model: OracleModel):
        self.model = model
        self.calls: list[list] = []

    def function(self, name: str):
        m = self.model
        T = tvm.runtime.Tensor
        if name == "embed":
            def embed(ids, params):
                self.calls.append(["embed", int(ids.shape[0]), -1, -1])
                return T(m.embed(ids.torch))
            return embed
        if name == "forward_hidden":
            def forward_hidden(x, bias, params):
                self.calls.append(["forward_hidden", int(x.shape[1]), -1, -1])
                return T(m.forward_hidden(x.torch, bias.torch))
            return forward_hidden
        if name == "get_logits":
            def get_logits(h, params):
                self.calls.append(["get_logits", int(h.shape[1]), -1, -1])
                return T(m.get_logits(h.torch))
            return get_logits
        if name == "build_prefix_cache":
            def build_prefix_cache(x, bias, k, v, params):
                self.calls.append(["build_prefix_cache", int(x.shape[1]), -1, -1])
                m.build_prefix_cache(x.torch, bias.torch, k.torch, v.torch)
                return k, v
            return build_prefix_cache
        if name == "forward_cached":
            def forward_cached(x, k, v, off, plen, params):
                o, p = int(off.torch.item()), int(plen[0])
                self.calls.append(["forward_cached", int(x.shape[1]), o, p])
                return T(m.forward_cached(x.torch, k.torch, v.torch, o, p))
            return forward_cached
        if name.startswith("forward_block_partial_rp"):
            rp = int(name[len("forward_block_partial_rp"):])

            def partial(x, k, v, off, plen, params):
                o, p = int(off.torch.item()), int(plen[0])
                self.calls.append([name, int(x.shape[1]), o, p])
                return T(m.forward_block_partial(x.torch, k.torch, v.torch, o, p, rp))
            return partial
        raise KeyError(name)  # no static or confidence siblings: the reference's host path runs


class OracleModule:
    def __init__(self, model: OracleModel):
        self.model = model

    def create_backend(self, dev):
        return OracleBackend(self.model)


CHOICE_CONTINUATIONS = (2, 5, 25, 1)  # the third needs more than one block: the cache grows


def make_choices(vm, params, dev, reshape, spec) -> None:
    """Multiple-choice scoring with prefix-cache reuse (runtime.py:546-548): one context scored
    against several continuations in turn, each call handed the (aligned prefix, cache) pair the
    previous call returned, then a different context (the cache is rebuilt).  Records every
    choice's logits and log-likelihood and the entry-point calls, which show one prefix build per
    context."""
    rng = np.random.default_rng(2)
    ctx_a = rng.integers(0, 1000, 75).tolist()
    ctx_b = rng.integers(0, 1000, 40).tolist()
    plan = [(ctx_a, rng.integers(0, 1000, n).tolist()) for n in CHOICE_CONTINUATIONS]
    plan.append((ctx_b, rng.integers(0, 1000, 3).tolist()))
    out = {}
    cached = None
    vm.backend.calls.clear()
    for i, (ctx, cont) in enumerate(plan):
        logits, cached = ref_rt.score_masked_continuation(
            vm, params, dev, reshape, ctx, cont, num_attention_heads=TINY.num_attention_heads, block_size=32,
            mask_id=TINY_MASK_ID, cache_spec=spec, eos_token_id=1022, cached_prefix=cached)
        lp = torch.log_softmax(torch.from_numpy(np.asarray(logits, dtype=np.float32)), dim=-1)
        ll = float(lp.gather(-1, torch.tensor(cont).unsqueeze(-1)).squeeze(-1).sum().item())
        out[f"choice{i}/context"] = np.asarray(ctx, np.int32)
        out[f"choice{i}/continuation"] = np.asarray(cont, np.int32)
        out[f"choice{i}/logits"] = np.asarray(logits, np.float32)
        out[f"choice{i}/loglik"] = np.asarray(ll, np.float64)
        print(f"choice{i}", len(ctx), len(cont), ll, flush=True)
    out["n_choices"] = np.asarray(len(plan), np.int32)
    out["calls"] = np.asarray(json.dumps(vm.backend.calls))
    np.savez_compressed(HERE / "tiny_choices.npz", **out)


def make_edges(vm, params, dev, reshape, spec) -> None:
    """Decode edge cases of runtime.py:591-880: no new tokens, one new token after a block-aligned
    prompt (:679-708 alone), a stop on the very first committed token, and limits that cut the
    first block mid-refinement (:839-849, the continuation trimmed at the first mask)."""
    rng = np.random.default_rng(3)
    p64, p40 = rng.integers(0, 1000, 64).tolist(), rng.integers(0, 1000, 40).tolist()
    cases = [dict(name="zero_new_tokens", prompt=p64, max_new_tokens=0, use_block_cache=True),
             dict(name="one_new_token_aligned", prompt=p64, max_new_tokens=1, use_block_cache=False),
             dict(name="cut_mid_block", prompt=p40, max_new_tokens=5, use_block_cache=True),
             dict(name="cut_mid_block_nocache", prompt=p64, max_new_tokens=11, use_block_cache=False)]
    out = {"mask_id": TINY_MASK_ID, "cases": []}

    def run(case):
        vm.backend.calls.clear()
        kw = dict(num_attention_heads=TINY.num_attention_heads, max_new_tokens=case["max_new_tokens"],
                  block_size=32, small_block_size=8, threshold=0.9, temperature=0.0, top_p=0.95,
                  use_block_cache=case["use_block_cache"], mask_id=TINY_MASK_ID,
                  stop_token=case.get("stop_token"), cache_spec=spec)
        toks, stats = ref_rt.relax_greedy_generate(vm, params, dev, reshape, None, list(case["prompt"]), **kw)
        print(case["name"], len(toks), stats, flush=True)
        return dict(case, tokens=[int(t) for t in toks], stats=stats, calls=list(vm.backend.calls))

    for c in cases:
        out["cases"].append(run(c))
    first = out["cases"][1]["tokens"][0]  # the token the aligned prompt's commit step yields
    out["cases"].append(run(dict(name="stop_on_first_token", prompt=p64, max_new_tokens=40,
                                 use_block_cache=True, stop_token=int(first))))
    (HERE / "tiny_decode_edges.json").write_text(json.dumps(out, indent=1) + "\n", encoding="utf-8")


def main() -> None:
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    torch.manual_seed(0)
    params_t = make_synthetic_params(TINY, seed=0, dtype="float32", mask_id=TINY_MASK_ID)
    model = OracleModel(oracle_config(TINY), params_t, "float32")
    dev = tvm.cpu(0)
    vm = tvm.relax.VirtualMachine(OracleModule(model), dev)
    params = [tvm.runtime.Tensor(p) for p in params_t]
    reshape = tvm.get_global_func("vm.builtin.reshape")
    spec = ref_rt.CacheSpec(TINY.num_hidden_layers, TINY.num_key_value_heads, TINY.head_dim, "float32")
    if only == "choices":
        make_choices(vm, params, dev, reshape, spec)
        return
    if only == "edges":
        make_edges(vm, params, dev, reshape, spec)
        return
    rng = np.random.default_rng(0)

    def prompt(n):
        return rng.integers(0, 1000, n).tolist()

    base64 = prompt(64)
    cases = [
        dict(name="cfg0_nocache", prompt=base64, max_new_tokens=64, use_block_cache=False),
        dict(name="cfg0_blockcache", prompt=base64, max_new_tokens=64, use_block_cache=True),
        dict(name="short_prompt_stateless", prompt=prompt(20), max_new_tokens=40, use_block_cache=True),
        dict(name="one_block_prompt", prompt=prompt(32), max_new_tokens=40, use_block_cache=False),
        dict(name="unaligned_prompt", prompt=prompt(45), max_new_tokens=50, use_block_cache=True),
        dict(name="low_threshold", prompt=base64, max_new_tokens=64, use_block_cache=True, threshold=0.0011),
        dict(name="chunked_prefill", prompt=prompt(96), max_new_tokens=33, use_block_cache=True,
             chunked_prefill=True),
    ]
    # A stop-token case: stop on a token the no-cache run generates (copied from its output).
    out = {"reference_runtime_sha256": hashlib.sha256((REF / "fast_dllm_relax/runtime.py").read_bytes()).hexdigest(),
           "model_cuda_sha256": hashlib.sha256((REF / "fast_dllm_relax/model/cuda.py").read_bytes()).hexdigest(),
           "config": json.loads(TINY.to_json()), "weights": "make_synthetic_params(TINY, seed=0, float32, mask_id=1023)",
           "mask_id": TINY_MASK_ID, "cases": []}

    def run(case):
        vm.backend.calls.clear()
        kw = dict(num_attention_heads=TINY.num_attention_heads, max_new_tokens=case["max_new_tokens"],
                  block_size=32, small_block_size=8, threshold=case.get("threshold", 0.9), temperature=0.0,
                  top_p=0.95, use_block_cache=case["use_block_cache"], mask_id=TINY_MASK_ID,
                  stop_token=case.get("stop_token"), cache_spec=spec,
                  chunked_prefill=case.get("chunked_prefill", False))
        toks, stats = ref_rt.relax_greedy_generate(vm, params, dev, reshape, None, list(case["prompt"]), **kw)
        rec = dict(case, tokens=[int(t) for t in toks], stats=stats, calls=list(vm.backend.calls))
        print(case["name"], len(toks), stats, flush=True)
        return rec

    for c in cases:
        out["cases"].append(run(c))
    first = out["cases"][0]["tokens"]
    out["cases"].append(run(dict(name="stop_token", prompt=base64, max_new_tokens=64, use_block_cache=True,
                                 stop_token=int(first[6]))))
    (HERE / "tiny_decode.json").write_text(json.dumps(out, indent=1) + "\n", encoding="utf-8")

    # ---- scoring (runtime.score_masked_continuation + runners.py:877-881 reduction) -------------
    scoring = {}
    sc_cases = [("ctx70_cont5", prompt(70), prompt(5)), ("ctx20_cont4", prompt(20), prompt(4)),
                ("ctx64_cont40", prompt(64), prompt(40)), ("ctx96_cont16", prompt(96), prompt(16))]
    for name, ctx, cont in sc_cases:
        logits, _ = ref_rt.score_masked_continuation(
            vm, params, dev, reshape, ctx, cont, num_attention_heads=TINY.num_attention_heads, block_size=32,
            mask_id=TINY_MASK_ID, cache_spec=spec, eos_token_id=1022)
        lp = torch.log_softmax(torch.from_numpy(np.asarray(logits, dtype=np.float32)), dim=-1)
        ll = float(lp.gather(-1, torch.tensor(cont).unsqueeze(-1)).squeeze(-1).sum().item())
        scoring[f"{name}/context"] = np.asarray(ctx, np.int32)
        scoring[f"{name}/continuation"] = np.asarray(cont, np.int32)
        scoring[f"{name}/logits"] = np.asarray(logits, np.float32)
        scoring[f"{name}/loglik"] = np.asarray(ll, np.float64)
        print(name, ll, flush=True)
    np.savez_compressed(HERE / "tiny_scoring.npz", **scoring)

    # ---- model/cuda.py helpers -------------------------------------------------------------
    helpers = {}
    for P, B, bs in ((0, 32, 32), (64, 32, 32), (0, 96, 32), (5, 11, 4), (0, 7, None)):
        helpers[f"bias/{P}_{B}_{bs}"] = build_prefix_block_attention_bias(P, B, block_size=bs)
    arr = np.random.default_rng(1).standard_normal((1, 12, 5)).astype(np.float32)
    helpers["shift/input"] = arr
    helpers["shift/p0_b12"] = extract_shifted_block_logits(arr, prefix_len=0, block_len=12)
    helpers["shift/p4_b8"] = extract_shifted_block_logits(arr, prefix_len=4, block_len=8)
    np.savez_compressed(HERE / "helpers.npz", **helpers)
    make_choices(vm, params, dev, reshape, spec)
    make_edges(vm, params, dev, reshape, spec)


if __name__ == "__main__":
    main()
