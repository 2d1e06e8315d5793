"""Time batched prefix-cache builds (the prefill of many requests in one call).

    python -m fast_dllm_relax_b200.prefillbench [--requests N] [--prefix P] [--layers L] [--vocab V]

Each step is one fdllm_build_prefix_cache_batch over N requests of P prompt tokens
(runtime.py:529-548 per request: build_prefix_cache writes the post-RoPE K/V of rows [0, P)).
Random bf16 weights (seed 2) with the 1.5B layer shapes.  --layers and --vocab shrink the model;
2 layers and a 4096-token vocabulary (0.4 GB of weights) is the small case used for ncu
captures of the prefill kernels.
"""

from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from .config import QWEN_1_5B, make_synthetic_params
from .engine import Engine


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requests", type=int, default=8)
    ap.add_argument("--prefix", type=int, default=4096)
    ap.add_argument("--layers", type=int, default=QWEN_1_5B.num_hidden_layers)
    ap.add_argument("--vocab", type=int, default=QWEN_1_5B.vocab_size)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args()
    cfg = dataclasses.replace(QWEN_1_5B, num_hidden_layers=args.layers, vocab_size=args.vocab,
                              context_window_size=max(QWEN_1_5B.context_window_size, args.prefix + 32))
    dev = torch.device("cuda", 0)
    eng = Engine(cfg, make_synthetic_params(cfg, seed=2, dtype="bfloat16", device=dev, mask_id=args.vocab - 1),
                 dtype="bfloat16")
    caches = [eng.new_cache(args.prefix + cfg.bd_size) for _ in range(args.requests)]
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((args.requests * args.prefix, cfg.hidden_size), generator=g, device=dev).to(torch.bfloat16)
    lens = [args.prefix] * args.requests

    for _ in range(args.warmup):
        eng.build_prefix_cache_batch(x, caches, lens)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.build_prefix_cache_batch(x, caches, lens)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    print(json.dumps({"requests": args.requests, "prefix": args.prefix, "layers": args.layers, "vocab": args.vocab,
                      "ms_per_build": ms, "prompt_tokens_per_s": args.requests * args.prefix / ms * 1e3,
                      "device_error": eng.device_error()}))


if __name__ == "__main__":
    main()
