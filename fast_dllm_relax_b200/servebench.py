"""Batched serving throughput of the 1.5B model (BASELINE configs[2] / configs[3] shapes).

    python -m fast_dllm_relax_b200.servebench [--requests 32] [--prompt 512] [--gen 512] [--block-cache]
    torchrun --nproc-per-node N -m fast_dllm_relax_b200.servebench --requests 256 ...

`--requests` is the whole job; ranks take contiguous slices (data-parallel by request, no
collective while decoding) and decode their slice as one batch (fast_dllm_relax_b200.batch_decode).
Random N(0, 0.02) bf16 weights (seed 1), uniform prompts, mask id 151665.  Prints one JSON line:
decode tokens/s over all ranks = generated tokens / (max over ranks of time - prefix-cache time),
the reference's definition (runners.py:748-750).
"""

from __future__ import annotations

import argparse
import datetime
import json

import numpy as np
import torch
import torch.distributed as dist

from . import dp
from .batch_decode import generate_batch
from .config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params
from .engine import Engine


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requests", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--block-cache", action="store_true")
    ap.add_argument("--warmup-gen", type=int, default=32, help="max_new_tokens of the warm-up run")
    args = ap.parse_args()
    world, rank, local = dp.world_info()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device=dev, mask_id=QWEN_MASK_ID)
    eng = Engine(QWEN_1_5B, params, dtype="bfloat16", device=local)
    mine = dp.request_range(args.requests, world, rank)
    prompts = [np.random.default_rng(1000 + i).integers(0, 151000, args.prompt).tolist() for i in mine]
    kw = dict(mask_id=QWEN_MASK_ID, use_block_cache=args.block_cache)
    generate_batch(eng, prompts, max_new_tokens=args.warmup_gen, **kw)  # warm-up (allocations, kernels)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = {}
    toks, stats = generate_batch(eng, prompts, max_new_tokens=args.gen, timing=t, **kw)
    (dec_ms, tot_ms), (n_tok, n_steps) = dp.reduce_max_sum(
        [t["total_ms"] - t["prefill_ms"], t["total_ms"]], [sum(len(x) for x in toks), sum(s["block_recomputes"] for s in stats)],
        device=dev)
    if rank == 0:
        print(json.dumps({"metric": "decode tokens/s (batched serving)", "value": n_tok / (dec_ms / 1e3),
                          "unit": "tokens/s", "n_gpus": world, "requests": args.requests,
                          "requests_per_gpu": len(mine), "prompt": args.prompt, "gen": args.gen,
                          "use_block_cache": args.block_cache, "tokens": int(n_tok), "decode_ms": dec_ms,
                          "total_ms": tot_ms, "forwards": int(n_steps), "dtype": "bf16",
                          "data": "synthetic (random N(0,0.02) weights, uniform prompts)"}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
