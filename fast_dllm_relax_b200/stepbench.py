"""Time single decode steps of the 1.5B model (the unit the decode loop repeats).

    python -m fast_dllm_relax_b200.stepbench [--steps N] [--prefix P] [--partial] [--requests R]

One full refinement step = embed(32) -> 28-layer cached forward (32 rows, prefix P) -> fused lm_head +
confidence -> unmask, as in fast_dllm_relax/runtime.py:376-395 + 796-805; --partial times the 8-row
rp8 step instead (runtime.py:398-436).  --requests R > 1 times the batched scheduler's device step
instead: one batched cached forward of R requests x 32 rows (prefix P each) and one fused confidence
launch over all rows.  Random bf16 weights (seed 1), 3.09 GB on the device.  Also the small,
self-contained case used for ncu captures of single kernels.
"""

from __future__ import annotations

import argparse
import json

import torch

from .config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params
from .engine import Engine


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--prefix", type=int, default=384)
    ap.add_argument("--partial", action="store_true")
    ap.add_argument("--requests", type=int, default=1)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device=dev, mask_id=QWEN_MASK_ID)
    eng = Engine(QWEN_1_5B, params, dtype="bfloat16")
    P, bs = args.prefix, QWEN_1_5B.bd_size
    k, v = eng.new_cache(P + bs)
    k.normal_(0, 0.5)
    v.normal_(0, 0.5)
    block = torch.randint(0, 151000, (bs,), device=dev, dtype=torch.int32)
    block[8:] = QWEN_MASK_ID

    if args.requests > 1:
        reqs = []
        for _ in range(args.requests):
            kr, vr = eng.new_cache(P + bs)
            kr.normal_(0, 0.5)
            vr.normal_(0, 0.5)
            reqs.append(dict(k=kr, v=vr, rows=bs, prefix_len=P))
        bids = torch.randint(0, 151000, (args.requests * bs,), device=dev, dtype=torch.int32)

    def step():
        if args.requests > 1:
            eng.confidence(eng.forward_cached_batch(eng.embed(bids), reqs))
            return
        if args.partial:
            h = eng.forward_block_partial(eng.embed(block[8:16])[None], k, v, P + 8, P, 8)
        else:
            h = eng.forward_cached(eng.embed(block)[None], k, v, P, P)
        ids, maxp = eng.confidence(h)
        eng.unmask(ids, maxp, block.clone(), 8, 8, args.partial, QWEN_MASK_ID, 0.9)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eng.profile_enable(True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    eng.profile_enable(False)
    prof = eng.profile_read()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    gemm_ms = prof["ms"] / max(1, args.steps)
    kind = f"batched_{args.requests}x32" if args.requests > 1 else ("partial_rp8" if args.partial else "full_32")
    print(json.dumps({"step": kind, "prefix": P, "ms_per_step": ms,
                      "gemm_ms_per_step": gemm_ms, "gemm_GBps": prof["bytes"] / max(prof["ms"], 1e-9) / 1e6,
                      "gemm_launches_per_step": prof["launches"] / max(1, args.steps),
                      "device_error": eng.device_error()}))


if __name__ == "__main__":
    main()
