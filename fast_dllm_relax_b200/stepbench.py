"""Time single decode steps of the 1.5B model (the unit the decode loop repeats).

    python -m fast_dllm_relax_b200.stepbench [--steps N] [--prefix P] [--partial] [--requests R] [--phases]

One full refinement step = embed(32) -> 28-layer cached forward (32 rows, prefix P) -> fused lm_head +
confidence -> unmask, as in fast_dllm_relax/runtime.py:376-395 + 796-805; --partial times the 8-row
rp8 step instead (runtime.py:398-436).  --requests R > 1 times the batched scheduler's device step
instead: one batched cached forward of R requests x 32 rows (prefix P each) and one fused confidence
launch over all rows.  Random bf16 weights (seed 1), 3.09 GB on the device.  Also the small,
self-contained case used for ncu captures of single kernels.

--phases also prints, per projection / attention kind, the median over one traced step's launches
of each recorded phase stamp (earliest / latest CTA, microseconds after the launch's first CTA
passed its dependency wait) and the gap from the previous stamped launch's last exit.  The normal
build records phases 1 (past the wait) and 7 (exit); a build with `python -m
fast_dllm_relax_b200.build --ktrace` records the inner phases too (per-tile GEMM: 2 accumulator
ready, 3 drained, 4 split-K summed, 5 epilogue done, 8 TMEM freed; decode attention: 2 key loop
done, 3 partials visible, 4 merge weights, 5 merged).
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
    ap.add_argument("--phases", action="store_true", help="print in-situ phase stamps per kernel kind")
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
    if args.phases:
        eng.kernel_trace_enable(True)
        step()
        torch.cuda.synchronize()
        stamps, kinds = eng.kernel_trace_read()
        eng.kernel_trace_enable(False)
        print_phases(stamps, kinds)


KIND_NAMES = {1: "attention (mma.sync)", 2: "attention (tcgen05)", 101: "qkv", 102: "o / down (residual)",
              103: "gate_up", 104: "logits", 105: "lm_head + confidence", 106: "lm_head + logprob",
              2101: "qkv (fused input norm)", 2103: "gate_up (fused norm)"}


def print_phases(stamps, kinds) -> None:
    """Median phase stamps per kernel kind of one traced step (see the module docstring)."""
    import numpy as np  # noqa: PLC0415
    unset = np.iinfo(np.uint64).max
    rows: dict[int, list] = {}
    gaps: dict[int, list] = {}
    prev_exit = None
    for st, kd in zip(stamps, kinds):
        kd = int(kd)
        if st[1, 0] == unset or st[7, 1] == 0:
            continue
        t0 = int(st[1, 0])
        ph = np.full((st.shape[0], 2), np.nan)
        for q in range(st.shape[0]):
            for j in range(2):
                if st[q, j] not in (0, unset):
                    ph[q, j] = (int(st[q, j]) - t0) / 1e3
        rows.setdefault(kd, []).append(ph)
        if prev_exit is not None:
            gaps.setdefault(kd, []).append((t0 - prev_exit) / 1e3)
        prev_exit = int(st[7, 1])
    for kd, lst in rows.items():
        a = np.stack(lst)
        med = [[float(np.median(a[~np.isnan(a[:, q, j]), q, j])) if (~np.isnan(a[:, q, j])).any() else None
                for j in range(2)] for q in range(a.shape[1])]
        print(json.dumps({"kind": kd, "name": KIND_NAMES.get(kd, str(kd)), "launches": len(lst),
                          "gap_before_us": float(np.median(gaps[kd])) if kd in gaps else None,
                          "phases_us": {str(q): [round(v, 2) for v in m] for q, m in enumerate(med)
                                        if m[1] is not None}}))


if __name__ == "__main__":
    main()
