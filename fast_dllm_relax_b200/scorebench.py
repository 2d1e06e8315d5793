"""Masked-continuation scoring throughput of the 1.5B model (BASELINE configs[4] shape).

    python -m fast_dllm_relax_b200.scorebench [--sequences 1024] [--context 512] [--cont 16] [--batch 64]
    torchrun --nproc-per-node N -m fast_dllm_relax_b200.scorebench ...

Each sequence follows the reference's scoring path (runtime.py:485-588): its context goes through
`build_prefix_cache`, then a 32-row block holding the continuation as masks, an eos and pad masks
goes through `forward_cached`, and the continuation tokens are scored by log_softmax(logits)[target]
(runners.py:877-881).  Here the prefix builds of `--batch` sequences run as one forward
(fdllm_build_prefix_cache_batch), so do their block forwards, and the log-softmax-gather runs on the device
(fdllm_token_logprob), so only one float per row crosses to the host.  `--sequences` is the whole job;
ranks take contiguous slices (data-parallel, no collective while scoring).  Random N(0, 0.02) bf16
weights (seed 1), uniform token ids.  Prints one JSON line: scored sequences/s over all ranks
(sequences / max over ranks of the device time).
"""

from __future__ import annotations

import argparse
import datetime
import json

import torch
import torch.distributed as dist

from . import dp
from .config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params
from .engine import Engine

EOS_ID = 151643  # a fixed token id after the continuation; the scores do not depend on its meaning


def score_batch(eng: Engine, caches, ctx: torch.Tensor, blocks: torch.Tensor, targets: torch.Tensor,
                n_cont: int) -> torch.Tensor:
    """Sum of the continuation log-probabilities of each sequence of the batch: ctx [b, C] ids,
    blocks [b, 32] ids, targets [b, 32] (the continuation ids in rows [0, n_cont))."""
    b, C = ctx.shape
    eng.build_prefix_cache_batch(eng.embed(ctx.reshape(-1)), caches[:b], [C] * b)
    reqs = [dict(k=k, v=v, rows=32, prefix_len=C) for k, v in caches[:b]]
    hidden = eng.forward_cached_batch(eng.embed(blocks.reshape(-1)), reqs)
    lp = eng.token_logprob(hidden, targets.reshape(-1))
    return lp.view(b, 32)[:, :n_cont].sum(dim=1)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sequences", type=int, default=1024)
    ap.add_argument("--context", type=int, default=512)
    ap.add_argument("--cont", type=int, default=16)
    ap.add_argument("--batch", type=int, default=64, help="sequences per batched block forward")
    args = ap.parse_args()
    if not 0 < args.cont < 32:
        raise ValueError("--cont must leave room for the eos inside the 32-row block")
    world, rank, local = dp.world_info()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device=dev, mask_id=QWEN_MASK_ID)
    eng = Engine(QWEN_1_5B, params, dtype="bfloat16", device=local)
    mine = list(dp.request_range(args.sequences, world, rank))
    n, C, N = len(mine), args.context, args.cont
    g = torch.Generator().manual_seed(2000 + (mine[0] if mine else 0))
    ctx = torch.randint(0, 151000, (n, C), generator=g, dtype=torch.int32).to(dev)
    cont = torch.randint(0, 151000, (n, N), generator=g, dtype=torch.int32)
    blocks = torch.full((n, 32), QWEN_MASK_ID, dtype=torch.int32)
    blocks[:, N] = EOS_ID
    targets = torch.zeros((n, 32), dtype=torch.int32)
    targets[:, :N] = cont
    blocks, targets = blocks.to(dev), targets.to(dev)
    caches = [eng.new_cache(C + 32) for _ in range(min(args.batch, max(n, 1)))]

    def run(lo: int, hi: int) -> list[torch.Tensor]:
        return [score_batch(eng, caches, ctx[s:min(s + args.batch, hi)], blocks[s:min(s + args.batch, hi)],
                            targets[s:min(s + args.batch, hi)], N) for s in range(lo, hi, args.batch)]

    if n:
        run(0, min(n, args.batch))  # warm-up (allocations, kernels)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    scores = run(0, n)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    finite = bool(torch.cat(scores).isfinite().all()) if scores else True
    (ms_max,), (n_all,) = dp.reduce_max_sum([ms], [n], device=dev)
    if rank == 0:
        print(json.dumps({"metric": "scored sequences/s (masked-continuation scoring)", "value": n_all / (ms_max / 1e3),
                          "unit": "sequences/s", "n_gpus": world, "sequences": args.sequences,
                          "sequences_per_gpu": n, "context": C, "continuation": N, "batch": args.batch,
                          "ms": ms_max, "scores_finite": finite, "dtype": "bf16",
                          "data": "synthetic (random N(0,0.02) weights, uniform token ids)"}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
