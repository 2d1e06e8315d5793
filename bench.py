"""Benchmark: Fast-dLLM v2 block-diffusion decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--block-cache]

Workload: the 1.5B architecture (28 layers, hidden 1536, 12/2 heads of 128,
SwiGLU 8960, vocab 151936, tied embeddings) in bf16 with random N(0, 0.02) weights (seed 1; RMSNorm
weights 1.0; the mask id's embedding row zeroed so greedy decoding never emits the mask), batch 1,
a 256-token prompt drawn uniformly from [0, 151000), 256 new tokens, 32-token blocks refined in
8-token sub-blocks, threshold 0.9.  One "step" is one whole generation of one request on each GPU
(data-parallel by request, no collective on the path: weak scaling).  The weights (3.09 GB) are far
larger than L2, so every step streams them from HBM.

value: decode tokens/s over all ranks = generated tokens / (generation time - prefill time), the
reference's definition (fast_dllm_relax/runners.py:748-750), with device time from CUDA events
inside the native driver (the max over ranks).  e2e: the same metric through the public call
(Engine.generate: host prompt in, host tokens out, per-step host reads) on the host clock.
roofline: the projection GEMM (tcgen05) -- algorithmic bytes (weights + activations + outputs) per
launch over its CUDA-event duration, against the measured HBM copy bandwidth.
step_roofline: one whole 32-row (and 8-row partial) refinement step at prefix 384 -- the slower of
(weights + KV bytes) / HBM and FLOPs / bf16 tensor peak, over the step's CUDA-event time, against
the measured peaks and the nominal 8 TB/s and 2.25 PFLOP/s.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tokens/s (Fast-dLLM v2 1.5B block-diffusion decode, batch 1 per GPU)"
UNIT = "tokens/s"
PROMPT_LEN, GEN_LEN, BLOCK, SUB_BLOCK, THRESHOLD = 256, 256, 32, 8, 0.9


PEAKS_FILE = REPO / "MEASURED_PEAKS.json"  # written by the measuring driver on each pod
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}  # an earlier measurement on this pool


def _peak(key: str, path: Path | None = None) -> tuple[float, str]:
    """The measured peak `key` from the peaks file, else the fallback figure (and which it is)."""
    p = PEAKS_FILE if path is None else path
    try:
        val = json.loads(p.read_text()).get(key)
        if isinstance(val, (int, float)) and val > 0:
            return float(val), "measured"
    except (OSError, ValueError, AttributeError):
        pass
    return FALLBACK_PEAKS[key], "fallback"


def _peaks() -> tuple[float, str]:
    return _peak("hbm_gbs")


def _tensor_peak() -> tuple[float, str]:
    return _peak("bf16_tflops")


# 1.5B bf16 algorithmic units of one refinement step (weights incl. biases and norms, tied lm_head)
STEP_WEIGHT_BYTES = 3_087_428_608
STEP_MACS_PER_ROW = 1_543_569_408
KV_BYTES_PER_KEY = 28 * 2 * 2 * 128 * 2  # layers x (K, V) x kv heads x head_dim x bf16


def step_roofline(rows: int, prefix: int, ms: float, hbm_gbs: float, tensor_tflops: float) -> dict:
    """Whole-step roofline of one refinement forward of `rows` query rows attending prefix + 32 keys:
    the slower of (weights + KV reads + KV writes) / HBM and FLOPs / bf16 tensor peak, over the
    measured step time."""
    keys = prefix + BLOCK
    nbytes = STEP_WEIGHT_BYTES + KV_BYTES_PER_KEY * keys + KV_BYTES_PER_KEY * rows
    flops = 2 * rows * STEP_MACS_PER_ROW + 28 * 12 * 4 * 128 * rows * keys
    out = {"rows": rows, "prefix": prefix, "bytes": nbytes, "flops": flops, "ms": ms}
    for tag, bw, tf in (("measured", hbm_gbs, tensor_tflops), ("nominal", 8000.0, 2250.0)):
        floor_ms = max(nbytes / (bw * 1e9), flops / (tf * 1e12)) * 1e3
        out[tag] = {"hbm_gbs": bw, "bf16_tflops": tf, "floor_ms": floor_ms,
                    "frac": floor_ms / ms if ms > 0 else None}
    return out


def _traffic() -> dict | None:
    """DRAM bytes per projection-GEMM launch (dram__bytes_read.sum + dram__bytes_write.sum from
    one ncu capture), from the committed summary's `bytes_per_launch:` line."""
    p = REPO / "profiles" / "gemm_tc_kernel_1p5b_p384.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("bytes_per_launch:"):
            return {"bytes_per_launch": float(line.split(":", 1)[1])}
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.gpu], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    from fast_dllm_relax_b200.dp import world_info
    return world_info()


def make_prompt(seed: int) -> list[int]:
    import numpy as np
    return np.random.default_rng(seed).integers(0, 151000, PROMPT_LEN).tolist()


def cpu_baseline_sample(params_cpu, steps: int = 2) -> dict:
    """The oracle (PyTorch CPU restatement of the reference graph) timed on the host cores:
    full 32-row refinement steps (forward_cached + get_logits + confidence) at P = 256."""
    import torch

    from fast_dllm_relax_b200.config import QWEN_1_5B as cfg
    from oracle.model import OracleConfig, OracleModel, confidence

    torch.set_num_threads(os.cpu_count() or 1)
    orc = OracleModel(OracleConfig(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                                   cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rms_norm_eps,
                                   cfg.rope_theta, cfg.tie_word_embeddings, cfg.bd_size), params_cpu, "bfloat16")
    P = PROMPT_LEN
    g = torch.Generator().manual_seed(0)
    shape = (cfg.num_hidden_layers, 1, P + BLOCK, cfg.num_key_value_heads, cfg.head_dim)
    k = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)  # a prefix cache's worth of K/V
    v = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.randint(0, 151000, (BLOCK,), generator=g)
    times = []
    for _ in range(steps + 1):
        t0 = time.perf_counter()
        h = orc.forward_cached(orc.embed(ids)[None], k, v, P, P)
        confidence(orc.get_logits(h)[0])
        times.append(time.perf_counter() - t0)
    ms = statistics.median(times[1:]) * 1e3
    return {"value": 1000.0 / ms, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} full 32-row refinement steps of the 1.5B model at prefix 256 (after 1 warm-up), "
                      f"{ms:.0f} ms/step; with random weights each refinement step commits one token",
            "ms_per_step": ms}


def workload_config(world: int, block_cache: bool) -> dict:
    """The `config` object both arms print (same workload, same keys)."""
    return {"workload": "BASELINE configs[1]: Fast-dLLM v2 1.5B bf16, batch 1 per GPU, prompt 256, "
                        "generate 256, block 32, sub-block 8, threshold 0.9",
            "use_block_cache": bool(block_cache), "parallelism": f"dp{world} (requests)",
            "l2": "inputs larger than L2: 3.09 GB of weights streamed per step"}


def run_reference(args) -> None:
    """--impl reference: the oracle port on the host cores (the reference's own stack, TVM Relax +
    the checkpoint's remote code, cannot run here), rank 0 only."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    import torch

    from fast_dllm_relax_b200.config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params

    torch.set_num_threads(os.cpu_count() or 1)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device="cpu", mask_id=QWEN_MASK_ID)
    warm = max(0, args.warmup)
    steps = max(1, args.steps)
    base = cpu_baseline_sample(params, steps=1)  # builds the oracle once; one warm + one timed step
    # Each bench step is one refinement step (a bounded sample of the generation).
    from oracle.model import OracleConfig, OracleModel, confidence
    cfg = QWEN_1_5B
    orc = OracleModel(OracleConfig(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                                   cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rms_norm_eps,
                                   cfg.rope_theta, cfg.tie_word_embeddings, cfg.bd_size), params, "bfloat16")
    g = torch.Generator().manual_seed(0)
    shape = (cfg.num_hidden_layers, 1, PROMPT_LEN + BLOCK, cfg.num_key_value_heads, cfg.head_dim)
    k = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(shape, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.randint(0, 151000, (BLOCK,), generator=g)

    # use_block_cache=True refines with 8-row partial steps (write_rel 8, attend the full block)
    rows = 8 if args.block_cache else BLOCK

    def one():
        if rows == BLOCK:
            h = orc.forward_cached(orc.embed(ids)[None], k, v, PROMPT_LEN, PROMPT_LEN)
        else:
            h = orc.forward_block_partial(orc.embed(ids[8:16])[None], k, v, PROMPT_LEN + 8, PROMPT_LEN, 8)
        confidence(orc.get_logits(h)[0])

    for _ in range(warm):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    el = time.perf_counter() - t0
    ms = el * 1e3 / steps
    value = 1000.0 / ms
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": workload_config(world, args.block_cache),
        "sample": f"one {rows}-row refinement step per bench step (1 token committed per step)",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{steps} {rows}-row refinement steps at prefix 256 on the host cores; "
                                   "oracle/ is the PyTorch CPU restatement of the reference graph "
                                   "(TVM Relax cannot be installed here)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "first_step_ms": base["ms_per_step"],
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--block-cache", action="store_true", help="use_block_cache=True (partial 8-row steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    from fast_dllm_relax_b200.config import QWEN_1_5B, QWEN_MASK_ID, make_synthetic_params
    from fast_dllm_relax_b200 import dp
    from fast_dllm_relax_b200.engine import Engine

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    params = make_synthetic_params(QWEN_1_5B, seed=1, dtype="bfloat16", device=dev, mask_id=QWEN_MASK_ID)
    eng = Engine(QWEN_1_5B, params, dtype="bfloat16", device=local)
    # batch 1 per GPU: the job is `world` requests, cut into one contiguous range per rank
    (req,) = dp.request_range(world, world, rank)
    prompt = make_prompt(1000 + req)
    gen_kw = dict(max_new_tokens=GEN_LEN, block_size=BLOCK, small_block_size=SUB_BLOCK, threshold=THRESHOLD,
                  use_block_cache=args.block_cache, mask_id=QWEN_MASK_ID, stop_token=None)

    for _ in range(max(args.warmup, 0)):
        eng.generate(prompt, **gen_kw)
    torch.cuda.synchronize()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_idx = vis.split(",")[local] if vis else str(local)
    tokens = 0
    dec_ms = tot_ms = 0.0
    stats_acc = None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = Engine.kernel_launches()
    with ClockSampler(gpu_idx) as clk:
        for _ in range(args.steps):
            t = {}
            toks, st = eng.generate(prompt, timing=t, **gen_kw)
            tokens += len(toks)
            dec_ms += t["total_ms"] - t["prefill_ms"]
            tot_ms += t["total_ms"]
            stats_acc = st
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    launches = Engine.kernel_launches() - launches0

    # Roofline of the dominant kernel: one more generation with a CUDA-event pair around every
    # projection-GEMM launch (captured as event nodes of the step graphs).  Timed apart from the
    # headline run because the event nodes break the programmatic overlap between kernels.
    eng.profile_enable(True)
    eng.generate(prompt, **gen_kw)  # captures the profiled step graphs
    eng.profile_read()
    eng.generate(prompt, **gen_kw)
    torch.cuda.synchronize()
    eng.profile_enable(False)
    prof = eng.profile_read()

    # e2e: the same generations through the public call on the host clock (pinned-free host lists)
    torch.cuda.synchronize()
    e2e_tokens, e2e_dec_s, e2e_pref_ms = 0, 0.0, 0.0
    for _ in range(args.steps):
        t = {}
        w0 = time.perf_counter()
        toks, _ = eng.generate(prompt, timing=t, **gen_kw)
        w = time.perf_counter() - w0
        e2e_tokens += len(toks)
        e2e_dec_s += w - t["prefill_ms"] / 1e3
    # the other use_block_cache setting, device-timed the same way (the reference evaluates with
    # use_block_cache=True, scripts/eval.sh:50; the headline keeps BASELINE's default)
    alt_kw = dict(gen_kw, use_block_cache=not args.block_cache)
    eng.generate(prompt, **alt_kw)  # captures that setting's step graphs
    alt_tokens, alt_dec_ms = 0, 0.0
    for _ in range(args.steps):
        t = {}
        toks, _ = eng.generate(prompt, timing=t, **alt_kw)
        alt_tokens += len(toks)
        alt_dec_ms += t["total_ms"] - t["prefill_ms"]
    # ms per 32-token block step (embed + forward_cached(32) + fused confidence + unmask) at P = 384
    blk = block_step_ms(eng, torch, dev)

    # off the decode path: max over ranks of the device-timed durations, sum of the work
    (dec_ms, tot_ms, e2e_dec_s, alt_dec_ms), (tokens, launches, e2e_tokens, alt_tokens) = dp.reduce_max_sum(
        [dec_ms, tot_ms, e2e_dec_s, alt_dec_ms], [tokens, launches, e2e_tokens, alt_tokens], device=dev)

    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = prof["bytes"] / (prof["ms"] / 1e3) / 1e9 if prof["ms"] > 0 else 0.0
        tr = _traffic()
        steps_per_gen = stats_acc["block_recomputes"] if stats_acc else 0
        n_blocks = (stats_acc["block_appends"] + 1) if stats_acc else 0
        h2d = 4 * PROMPT_LEN + 4 * BLOCK * n_blocks
        d2h = 4 * (2 + 64) * (steps_per_gen - (stats_acc["block_appends"] if stats_acc else 0)) + 4 * n_blocks
        line = {
            "metric": METRIC, "value": tokens / (dec_ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tot_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random N(0,0.02) weights, uniform prompts)",
            "config": workload_config(world, args.block_cache),
            "tokens_per_generation": tokens / max(1, args.steps * world),
            "refinement_forwards_per_generation": steps_per_gen,
            "ms_per_block_step": blk["full_ms"], "ms_per_partial_step": blk["partial_ms"],
            "ms_per_append_step": blk["append_ms"],
            "other_block_cache_setting": {"use_block_cache": not args.block_cache,
                                          "value": alt_tokens / (alt_dec_ms / 1e3) if alt_dec_ms > 0 else None,
                                          "unit": UNIT},
            "prefill_ms": (tot_ms - dec_ms) / args.steps,
            "e2e": {"value": e2e_tokens / e2e_dec_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "path": "Engine.generate -> fdllm_generate (host buffers)"},
            "roofline": {"bound": "hbm", "kernel": "gemm_tc_kernel (tcgen05 projection GEMM)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak if peak else None, "peak_kind": peak_kind,
                         "traffic": tr.get("bytes_per_launch") if tr else None,
                         "algorithmic_bytes_per_launch": prof["bytes"] / max(1, prof["launches"]),
                         "avg_launch_us": 1e3 * prof["ms"] / max(1, prof["launches"]),
                         "launches": prof["launches"]},
            "step_roofline": {
                "full": step_roofline(BLOCK, 384, blk["full_ms"], peak, _tensor_peak()[0]),
                "partial": step_roofline(SUB_BLOCK, 384, blk["partial_ms"], peak, _tensor_peak()[0]),
                "bound": "hbm", "peak_kind": f"{peak_kind} / nominal 8 TB/s, 2.25 PFLOP/s"},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            params_cpu = [p.cpu() for p in params]
            line["cpu_baseline"] = cpu_baseline_sample(params_cpu)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def block_step_ms(eng, torch, dev, iters: int = 20) -> dict:
    """CUDA-event time of one full refinement step, one rp8 partial step and one block append
    (the 32-row cached forward alone) at P = 384."""
    from fast_dllm_relax_b200.config import QWEN_MASK_ID
    P = 384
    k, v = eng.new_cache(P + BLOCK)
    k.normal_(0, 0.5)
    v.normal_(0, 0.5)
    ids = torch.randint(0, 151000, (BLOCK,), device=dev, dtype=torch.int32)
    block = ids.clone()
    block[8:] = QWEN_MASK_ID

    def full():
        h = eng.forward_cached(eng.embed(block)[None], k, v, P, P)
        i, m = eng.confidence(h)
        eng.unmask(i, m, block.clone(), 8, 8, False, QWEN_MASK_ID, THRESHOLD)

    def partial():
        h = eng.forward_block_partial(eng.embed(block[8:16])[None], k, v, P + 8, P, 8)
        i, m = eng.confidence(h)
        eng.unmask(i, m, block.clone(), 8, 8, True, QWEN_MASK_ID, THRESHOLD)

    def append():  # the committed block written into the cache (runtime.py's block append)
        eng.forward_cached(eng.embed(ids)[None], k, v, P, P)

    out = {}
    for name, fn in (("full_ms", full), ("partial_ms", partial), ("append_ms", append)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        out[name] = e0.elapsed_time(e1) / iters
    return out


if __name__ == "__main__":
    main()
