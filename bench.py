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
roofline: the projection GEMM (tcgen05) in situ -- every projection launch of an eager 32-row
refinement step at prefix 384 carries its dependency-wait and exit stamps (%globaltimer, programmatic
launch kept); a launch's time is the span from its first CTA passing the wait (its predecessor done)
to its last CTA leaving, so the spans partition the step's critical path and their sum stays under
the step's CUDA-event time.  achieved = algorithmic bytes (weights + activations + outputs) over
that time, against the measured HBM copy bandwidth; per projection and for the attention too.
workloads: BASELINE configs[2] (32 requests per GPU, prompt 512, generate 512), configs[3] (8
requests of prompt 4096, generate 256, split over the GPUs) and configs[4] (1024 sequences of a
512-token context + 16-token continuation scored, batch 64 per GPU) at the same N.
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


# Algorithmic bytes of one projection launch over `rows` token rows (bf16): weights + activations in
# + outputs, as the library counts them (csrc/model.cu gemm_bytes).
H, I, HQKV, V_SLABS = 1536, 8960, 2048, 1187


def _proj_bytes(name: str, rows: int) -> float:
    n, k, out = {"qkv": (HQKV, H, rows * HQKV * 2), "o": (H, H, 2 * rows * H * 2),
                 "gate_up": (2 * I, H, rows * I * 2), "down": (H, I, 2 * rows * H * 2),
                 "lm_head": (151936, H, 16 * rows * V_SLABS)}[name]
    return n * k * 2 + rows * k * 2 + out


def in_situ_step(eng, torch, dev, peak_gbs: float, rows: int = 32, prefix: int = 384, steps: int = 3) -> dict:
    """Critical-path attribution of the eager refinement step (embed, forward_cached, fused lm_head
    + confidence, unmask) at `prefix`, from the always-on launch stamps of the projection and
    attention kernels (fdllm_kernel_trace_*): each launch's span runs from its first CTA past the
    dependency wait to its last CTA's exit.  Median over `steps` steps."""
    from fast_dllm_relax_b200.config import QWEN_MASK_ID
    k, v = eng.new_cache(prefix + BLOCK)
    k.normal_(0, 0.5)
    v.normal_(0, 0.5)
    block = torch.randint(0, 151000, (BLOCK,), device=dev, dtype=torch.int32)
    block[8:] = QWEN_MASK_ID

    def step():
        if rows == BLOCK:
            h = eng.forward_cached(eng.embed(block)[None], k, v, prefix, prefix)
        else:
            h = eng.forward_block_partial(eng.embed(block[8:16])[None], k, v, prefix + 8, prefix, 8)
        i, m = eng.confidence(h)
        eng.unmask(i, m, block.clone(), 8, 8, rows != BLOCK, QWEN_MASK_ID, THRESHOLD)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    eng.kernel_trace_enable(True)
    recs = []
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        stamps, kinds = eng.kernel_trace_read()
        spans = [(int(kd), (int(st[7, 1]) - int(st[1, 0])) / 1e6) for st, kd in zip(stamps, kinds)
                 if st[1, 0] != 0xFFFFFFFFFFFFFFFF and st[7, 1] != 0]
        recs.append((e0.elapsed_time(e1), spans))
    eng.kernel_trace_enable(False)
    step_ms, spans = sorted(recs, key=lambda r: r[0])[len(recs) // 2]
    groups: dict[str, list[float]] = {n: [] for n in ("qkv", "attention", "o", "gate_up", "down", "lm_head")}
    seen_o = False
    for kd, ms in spans:
        base = kd % 1000
        if kd in (1, 2):
            groups["attention"].append(ms)
            seen_o = False
        elif base == 101:
            groups["qkv"].append(ms)
        elif base == 102:
            groups["down" if seen_o else "o"].append(ms)
            seen_o = not seen_o
        elif base == 103:
            groups["gate_up"].append(ms)
        elif base == 105:
            groups["lm_head"].append(ms)
    out: dict = {"rows": rows, "prefix": prefix, "step_ms": step_ms,
                 "stamped_ms": sum(ms for _, ms in spans), "launches": len(spans), "per_kernel": {}}
    gemm_bytes = gemm_ms = 0.0
    for name, ms_list in groups.items():
        if not ms_list:
            continue
        tot = sum(ms_list)
        if name == "attention":
            nbytes = len(ms_list) * ((prefix + BLOCK) * 1024 + 2 * rows * H * 2)
        else:
            nbytes = len(ms_list) * _proj_bytes(name, rows)
            gemm_bytes += nbytes
            gemm_ms += tot
        gbs = nbytes / (tot / 1e3) / 1e9
        out["per_kernel"][name] = {"launches": len(ms_list), "ms": tot, "us_per_launch": 1e3 * tot / len(ms_list),
                                   "gbs": gbs, "frac": gbs / peak_gbs}
    out["gemm"] = {"launches": sum(len(groups[n]) for n in groups if n != "attention"), "ms": gemm_ms,
                   "bytes": gemm_bytes, "gbs": gemm_bytes / (gemm_ms / 1e3) / 1e9 if gemm_ms else None}
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
    ap.add_argument("--headline-only", action="store_true", help="skip the configs[2]-[4] workloads")
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
    peak, peak_kind = _peaks()
    situ = in_situ_step(eng, torch, dev, peak)
    situ_partial = in_situ_step(eng, torch, dev, peak, rows=SUB_BLOCK)
    # BASELINE configs[2]-[4] at this N (every rank runs them; collectives in the same order)
    loads = {} if args.headline_only else workloads(eng, torch, dev, world, rank)

    # off the decode path: max over ranks of the device-timed durations, sum of the work
    (dec_ms, tot_ms, e2e_dec_s, alt_dec_ms), (tokens, launches, e2e_tokens, alt_tokens) = dp.reduce_max_sum(
        [dec_ms, tot_ms, e2e_dec_s, alt_dec_ms], [tokens, launches, e2e_tokens, alt_tokens], device=dev)

    if rank == 0:
        achieved = situ["gemm"]["gbs"] or 0.0
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
            "roofline": {"bound": "hbm", "kernel": "gemm_tc_kernel (tcgen05 projection GEMM, in situ)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak if peak else None, "peak_kind": peak_kind,
                         "traffic": tr.get("bytes_per_launch") if tr else None,
                         "algorithmic_bytes_per_launch": situ["gemm"]["bytes"] / max(1, situ["gemm"]["launches"]),
                         "avg_launch_us": 1e3 * situ["gemm"]["ms"] / max(1, situ["gemm"]["launches"]),
                         "launches": situ["gemm"]["launches"],
                         "timing": "launch stamps inside the eager 32-row step at prefix 384 (programmatic "
                                   "launch kept): first CTA past the dependency wait to last CTA exit",
                         "in_situ": situ, "in_situ_partial": situ_partial},
            "step_roofline": {
                "full": step_roofline(BLOCK, 384, blk["full_ms"], peak, _tensor_peak()[0]),
                "partial": step_roofline(SUB_BLOCK, 384, blk["partial_ms"], peak, _tensor_peak()[0]),
                "bound": "hbm", "peak_kind": f"{peak_kind} / nominal 8 TB/s, 2.25 PFLOP/s"},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "workloads": loads,
        }
        if world == 1 and not args.no_cpu_baseline:
            params_cpu = [p.cpu() for p in params]
            line["cpu_baseline"] = cpu_baseline_sample(params_cpu)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def workloads(eng, torch, dev, world: int, rank: int) -> dict:
    """BASELINE configs[2]-[4] on this engine, data-parallel by request over the ranks (no
    collective while decoding; the max over ranks of the device time and the sum of the work are
    reduced after each).  Device time from CUDA events; decode tokens/s excludes the prefix-cache
    builds (runners.py:748-750)."""
    import numpy as np

    from fast_dllm_relax_b200 import dp
    from fast_dllm_relax_b200.batch_decode import generate_batch
    from fast_dllm_relax_b200.config import QWEN_MASK_ID
    from fast_dllm_relax_b200.scorebench import EOS_ID, score_batch

    out = {}
    kw = dict(mask_id=QWEN_MASK_ID, use_block_cache=False)

    def serve(name, n_total, per_gpu, prompt_len, gen, desc):
        mine = dp.request_range(n_total, world, rank) if per_gpu is None else range(rank * per_gpu, (rank + 1) * per_gpu)
        prompts = [np.random.default_rng(1000 + i).integers(0, 151000, prompt_len).tolist() for i in mine]
        if prompts:
            generate_batch(eng, prompts, max_new_tokens=32, **kw)  # warm-up: allocations, kernels
        torch.cuda.synchronize()
        t = {}
        toks = generate_batch(eng, prompts, max_new_tokens=gen, timing=t, **kw)[0] if prompts else []
        dec = (t["total_ms"] - t["prefill_ms"]) if prompts else 0.0
        (dec_ms, tot_ms, pre_ms), (n_tok, n_req) = dp.reduce_max_sum(
            [dec, t.get("total_ms", 0.0), t.get("prefill_ms", 0.0)], [sum(len(x) for x in toks), len(prompts)],
            device=dev)
        out[name] = {"workload": desc, "metric": "decode tokens/s", "value": n_tok / (dec_ms / 1e3) if dec_ms else None,
                     "unit": "tokens/s", "requests": int(n_req), "tokens": int(n_tok), "decode_ms": dec_ms,
                     "prefill_ms": pre_ms, "total_ms": tot_ms}

    serve("serving", None, 32, 512, 512,
          "BASELINE configs[2]: 1.5B bf16, 32 requests per GPU (prompt 512, generate 512), block 32, threshold 0.9")
    serve("long_prefix", 8, None, 4096, 256,
          "BASELINE configs[3]: 1.5B bf16, 8 requests (prompt 4096, generate 256) split over the GPUs")

    # masked-continuation scoring, 1024 sequences split over the GPUs, batch 64 per GPU
    n_seq, C, N, B = 1024, 512, 16, 64
    mine = list(dp.request_range(n_seq, world, rank))
    n = len(mine)
    g = torch.Generator().manual_seed(2000 + (mine[0] if mine else 0))
    ctx = torch.randint(0, 151000, (n, C), generator=g, dtype=torch.int32).to(dev)
    cont = torch.randint(0, 151000, (n, N), generator=g, dtype=torch.int32)
    blocks = torch.full((n, 32), QWEN_MASK_ID, dtype=torch.int32)
    blocks[:, N] = EOS_ID
    targets = torch.zeros((n, 32), dtype=torch.int32)
    targets[:, :N] = cont
    blocks, targets = blocks.to(dev), targets.to(dev)
    caches = [eng.new_cache(C + 32) for _ in range(min(B, max(n, 1)))]

    def run(lo, hi):
        return [score_batch(eng, caches, ctx[s0:min(s0 + B, hi)], blocks[s0:min(s0 + B, hi)],
                            targets[s0:min(s0 + B, hi)], N) for s0 in range(lo, hi, B)]

    if n:
        run(0, min(n, B))
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    scores = run(0, n)
    e1.record()
    e1.synchronize()
    finite = float(bool(torch.cat(scores).isfinite().all())) if scores else 1.0
    (ms,), (n_all, fin) = dp.reduce_max_sum([e0.elapsed_time(e1)], [n, finite], device=dev)
    out["scoring"] = {"workload": "BASELINE configs[4]: 1.5B bf16, 1024 sequences (context 512 + continuation "
                                  "16) split over the GPUs, batch 64 per GPU, device log-softmax gather",
                      "metric": "scored sequences/s", "value": n_all / (ms / 1e3), "unit": "sequences/s",
                      "sequences": int(n_all), "ms": ms, "scores_finite": fin == world}
    return out


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
