"""Batched block-diffusion decoding: many requests served together on one GPU.

Each request follows the greedy decode loop of the reference's runtime
(fast_dllm_relax/runtime.py:591-880, `relax_greedy_generate`) exactly: the block-aligned
prompt fast path (:679-708), the prefix-cache rebuild rule (:718-739), the sub-block refinement
loop with the full / partial step choice (:748-805), the stateless first block of short prompts
(:806-837, 862-873), the length and stop checks (:655-669, 839-849) and block-append
(:851-878).  The loop of each request is written as a generator that yields the model work it
needs next; the scheduler gathers the pending work of all requests and runs it together:

* every cached step of every request that needs one (full 32-row refinements, 8-row partial
  refinements, block appends, in any mix) is ONE batched forward (fdllm_forward_cached_batch)
  plus ONE fused lm_head + confidence launch over all rows;
* every pending prefix-cache build is ONE batched forward (fdllm_build_prefix_cache_batch, the
  implicit block-causal mask inside each request, no O(P^2) bias);
* the unmask decision (runtime.py:158-181 shift, 794-805 rule) of every request runs on the
  device in the same step (fdllm_unmask_batch, one warp per request) from the fused confidence
  results; the host reads back, per request, the bit mask of the rows to unmask, their tokens and
  the token after the block (136 bytes), and applies them to its block.

Requests are independent: batching changes which kernels run together, not what any request
computes, up to the bf16 rounding of the larger token tiles.
"""

from __future__ import annotations

import dataclasses
import itertools
from typing import Generator, Sequence

import numpy as np
import torch

from .engine import Engine


@dataclasses.dataclass
class _Cache:
    k: torch.Tensor
    v: torch.Tensor
    prefix_len: int = 0

    @property
    def capacity(self) -> int:
        return int(self.k.shape[2])


# Work items a request program yields (and what it receives back):
#   ("prefill", cache, ids)                      -> None; rows [0, len(ids)) of `cache` written
#   ("step", cache, ids, write_rel, attend_rel, base, win, masked_bits)
#                                                -> (unmasked_bits, last_id, window_tokens): the device
#                                                   decision for window rows [0, win) (window row r takes
#                                                   shifted row base + r); win 0 for a block append
#   ("dense", seq_ids)                           -> float32 logits [len(seq_ids), vocab] (stateless path)

def _id_tensor(seqs, n: int, dev) -> torch.Tensor:
    """The token ids of several requests, concatenated, as int32 on `dev` (one host buffer)."""
    flat = np.fromiter(itertools.chain.from_iterable(seqs), dtype=np.int32, count=n)
    return torch.from_numpy(flat).to(dev)




def request_program(engine: Engine, prompt_ids: Sequence[int], *, max_new_tokens: int, block_size: int,
                    small_block_size: int, threshold: float, use_block_cache: bool, mask_id: int,
                    stop_token: int | None, stats: dict) -> Generator:
    """One request's decode loop (runtime.py:591-880, greedy); returns its continuation."""
    if max_new_tokens < 0:
        raise ValueError("max_new_tokens must be non-negative.")
    bs = block_size
    gen = [int(t) for t in prompt_ids]
    n0 = len(gen)
    cap = -(-(n0 + max_new_tokens) // bs) * bs + bs
    cache: _Cache | None = None
    kv_valid = False

    def new_cache() -> _Cache:
        k, v = engine.new_cache(cap)
        return _Cache(k, v, 0)

    def done_stop(seq, plen):
        if stop_token is None:
            return False
        suf = seq[plen:]
        if stop_token not in suf:
            return False
        return mask_id not in suf[:suf.index(stop_token)]

    def continuation(toks):
        raw = toks[n0:n0 + max_new_tokens]
        fm = next((i for i, t in enumerate(raw) if t == mask_id), len(raw))
        return raw[:fm]

    if n0 % bs == 0 and n0 > 0 and max_new_tokens > 0:  # block-aligned prompt: commit its last block
        lb = n0 - bs
        cache = new_cache()
        if lb > 0:
            yield ("prefill", cache, gen[:lb])
            cache.prefix_len = lb
        _, nxt, _ = yield ("step", cache, gen[lb:], 0, bs, 0, 0, 0)
        cache.prefix_len += bs
        stats["block_recomputes"] += 1
        stats["block_appends"] += 1
        gen.append(nxt)
        if stop_token is not None and nxt == int(stop_token):
            return continuation(gen)

    while len(gen) - n0 < max_new_tokens:
        plen = len(gen)
        x = gen + [mask_id] * (bs - plen % bs)
        a0 = len(x) - bs
        use_cache = a0 != 0
        if use_cache and (cache is None or cache.prefix_len != a0):  # (re)build the prefix cache
            cache = new_cache()
            yield ("prefill", cache, x[:a0])
            cache.prefix_len = a0
            kv_valid = False
        for s0 in range(0, bs, small_block_size):
            s1 = min(bs, s0 + small_block_size)
            while True:
                masked = [i for i, t in enumerate(x[a0 + s0:a0 + s1]) if t == mask_id]
                if not masked:
                    break
                if done_stop(x, plen):
                    return continuation(x)
                if use_cache:
                    partial = use_block_cache and kv_valid and x[a0 + s0] != mask_id
                    bits = sum(1 << r for r in masked)
                    if partial:  # the step's rows are the window itself
                        taken, _, toks = yield ("step", cache, x[a0 + s0:a0 + s1], s0, bs, 0, s1 - s0, bits)
                    else:  # the step's rows are the whole block; the window starts at row s0
                        taken, _, toks = yield ("step", cache, x[a0:], 0, bs, s0, s1 - s0, bits)
                        kv_valid = use_block_cache
                    stats["block_recomputes"] += 1
                    stats["partial_recomputes"] += int(partial)
                    for r in range(s1 - s0):
                        if taken >> r & 1:
                            x[a0 + s0 + r] = toks[r]
                            stats["unmask_updates"] += 1
                else:  # stateless first block (runtime.py:806-837): dense forward over the sequence
                    logits = yield ("dense", x)
                    stats["block_recomputes"] += 1
                    act = logits[-bs:]
                    sh = np.concatenate([act[:1], act[:-1]], axis=0)  # model/cuda.py:180-204
                    small = sh[s0:s1].astype(np.float64)
                    chosen = small.argmax(axis=-1)
                    e = np.exp(small - small.max(axis=-1, keepdims=True))
                    probs = e[np.arange(len(chosen)), chosen] / e.sum(axis=-1)
                    gated = np.full_like(probs, -np.inf)
                    gated[masked] = probs[masked]
                    rows = [r for r in masked if gated[r] > threshold] or [int(np.argmax(gated))]
                    for r in rows:
                        x[a0 + s0 + r] = int(chosen[r])
                    stats["unmask_updates"] += len(rows)
                if len(x) - n0 >= max_new_tokens:
                    break
            if len(x) - n0 >= max_new_tokens:
                break
        gen = x
        if len(gen) - n0 >= max_new_tokens or done_stop(gen, n0):
            break
        if use_cache:  # block-append: the committing forward
            _, nxt, _ = yield ("step", cache, gen[a0:], 0, bs, 0, 0, 0)
            cache.prefix_len += bs
            kv_valid = False
        else:
            logits = yield ("dense", gen)
            nxt = int(np.argmax(logits[-1]))
        stats["block_recomputes"] += 1
        stats["block_appends"] += 1
        gen.append(nxt)
        if stop_token is not None and nxt == int(stop_token):
            break
    return continuation(gen)


def generate_batch(engine: Engine, prompts: Sequence[Sequence[int]], *, max_new_tokens: int,
                   block_size: int = 32, small_block_size: int = 8, threshold: float = 0.9,
                   use_block_cache: bool = False, mask_id: int, stop_token: int | None = None,
                   timing: dict | None = None) -> tuple[list[list[int]], list[dict]]:
    """Decode every prompt; returns (continuations, per-request statistics).  `timing`, when a
    dict, receives total_ms and prefill_ms (the prefix-cache builds), measured with CUDA events."""
    if block_size != engine.cfg.bd_size:
        raise ValueError("block_size must equal the model's bd_size")
    dev = engine.device
    stats = [dict(unmask_updates=0, block_recomputes=0, partial_recomputes=0, block_appends=0) for _ in prompts]
    progs = [request_program(engine, p, max_new_tokens=max_new_tokens, block_size=block_size,
                             small_block_size=small_block_size, threshold=threshold,
                             use_block_cache=use_block_cache, mask_id=mask_id, stop_token=stop_token,
                             stats=st) for p, st in zip(prompts, stats)]
    results: list[list[int] | None] = [None] * len(progs)
    pending: dict[int, tuple] = {}

    def advance(i, value):
        try:
            pending[i] = progs[i].send(value)
        except StopIteration as stop:
            results[i] = list(stop.value)
            pending.pop(i, None)

    ev = []  # (start, end) CUDA event pairs around prefix-cache builds
    staging = None  # pinned host buffer of a step's token ids and unmask descriptors
    t0 = torch.cuda.Event(enable_timing=True) if timing is not None else None
    if t0 is not None:
        t0.record()
    for i in range(len(progs)):
        advance(i, None)
    while pending:
        # every pending prefix-cache build in one forward (fdllm_build_prefix_cache_batch: the
        # block-causal mask inside each request, runtime.py:718-739 per request)
        pre = [i for i, op in pending.items() if op[0] == "prefill"]
        if pre:
            if timing is not None:
                ev.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                ev[-1][0].record()
            ids_all = _id_tensor([pending[i][2] for i in pre], sum(len(pending[i][2]) for i in pre), dev)
            engine.build_prefix_cache_batch(engine.embed(ids_all), [(pending[i][1].k, pending[i][1].v) for i in pre],
                                            [len(pending[i][2]) for i in pre])
            if timing is not None:
                ev[-1][1].record()
            for i in pre:
                advance(i, None)
        # stateless dense forwards (the first block of short prompts): one request at a time
        for i in [i for i, op in pending.items() if op[0] == "dense"]:
            _, seq = pending[i]
            x = engine.embed(torch.tensor(seq, dtype=torch.int32, device=dev))[None]
            hidden = engine.forward_hidden(x, None)
            advance(i, engine.get_logits(hidden)[0].float().cpu().numpy())
        steps = [(i, op) for i, op in pending.items() if op[0] == "step"]
        if not steps:
            continue
        # every pending cached step in one batched forward, one fused confidence launch and one
        # unmask launch; the token ids and the unmask descriptors go up in one copy, from a pinned
        # staging buffer (a copy from pageable memory blocks the host for the whole transfer)
        n_ids = sum(len(op[2]) for _, op in steps)
        need = n_ids + 5 * len(steps)
        if staging is None or staging.numel() < need:
            staging = torch.empty(max(need, 4096), dtype=torch.int32, pin_memory=torch.device(dev).type == "cuda")
        buf = staging.numpy()[:need]
        reqs, o = [], 0
        for j, (_, (_, cache, ids, write_rel, attend_rel, base, win, bits)) in enumerate(steps):
            rows = len(ids)
            buf[o:o + rows] = ids
            buf[n_ids + 5 * j:n_ids + 5 * j + 5] = (o, rows, base, win, bits)
            reqs.append(dict(k=cache.k, v=cache.v, rows=rows, prefix_len=cache.prefix_len, write_rel=write_rel,
                             attend_rel=attend_rel))
            o += rows
        up = staging[:need].to(dev, non_blocking=True)
        hidden = engine.forward_cached_batch(engine.embed(up[:n_ids]), reqs)
        cid, cmax = engine.confidence(hidden)
        dec = engine.unmask_batch(cid, cmax, up[n_ids:].view(len(steps), 5), threshold).cpu().numpy()
        for j, (i, op) in enumerate(steps):
            advance(i, (int(dec[j, 0]), int(dec[j, 1]), dec[j, 2:2 + op[6]].tolist()))
    if timing is not None:
        t1 = torch.cuda.Event(enable_timing=True)
        t1.record()
        t1.synchronize()
        timing["total_ms"] = t0.elapsed_time(t1)
        timing["prefill_ms"] = sum(a.elapsed_time(b) for a, b in ev)
    return results, stats
