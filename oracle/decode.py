"""CPU oracle for the reference's decode loop and scoring (fast_dllm_relax/runtime.py).

TEST INFRASTRUCTURE ONLY (see oracle/model.py's header for the import rule).

A restatement of the host-side semantics of the reference runtime over `OracleModel`, used as the
checker for the product's native decode driver and its Python runtime:

* `PrefixCache` / capacity rule              runtime.py:206-255, 653
* `_check_write`                             runtime.py:258-263
* `build_prefix_cache_from_ids` (+chunked)   runtime.py:266-323
* `shifted_confidence` (host torch path)     runtime.py:158-181
* step scorers                               runtime.py:333-436
* `score_sequence_block`                     runtime.py:439-482, model/cuda.py:180-204
* `score_masked_continuation`                runtime.py:485-588
* `relax_greedy_generate`                    runtime.py:591-880
* loglikelihood reduction                    runners.py:877-881

This module's outputs are pinned against the reference's own runtime.py, driven by the same
oracle arithmetic through a TVM stand-in, by the fixtures in tests/golden/ (make_golden.py).
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch

from .model import OracleModel, build_block_bias


@dataclasses.dataclass
class PrefixCache:
    k: torch.Tensor  # [layers, 1, cap, kv_heads, head_dim]
    v: torch.Tensor
    prefix_len: int

    @property
    def capacity(self) -> int:
        return int(self.k.shape[2])

    def commit(self, rows: int) -> None:
        if self.prefix_len + rows > self.capacity:
            raise ValueError(f"commit past capacity: {self.prefix_len} + {rows} > {self.capacity}")
        self.prefix_len += rows

    def ensure_capacity(self, rows: int, model: OracleModel) -> None:
        if rows <= self.capacity:
            return
        bigger = allocate_prefix_cache(model, rows)
        bigger.k[:, :, :self.prefix_len] = self.k[:, :, :self.prefix_len]
        bigger.v[:, :, :self.prefix_len] = self.v[:, :, :self.prefix_len]
        self.k, self.v = bigger.k, bigger.v


def allocate_prefix_cache(model: OracleModel, rows: int, block_size: int = 32) -> PrefixCache:
    cfg = model.cfg
    cap = -(-max(int(rows), 1) // block_size) * block_size
    shape = (cfg.num_hidden_layers, 1, cap, cfg.num_key_value_heads, cfg.head_dim)
    return PrefixCache(torch.zeros(shape, dtype=model.dtype), torch.zeros(shape, dtype=model.dtype), 0)


def _check_write(cache: PrefixCache, write_start: int, attend_len: int) -> None:
    if write_start < cache.prefix_len:
        raise ValueError(f"KV write at row {write_start} would overwrite the committed prefix [0, {cache.prefix_len})")
    if attend_len > cache.capacity:
        raise ValueError(f"cached call needs {attend_len} rows; cache capacity is {cache.capacity}")


def _embed(model: OracleModel, ids) -> torch.Tensor:
    return model.embed(torch.as_tensor(np.asarray(ids, dtype=np.int32)))[None]


def _prefill(model: OracleModel, ids, cache: PrefixCache, block_size: int) -> None:
    if cache.prefix_len != 0:
        raise ValueError("build_prefix_cache writes from row 0; the cache already has a prefix")
    _check_write(cache, 0, len(ids))
    bias = build_block_bias(0, len(ids), block_size)
    model.build_prefix_cache(_embed(model, ids), bias, cache.k, cache.v)
    cache.commit(len(ids))


def _forward_cached(model: OracleModel, ids, cache: PrefixCache) -> torch.Tensor:
    _check_write(cache, cache.prefix_len, cache.prefix_len + len(ids))
    return model.forward_cached(_embed(model, ids), cache.k, cache.v, cache.prefix_len, cache.prefix_len)


def build_prefix_cache_from_ids(model: OracleModel, prefix_ids, *, block_size: int,
                                capacity: int | None = None, chunked_prefill: bool = False) -> PrefixCache:
    P = len(prefix_ids)
    cache = allocate_prefix_cache(model, max(P, capacity or 0), block_size)
    if P == 0:
        return cache
    if chunked_prefill and P > block_size:
        if P % block_size != 0:
            raise ValueError("chunked_prefill requires a block-aligned prefix")
        _prefill(model, prefix_ids[:block_size], cache, block_size)
        for s in range(block_size, P, block_size):
            _forward_cached(model, prefix_ids[s:s + block_size], cache)
            cache.commit(block_size)
        return cache
    _prefill(model, prefix_ids, cache, block_size)
    return cache


def shifted_confidence(model: OracleModel, hidden: torch.Tensor):
    """Host torch path of runtime.py:176-181."""
    logits = model.get_logits(hidden)
    shifted = torch.cat([logits[:, :1, :], logits[:, :-1, :]], dim=1)
    ids = shifted.argmax(dim=-1)[0].numpy()
    maxp = shifted.softmax(dim=-1).max(dim=-1).values[0].numpy()
    return ids, maxp, int(logits[0, -1, :].argmax().item())


def score_sequence_block(model: OracleModel, seq_ids, *, block_size: int):
    if len(seq_ids) <= block_size:
        pre, act = [], list(seq_ids)
    else:
        plen = ((len(seq_ids) - 1) // block_size) * block_size
        pre, act = seq_ids[:plen], seq_ids[plen:]
    bias = build_block_bias(len(pre), len(act), block_size)
    hidden = model.forward_hidden(_embed(model, list(pre) + list(act)), bias)
    logits = model.get_logits(hidden).numpy()
    cur = logits[:, -len(act):, :]
    p = len(pre)
    src = ([p - 1] + list(range(p, p + len(act) - 1))) if p > 0 else ([0] + list(range(0, len(act) - 1)))
    return cur, logits[:, src, :]


def score_masked_continuation(model: OracleModel, prefix_ids, continuation_ids, *, block_size: int,
                              mask_id: int, eos_token_id: int | None = None, cached_prefix=None,
                              chunked_prefill: bool = False):
    if not continuation_ids:
        return np.empty((0, 0), dtype=np.float32), cached_prefix
    plen = (len(prefix_ids) // block_size) * block_size
    if plen == 0:
        seq = list(prefix_ids) + [mask_id] * len(continuation_ids)
        _, shifted = score_sequence_block(model, seq, block_size=block_size)
        return shifted[0, -len(continuation_ids):, :], None
    aligned = list(prefix_ids[:plen])
    tail_rows = max(len(prefix_ids) - plen + len(continuation_ids), block_size)
    if cached_prefix is not None and cached_prefix[0] == aligned:
        cache = cached_prefix[1]
        cache.ensure_capacity(plen + tail_rows, model)
    else:
        cache = build_prefix_cache_from_ids(model, aligned, block_size=block_size,
                                            capacity=plen + tail_rows, chunked_prefill=chunked_prefill)
    real = list(prefix_ids[cache.prefix_len:])
    active = real + [mask_id] * len(continuation_ids)
    if len(active) <= block_size:
        pad = block_size - len(active)
        if pad:
            active = active + [mask_id] * pad
            if eos_token_id is not None:
                active[len(real) + len(continuation_ids)] = eos_token_id
    hidden = _forward_cached(model, active, cache)
    logits = model.get_logits(hidden)
    shifted = torch.cat([logits[:, :1, :], logits[:, :-1, :]], dim=1)
    end = len(real) + len(continuation_ids)
    return shifted[0, len(real):end, :].numpy(), (aligned, cache)


def loglikelihood(logits_rows: np.ndarray, continuation_ids) -> float:
    """runners.py:877-881: log_softmax over fp32 rows, gather the continuation ids, sum."""
    lp = torch.log_softmax(torch.from_numpy(np.asarray(logits_rows, dtype=np.float32)), dim=-1)
    tgt = torch.tensor(list(continuation_ids))
    return float(lp.gather(-1, tgt.unsqueeze(-1)).squeeze(-1).sum().item())


def relax_greedy_generate(model: OracleModel, prompt_ids, *, max_new_tokens: int, block_size: int = 32,
                          small_block_size: int = 8, threshold: float = 0.9, use_block_cache: bool = False,
                          mask_id: int, stop_token: int | None = None, chunked_prefill: bool = False,
                          trace: list | None = None):
    """runtime.py:591-880 (greedy; temperature 0).  `trace`, when a list, receives one
    (kind, sub_block_start, rows_unmasked) tuple per refinement step."""
    if max_new_tokens < 0:
        raise ValueError("max_new_tokens must be non-negative.")
    gen = list(prompt_ids)
    n0 = len(gen)
    st = dict(unmask_updates=0, block_recomputes=0, partial_recomputes=0, block_appends=0)
    cache: PrefixCache | None = None
    kv_valid = False
    cap = -(-(n0 + max_new_tokens) // block_size) * block_size + block_size

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

    if n0 % block_size == 0 and n0 > 0 and max_new_tokens > 0:
        lb = n0 - block_size
        cache = build_prefix_cache_from_ids(model, gen[:lb], block_size=block_size, capacity=cap,
                                            chunked_prefill=chunked_prefill)
        hidden = _forward_cached(model, gen[lb:], cache)
        cache.commit(block_size)
        _, _, nxt = shifted_confidence(model, hidden)
        st["block_recomputes"] += 1
        st["block_appends"] += 1
        gen.append(nxt)
        if stop_token is not None and nxt == int(stop_token):
            return continuation(gen), st

    while len(gen) - n0 < max_new_tokens:
        plen = len(gen)
        x = gen + [mask_id] * (block_size - plen % block_size)
        a0 = len(x) - block_size
        if a0 == 0:
            use_cache = False
        else:
            use_cache = True
            cur = cache.prefix_len if cache is not None else 0
            if a0 != cur:
                cache = build_prefix_cache_from_ids(model, x[:a0], block_size=block_size, capacity=cap,
                                                    chunked_prefill=chunked_prefill)
                kv_valid = False
        for s0 in range(0, block_size, small_block_size):
            s1 = min(block_size, s0 + small_block_size)
            while True:
                masked = [i for i, t in enumerate(x[a0 + s0:a0 + s1]) if t == mask_id]
                if not masked:
                    break
                if done_stop(x, plen):
                    return continuation(x), st
                if use_cache:
                    partial = use_block_cache and kv_valid and x[a0 + s0] != mask_id
                    if partial:
                        ids = x[a0 + s0:a0 + s1]
                        ws = cache.prefix_len + s0
                        _check_write(cache, ws, cache.prefix_len + block_size)
                        hidden = model.forward_block_partial(_embed(model, ids), cache.k, cache.v, ws,
                                                             cache.prefix_len, s0)
                        tok, prob, _ = shifted_confidence(model, hidden)
                    else:
                        hidden = _forward_cached(model, x[a0:], cache)
                        tok, prob, _ = shifted_confidence(model, hidden)
                        kv_valid = use_block_cache
                        tok, prob = tok[s0:s1], prob[s0:s1]
                    st["block_recomputes"] += 1
                    if partial:
                        st["partial_recomputes"] += 1
                    rows = [r for r in masked if prob[r] > threshold]
                    if not rows:
                        rows = [masked[int(np.argmax([prob[r] for r in masked]))]]
                    for r in rows:
                        x[a0 + s0 + r] = int(tok[r])
                        st["unmask_updates"] += 1
                    if trace is not None:
                        trace.append(("partial" if partial else "full", s0, list(rows)))
                else:
                    _, sh = score_sequence_block(model, x, block_size=block_size)
                    st["block_recomputes"] += 1
                    small = sh[:, s0:s1, :][0]
                    chosen = small.argmax(axis=-1)
                    probs = np.empty(small.shape[0], dtype=np.float64)
                    for r in range(small.shape[0]):
                        row = small[r].astype(np.float64)
                        e = np.exp(row - row.max())
                        probs[r] = e[chosen[r]] / e.sum()
                    gated = np.full_like(probs, -np.inf)
                    for r in masked:
                        gated[r] = probs[r]
                    rows = [r for r in masked if gated[r] > threshold]
                    if not rows:
                        rows = [int(np.argmax(gated))]
                    for r in rows:
                        x[a0 + s0 + r] = int(chosen[r])
                        st["unmask_updates"] += 1
                    if trace is not None:
                        trace.append(("stateless", s0, list(rows)))
                if len(x) - n0 >= max_new_tokens:
                    break
            if len(x) - n0 >= max_new_tokens:
                break
        gen = x
        if len(gen) - n0 >= max_new_tokens:
            break
        if done_stop(gen, n0):
            break
        if use_cache:
            hidden = _forward_cached(model, gen[a0:], cache)
            cache.commit(len(gen) - a0)
            _, _, nxt = shifted_confidence(model, hidden)
            kv_valid = False
        else:
            cur_logits, _ = score_sequence_block(model, gen, block_size=block_size)
            nxt = int(cur_logits[0, -1, :].argmax())
        st["block_recomputes"] += 1
        gen.append(nxt)
        st["block_appends"] += 1
        if stop_token is not None and nxt == int(stop_token):
            break
    return continuation(gen), st
