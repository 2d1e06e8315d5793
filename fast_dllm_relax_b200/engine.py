"""PyTorch-facing wrapper of the sm_100a library: the nine entry points of the reference's compiled
module over torch CUDA tensors, plus the batched, fused-confidence, unmask, log-prob and native
decode calls.  PyTorch only owns memory and supplies the current stream; all compute happens in the
library's kernels.

Entry points and the reference interfaces they replace (fast_dllm_relax/model/cuda.py):
    embed                      :698-699   (spec :810-813)
    forward_hidden             :701-702   (spec :814-818)
    get_logits                 :704-711   (spec :819-822)
    build_prefix_cache         :713-721   (spec :823-829)
    forward_cached             :723-738   (spec :830-837)
    forward_block_partial_rpN  :740-788   (spec :801-808)
"""

from __future__ import annotations

import ctypes
import weakref
from typing import Sequence

import torch

from . import _lib
from .config import ModelConfig

_DT = {"float32": (torch.float32, 0), "bfloat16": (torch.bfloat16, 1)}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class Engine:
    """One library handle on one CUDA device with a bound parameter list."""

    def __init__(self, cfg: ModelConfig, params: Sequence[torch.Tensor], dtype: str = "bfloat16",
                 device: int | torch.device | None = None, max_positions: int | None = None):
        if dtype not in _DT:
            raise ValueError(f"unsupported dtype {dtype}")
        self.cfg = cfg
        self.dtype_name = dtype
        self.dtype, code = _DT[dtype]
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", torch.device(device).index if isinstance(device, torch.device) else int(device))
        self.lib = _lib.load()
        self._cache_ok: dict = {}  # id(k) -> (ref(k), ref(v), shape): caches validated before
        c = _lib.FdllmConfig(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                             cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rms_norm_eps,
                             cfg.rope_theta, int(cfg.tie_word_embeddings), cfg.bd_size,
                             int(max_positions or cfg.context_window_size), code)
        h = ctypes.c_void_p()
        _lib.check(self.lib.fdllm_create(ctypes.byref(c), self.device.index, ctypes.byref(h)))
        self._h = h
        self.bind(params)

    def bind(self, params: Sequence[torch.Tensor]) -> None:
        ps = []
        for i, p in enumerate(params):
            if p.device != self.device or p.dtype != self.dtype or not p.is_contiguous():
                raise ValueError(f"param {i}: expected a contiguous {self.dtype} tensor on {self.device}")
            ps.append(p)
        self._params = list(ps)  # keep the storage alive while bound
        arr = (ctypes.c_void_p * len(ps))(*[p.data_ptr() for p in ps])
        _lib.check(self.lib.fdllm_bind_params(self._h, arr, len(ps)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.fdllm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    # ---- helpers ---------------------------------------------------------------------------
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _act(self, x: torch.Tensor, name: str) -> torch.Tensor:
        if x.dim() == 3:
            if x.shape[0] != 1:
                raise ValueError(f"{name}: batch dimension must be 1, got {tuple(x.shape)}")
            x = x[0]
        if x.dim() != 2 or x.shape[1] != self.cfg.hidden_size:
            raise ValueError(f"{name}: expected [rows, {self.cfg.hidden_size}], got {tuple(x.shape)}")
        if x.device != self.device or x.dtype != self.dtype:
            raise ValueError(f"{name}: expected {self.dtype} on {self.device}")
        return x.contiguous()

    def _cache(self, k: torch.Tensor, v: torch.Tensor) -> int:
        """Validate a K/V cache pair; returns its capacity.  A pair that passed before is known by
        identity (weak references confirm the same objects) and unchanged shape, so a scheduler
        that passes the same caches every step pays one dictionary lookup, not the full checks."""
        hit = self._cache_ok.get(id(k))
        if hit is not None and hit[0]() is k and hit[1]() is v and k.shape == hit[2] and v.shape == hit[2]:
            return int(hit[2][2])
        c = self.cfg
        exp = (c.num_hidden_layers, 1, None, c.num_key_value_heads, c.head_dim)
        for t in (k, v):
            if t.dim() != 5 or any(e is not None and s != e for s, e in zip(t.shape, exp)):
                raise ValueError(f"KV cache must be {exp}, got {tuple(t.shape)}")
            if t.device != self.device or t.dtype != self.dtype or not t.is_contiguous():
                raise ValueError("KV cache must be contiguous, on the engine's device, in the model dtype")
        if k.shape != v.shape:
            raise ValueError("k and v caches differ in shape")
        if len(self._cache_ok) > 4096:  # entries of freed caches fail the identity check; bound them
            self._cache_ok.clear()
        self._cache_ok[id(k)] = (weakref.ref(k), weakref.ref(v), k.shape)
        return int(k.shape[2])

    def new_cache(self, capacity: int) -> tuple[torch.Tensor, torch.Tensor]:
        c = self.cfg
        shape = (c.num_hidden_layers, 1, int(capacity), c.num_key_value_heads, c.head_dim)
        return (torch.empty(shape, dtype=self.dtype, device=self.device),
                torch.empty(shape, dtype=self.dtype, device=self.device))

    # ---- the nine entry points ---------------------------------------------------------------
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous().reshape(-1)
        out = torch.empty((ids.numel(), self.cfg.hidden_size), dtype=self.dtype, device=self.device)
        _lib.check(self.lib.fdllm_embed(self._h, ids.data_ptr(), ids.numel(), out.data_ptr(), self._stream()))
        return out

    def forward_hidden(self, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        x2 = self._act(x, "forward_hidden")
        T = x2.shape[0]
        b = self._bias(bias, T)
        out = torch.empty_like(x2)
        _lib.check(self.lib.fdllm_forward_hidden(self._h, x2.data_ptr(), _ptr(b), T, out.data_ptr(), self._stream()))
        return out[None]

    def get_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        h2 = self._act(hidden, "get_logits")
        out = torch.empty((h2.shape[0], self.cfg.vocab_size), dtype=torch.float32, device=self.device)
        _lib.check(self.lib.fdllm_get_logits(self._h, h2.data_ptr(), h2.shape[0], out.data_ptr(), self._stream()))
        return out[None]

    def build_prefix_cache(self, x: torch.Tensor, bias: torch.Tensor | None, k: torch.Tensor, v: torch.Tensor) -> None:
        x2 = self._act(x, "build_prefix_cache")
        P = x2.shape[0]
        cap = self._cache(k, v)
        b = self._bias(bias, P)
        _lib.check(self.lib.fdllm_build_prefix_cache(self._h, x2.data_ptr(), _ptr(b), P, k.data_ptr(), v.data_ptr(),
                                                     cap, self._stream()))

    def forward_cached(self, x: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache_offset, prefix_len: int,
                       write_rel: int = 0, attend_rel: int | None = None) -> torch.Tensor:
        x2 = self._act(x, "forward_cached")
        rows = x2.shape[0]
        cap = self._cache(k, v)
        if attend_rel is None:
            attend_rel = rows
        off_t = self._offset(cache_offset)
        out = torch.empty_like(x2)
        _lib.check(self.lib.fdllm_forward_cached(self._h, x2.data_ptr(), rows, k.data_ptr(), v.data_ptr(), cap,
                                                 off_t.data_ptr(), int(prefix_len), int(write_rel), int(attend_rel),
                                                 out.data_ptr(), self._stream()))
        return out[None]

    def forward_block_partial(self, x, k, v, cache_offset, prefix_len: int, replace_position: int) -> torch.Tensor:
        return self.forward_cached(x, k, v, cache_offset, prefix_len, write_rel=replace_position,
                                   attend_rel=self.cfg.bd_size)

    # ---- batched / fused extensions ----------------------------------------------------------
    def build_prefix_cache_batch(self, x: torch.Tensor, caches: Sequence[tuple[torch.Tensor, torch.Tensor]],
                                 rows: Sequence[int]) -> None:
        """build_prefix_cache of several requests in one forward: x [sum(rows), hidden], request i's
        prefix is the next rows[i] rows, written to caches[i] = (k, v) rows [0, rows[i])."""
        x2 = self._act(x, "build_prefix_cache_batch")
        if len(caches) != len(rows) or not rows:
            raise ValueError("one (k, v) cache per request")
        if sum(int(r) for r in rows) != x2.shape[0]:
            raise ValueError(f"requests cover {sum(rows)} rows, x has {x2.shape[0]}")
        arr = (_lib.FdllmRequest * len(rows))()
        for i, ((k, v), r) in enumerate(zip(caches, rows)):
            arr[i] = _lib.FdllmRequest(k.data_ptr(), v.data_ptr(), self._cache(k, v), int(r), 0, 0, int(r), 0, None)
        _lib.check(self.lib.fdllm_build_prefix_cache_batch(self._h, arr, len(rows), x2.data_ptr(), self._stream()))

    def forward_cached_batch(self, x: torch.Tensor, requests: Sequence[dict]) -> torch.Tensor:
        """x: [sum(rows), hidden]; each request: dict(k, v, rows, prefix_len, write_rel=0,
        attend_rel=rows, cache_offset=int or device int32 tensor)."""
        x2 = self._act(x, "forward_cached_batch")
        arr = (_lib.FdllmRequest * len(requests))()
        keep = []
        total = 0
        for i, r in enumerate(requests):
            cap = self._cache(r["k"], r["v"])
            rows = int(r["rows"])
            off = r.get("cache_offset", int(r["prefix_len"]) + int(r.get("write_rel", 0)))
            dev_ptr, host = None, 0
            if isinstance(off, torch.Tensor):
                off_t = self._offset(off)
                keep.append(off_t)
                dev_ptr = off_t.data_ptr()
            else:
                host = int(off)
            arr[i] = _lib.FdllmRequest(r["k"].data_ptr(), r["v"].data_ptr(), cap, rows, int(r["prefix_len"]),
                                       int(r.get("write_rel", 0)), int(r.get("attend_rel", rows)), host, dev_ptr)
            total += rows
        if total != x2.shape[0]:
            raise ValueError(f"requests cover {total} rows, x has {x2.shape[0]}")
        out = torch.empty_like(x2)
        _lib.check(self.lib.fdllm_forward_cached_batch(self._h, arr, len(requests), x2.data_ptr(), out.data_ptr(),
                                                       self._stream()))
        return out

    def confidence(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """get_confidence_m{rows}: unshifted (ids int32 [rows], maxp fp32 [rows])."""
        h2 = self._act(hidden, "confidence")
        n = h2.shape[0]
        ids = torch.empty(n, dtype=torch.int32, device=self.device)
        maxp = torch.empty(n, dtype=torch.float32, device=self.device)
        _lib.check(self.lib.fdllm_confidence(self._h, h2.data_ptr(), n, ids.data_ptr(), maxp.data_ptr(), self._stream()))
        return ids, maxp

    def confidence_static(self, hidden: torch.Tensor, ids: torch.Tensor, maxp: torch.Tensor) -> None:
        """confidence() into caller-owned ids / maxp through fdllm_confidence_static, which
        allocates no device memory (its scratch is a fixed 4 MiB device array per device)."""
        # The kernel writes ids / maxp through raw pointers: a host tensor, a tensor on another GPU or
        # a strided view would be written at the wrong addresses, so refuse them before any launch.
        for t, dt, name in ((ids, torch.int32, "ids"), (maxp, torch.float32, "maxp")):
            if t.device != self.device or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"confidence_static: {name} must be a contiguous {dt} tensor on {self.device}")
        h2 = self._act(hidden, "confidence_static")
        n = h2.shape[0]
        if ids.numel() < n or maxp.numel() < n:
            raise ValueError("confidence_static: ids and maxp need at least rows elements")
        _lib.check(self.lib.fdllm_confidence_static(self._h, h2.data_ptr(), n, ids.data_ptr(), maxp.data_ptr(),
                                                    self._stream()))

    def confidence_from_logits(self, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        l2 = logits.reshape(-1, self.cfg.vocab_size).to(self.device, torch.float32).contiguous()
        n = l2.shape[0]
        ids = torch.empty(n, dtype=torch.int32, device=self.device)
        maxp = torch.empty(n, dtype=torch.float32, device=self.device)
        _lib.check(self.lib.fdllm_confidence_from_logits(self._h, l2.data_ptr(), n, ids.data_ptr(), maxp.data_ptr(),
                                                         self._stream()))
        return ids, maxp

    def unmask(self, ids: torch.Tensor, maxp: torch.Tensor, block: torch.Tensor, sub_start: int, sub_len: int,
               partial: bool, mask_id: int, threshold: float):
        """Device unmask step; updates `block` (int32 device) in place.  Returns (tokens, conf,
        unmask flags, status) device tensors."""
        n = int(ids.numel())
        tok = torch.empty(sub_len, dtype=torch.int32, device=self.device)
        conf = torch.empty(sub_len, dtype=torch.float32, device=self.device)
        flag = torch.empty(sub_len, dtype=torch.int32, device=self.device)
        status = torch.empty(2, dtype=torch.int32, device=self.device)
        _lib.check(self.lib.fdllm_unmask(self._h, ids.data_ptr(), maxp.data_ptr(), n, block.data_ptr(), int(sub_start),
                                         int(sub_len), int(bool(partial)), int(mask_id), float(threshold),
                                         tok.data_ptr(), conf.data_ptr(), flag.data_ptr(), status.data_ptr(),
                                         self._stream()))
        return tok, conf, flag, status

    def unmask_batch(self, ids: torch.Tensor, maxp: torch.Tensor, desc: torch.Tensor, threshold: float) -> torch.Tensor:
        """Unmask decisions of a batched step on the device (fdllm_unmask_batch): ids / maxp the
        step's confidence results, desc int32 [n, 5] (row0, rows, base, win, masked bits) on the
        device.  Returns int32 [n, 34]: unmasked bits, last-row argmax, window tokens."""
        n = int(desc.shape[0])
        for t, dt, name in ((ids, torch.int32, "ids"), (maxp, torch.float32, "maxp"), (desc, torch.int32, "desc")):
            if t.device != self.device or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"unmask_batch: {name} must be a contiguous {dt} tensor on {self.device}")
        out = torch.empty((n, 34), dtype=torch.int32, device=self.device)
        _lib.check(self.lib.fdllm_unmask_batch(self._h, ids.data_ptr(), maxp.data_ptr(), desc.data_ptr(), n,
                                               float(threshold), out.data_ptr(), self._stream()))
        return out

    def token_logprob(self, hidden: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        h2 = self._act(hidden, "token_logprob")
        n = h2.shape[0]
        tg = targets.to(self.device, torch.int32).contiguous().reshape(-1)
        if tg.numel() != n:
            raise ValueError("one target per row")
        out = torch.empty(n, dtype=torch.float32, device=self.device)
        _lib.check(self.lib.fdllm_token_logprob(self._h, h2.data_ptr(), n, tg.data_ptr(), out.data_ptr(), self._stream()))
        return out

    def generate(self, prompt_ids: Sequence[int], *, max_new_tokens: int, block_size: int = 32,
                 small_block_size: int = 8, threshold: float = 0.9, use_block_cache: bool = False, mask_id: int,
                 stop_token: int | None = None, timing: dict | None = None) -> tuple[list[int], dict]:
        """Native device-resident decode (runtime.py:591-880 for prompts of >= one block).
        `timing`, when a dict, receives prefill_ms and total_ms (CUDA events on the stream)."""
        prompt = (ctypes.c_int32 * len(prompt_ids))(*[int(t) for t in prompt_ids])
        out = (ctypes.c_int32 * max(int(max_new_tokens), 1))()
        n_out = ctypes.c_int(0)
        stats = (ctypes.c_int32 * 4)()
        tms = (ctypes.c_float * 2)()
        _lib.check(self.lib.fdllm_generate(self._h, prompt, len(prompt_ids), int(max_new_tokens), int(block_size),
                                           int(small_block_size), float(threshold), int(bool(use_block_cache)),
                                           int(mask_id), -1 if stop_token is None else int(stop_token), out,
                                           ctypes.byref(n_out), stats, tms if timing is not None else None,
                                           self._stream()))
        if timing is not None:
            timing["prefill_ms"] = float(tms[0])
            timing["total_ms"] = float(tms[1])
        keys = ("unmask_updates", "block_recomputes", "partial_recomputes", "block_appends")
        return [int(out[i]) for i in range(n_out.value)], dict(zip(keys, (int(s) for s in stats)))

    def profile_enable(self, enable: bool = True) -> None:
        _lib.check(self.lib.fdllm_profile_enable(self._h, int(bool(enable))))

    def profile_read(self) -> dict:
        """Totals of the profiled projection-GEMM launches since the last read (synchronises)."""
        buf = (ctypes.c_double * 4)()
        _lib.check(self.lib.fdllm_profile_read(self._h, buf))
        return {"ms": buf[0], "bytes": buf[1], "launches": int(buf[2]), "flops": buf[3]}

    @staticmethod
    def kernel_launches() -> int:
        return int(_lib.load().fdllm_kernel_launches())

    def device_error(self) -> int:
        code = ctypes.c_int(0)
        _lib.check(self.lib.fdllm_device_error(self._h, ctypes.byref(code)))
        return code.value

    def device_error_detail(self) -> list[int]:
        """[code, wait site, token rows, block | splits << 16] of the first recorded device error
        (zeros when none); clears the record."""
        buf = (ctypes.c_int32 * 4)()
        _lib.check(self.lib.fdllm_device_error_detail(self._h, buf))
        return [int(x) for x in buf]

    def wait_selftest(self, limit_ns: int = 200_000_000) -> int:
        code = ctypes.c_int(0)
        _lib.check(self.lib.fdllm_wait_selftest(self._h, int(limit_ns), ctypes.byref(code)))
        return code.value

    def kernel_trace_enable(self, enable: bool = True) -> None:
        """Record per-launch phase stamps of later eager projection / attention launches
        (diagnostics; clears the record)."""
        _lib.check(self.lib.fdllm_kernel_trace_enable(self._h, int(bool(enable))))

    def kernel_trace_read(self):
        """(stamps uint64 ns [n, 12 phases, 2 (min, max)], kinds int32 [n]); clears the record."""
        import numpy as np  # noqa: PLC0415
        n = ctypes.c_int(0)
        _lib.check(self.lib.fdllm_kernel_trace_read(self._h, None, None, 0, ctypes.byref(n)))
        out = np.zeros((n.value, 12, 2), dtype=np.uint64)
        kinds = np.zeros(n.value, dtype=np.int32)
        if n.value:
            _lib.check(self.lib.fdllm_kernel_trace_read(self._h, out.ctypes.data, kinds.ctypes.data, n.value,
                                                        ctypes.byref(n)))
        return out, kinds

    def workspace_bytes(self) -> int:
        return int(self.lib.fdllm_workspace_bytes(self._h))

    # ---- argument normalisation --------------------------------------------------------------
    def _bias(self, bias: torch.Tensor | None, T: int) -> torch.Tensor | None:
        if bias is None:
            return None
        b = bias.reshape(bias.shape[-2], bias.shape[-1])
        if tuple(b.shape) != (T, T):
            raise ValueError(f"attention bias must be [1, 1, {T}, {T}], got {tuple(bias.shape)}")
        return b.to(self.device, torch.float32).contiguous()

    def _offset(self, off) -> torch.Tensor:
        if isinstance(off, torch.Tensor):
            if off.numel() != 1:
                raise ValueError("cache_offset must be a scalar")
            return off.to(self.device, torch.int32).reshape(())
        return torch.tensor(int(off), dtype=torch.int32, device=self.device)
