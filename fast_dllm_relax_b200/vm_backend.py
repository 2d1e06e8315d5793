"""The compiled module's entry points, served by the sm_100a library, for the TVM stand-in.

`tvm.runtime.load_module(<artifact>/fast_dllm_relax_nn.so)` returns an `ArtifactModule`;
`tvm.relax.VirtualMachine(module, tvm.cuda(i))` then resolves `vm[name]` through
`B200Backend.function(name)`.  The call signatures are those of the reference's compiled module
(fast_dllm_relax/model/cuda.py:799-842) as its runtime calls them:

    vm["embed"](ids int32[n], params)                          -> [n, hidden]          runtime.py:326-330
    vm["forward_hidden"](x [1,T,H], bias f32[1,1,T,T], params) -> [1, T, H]            runtime.py:439-482
    vm["get_logits"](h [1,R,H], params)                        -> f32 [1, R, vocab]    runtime.py:176-181
    vm["build_prefix_cache"](x, bias, k, v, params)            -> (k, v), in place     runtime.py:312-323
    vm["forward_cached"](x, k, v, off, ShapeTuple([P]), params)            -> [1,R,H]  runtime.py:333-343
    vm["forward_block_partial_rp{0,8,16,24}"](x, k, v, off, ShapeTuple([P]), params) runtime.py:413-436
    vm["get_confidence_m{R}"](h [1,R,H], params) -> (ids int32 [1,R], maxp f32 [1,R]) runtime.py:131-174

`off` is the 0-d int32 device tensor of the RoPE start (read on the device), `P` the committed
prefix length (host).  Caches are [layers, 1, cap, kv_heads, head_dim] tensors written in place.
Names the reference's runtime probes but this library does not need (the fixed-row siblings
forward_cached_b32 / get_logits_m{8,32}, runtime.py:100-128) raise KeyError, so the runtime
keeps its dynamic calls.  There is no CPU path: a VirtualMachine on a non-CUDA device raises.
"""

from __future__ import annotations

import re
from pathlib import Path

import torch

from . import artifacts
from .config import ModelConfig

_PARTIAL = re.compile(r"forward_block_partial_rp(\d+)$")
_CONF = re.compile(r"get_confidence_m(\d+)$")


def _tensor_cls():
    import tvm  # noqa: PLC0415  (the stand-in; imported lazily so this module loads without it)
    return tvm.runtime.Tensor


class ArtifactModule:
    """What `tvm.runtime.load_module` returns for an artifact directory's library path."""

    def __init__(self, library_path: str | Path):
        self.library_path = Path(library_path)
        self.dir = self.library_path.parent
        self.dtype = artifacts.read_dtype(self.dir)
        self.cfg: ModelConfig = artifacts.read_config(self.dir)
        artifacts.read_kv_manifest(self.dir)

    def create_backend(self, dev) -> "B200Backend":
        return B200Backend(self, dev)


class B200Backend:
    """One library handle (Engine) per VirtualMachine, bound to the `params` list the calls pass."""

    def __init__(self, module: ArtifactModule, dev):
        if getattr(dev, "kind", None) != "cuda":
            raise RuntimeError(f"the sm_100a library runs on CUDA devices only (got {dev!r}); there is no CPU path")
        self.module = module
        self.cfg = module.cfg
        self.dtype = module.dtype
        self.dev = dev
        self.engine = None
        self._params_obj = None
        self._params_ptrs: tuple[int, ...] = ()

    # ---- params binding ----------------------------------------------------------------------
    def _bind(self, params):
        """Bind `params` once; rebind only when the caller passes different storage."""
        if params is self._params_obj and self.engine is not None:
            return self.engine
        ts = [p.torch if hasattr(p, "torch") else torch.from_dlpack(p) for p in params]
        ptrs = tuple(t.data_ptr() for t in ts)
        if self.engine is None:
            from .engine import Engine  # noqa: PLC0415
            self.engine = Engine(self.cfg, ts, dtype=self.dtype, device=self.dev.index)
        elif ptrs != self._params_ptrs:
            self.engine.bind(ts)
        self._params_obj = params
        self._params_ptrs = ptrs
        return self.engine

    # ---- entry points ------------------------------------------------------------------------
    def function(self, name: str):
        T = _tensor_cls()

        def t(x):
            return x.torch if hasattr(x, "torch") else torch.from_dlpack(x)

        if name == "embed":
            def embed(ids, params):
                return T(self._bind(params).embed(t(ids)))
            return embed
        if name == "forward_hidden":
            def forward_hidden(x, bias, params):
                return T(self._bind(params).forward_hidden(t(x), t(bias)))
            return forward_hidden
        if name == "get_logits":
            def get_logits(h, params):
                return T(self._bind(params).get_logits(t(h)))
            return get_logits
        if name == "build_prefix_cache":
            def build_prefix_cache(x, bias, k, v, params):
                self._bind(params).build_prefix_cache(t(x), t(bias), t(k), t(v))
                return k, v
            return build_prefix_cache
        if name == "forward_cached":
            def forward_cached(x, k, v, off, plen, params):
                return T(self._bind(params).forward_cached(t(x), t(k), t(v), t(off), int(plen[0])))
            return forward_cached
        m = _PARTIAL.match(name)
        if m:
            rp = int(m.group(1))
            if rp % 8 != 0 or rp >= self.cfg.bd_size:
                raise KeyError(name)

            def partial(x, k, v, off, plen, params):
                return T(self._bind(params).forward_block_partial(t(x), t(k), t(v), t(off), int(plen[0]), rp))
            return partial
        m = _CONF.match(name)
        if m:
            rows = int(m.group(1))

            def confidence(h, params):
                hh = t(h)
                if hh.shape[-2] != rows:
                    raise ValueError(f"{name}: expected {rows} rows, got {tuple(hh.shape)}")
                ids, maxp = self._bind(params).confidence(hh)
                return T(ids[None]), T(maxp[None])
            return confidence
        raise KeyError(name)
