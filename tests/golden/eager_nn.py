"""Eager PyTorch stand-in for the slice of TVM's Relax `nn` frontend (and the `relax` ops) that the
reference's model definition, fast_dllm_relax/model/cuda.py, is written against.

TEST INFRASTRUCTURE ONLY: tests/golden/make_model_golden.py installs it into its own process
before importing the reference model, so that the reference's graph runs op by op on the CPU and
its outputs can be recorded as golden vectors.  Nothing else imports it.

Semantics follow TVM's op definitions:
* elementwise ops take operands of one dtype (a mismatch raises instead of promoting); bf16 ops
  compute in fp32 and round once, as TVM's bf16 legalisation does;
* `matmul(a, b, out_dtype)` accumulates in fp32 and rounds once to `out_dtype` (default: a's);
* `repeat` is numpy.repeat (each element repeated), `split` with a list splits at those indices;
* `nn.Linear` is matmul(x, weight^T) + bias accumulated in fp32 and rounded once: the reference's
  production pipeline (model/cuda.py:31-60) hands matmul + bias to cuBLAS, whose bias epilogue
  adds the bias before the single rounding; `nn.Embedding` is take(weight, ids, axis=0);
* `call_inplace_packed` calls the registered global function with the in-place buffers (shared
  storage through DLPack) and returns what it returns.
Elementwise bf16 ops round after every op, as TVM's bf16 legalisation does even inside fused
kernels; in fp32 none of these choices changes a result beyond summation order.
"""

from __future__ import annotations

import sys
import types

import torch

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16, "int32": torch.int32,
       "int64": torch.int64}
_NAMES = {v: k for k, v in _DT.items()}


class _E(torch.Tensor):
    """A torch tensor standing for a Relax expression; `.struct_info` is all the model reads."""

    @property
    def struct_info(self):
        return None


def _e(t) -> _E:
    if isinstance(t, _E):
        return t
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    return t.as_subclass(_E)


def _raw(x) -> torch.Tensor:
    if isinstance(x, Tensor):
        x = x._expr
    return x.as_subclass(torch.Tensor) if isinstance(x, torch.Tensor) else x


def _low(t: torch.Tensor) -> bool:
    return t.dtype in (torch.bfloat16, torch.float16)


class Tensor:
    """nn.Tensor: a wrapper of one expression (here a torch tensor)."""

    def __init__(self, expr):
        self._expr = _e(expr)

    @property
    def shape(self):
        return tuple(int(s) for s in self._expr.shape)

    @property
    def ndim(self) -> int:
        return self._expr.dim()

    @property
    def dtype(self) -> str:
        return _NAMES[self._expr.dtype]

    @staticmethod
    def from_scalar(value, dtype: str) -> "Tensor":
        return Tensor(torch.tensor(value, dtype=_DT[dtype]))

    def astype(self, dtype: str) -> "Tensor":
        return op.astype(self, dtype)

    def __add__(self, other):
        return op.add(self, other)

    def __mul__(self, other):
        return op.multiply(self, other)


class Parameter(Tensor):
    def __init__(self, shape, dtype: str = "float32"):
        self._shape = tuple(shape)
        self._dtype = dtype
        self._bound = None

    def bind(self, t: torch.Tensor) -> None:
        if tuple(t.shape) != self._shape:
            raise ValueError(f"parameter shape {tuple(t.shape)} != declared {self._shape}")
        self._bound = _e(t.to(_DT[self._dtype]).contiguous())

    @property
    def _expr(self):
        if self._bound is None:
            raise RuntimeError("parameter not bound")
        return self._bound


class Module:
    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def to(self, dtype=None):
        return self

    def named_parameters(self, prefix: str = ""):
        for name, val in vars(self).items():
            full = f"{prefix}{name}"
            if isinstance(val, Parameter):
                yield full, val
            elif isinstance(val, ModuleList):
                for i, m in enumerate(val):
                    yield from m.named_parameters(f"{full}.{i}.")
            elif isinstance(val, Module):
                yield from val.named_parameters(f"{full}.")


class ModuleList(Module):
    def __init__(self, modules):
        self._modules = list(modules)

    def __iter__(self):
        return iter(self._modules)

    def __len__(self):
        return len(self._modules)

    def __getitem__(self, i):
        return self._modules[i]


class Linear(Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True, dtype: str = "float32",
                 out_dtype: str | None = None):
        self.weight = Parameter((out_features, in_features), dtype)
        self.bias = Parameter((out_features,), dtype) if bias else None
        self.out_dtype = out_dtype

    def forward(self, x: Tensor) -> Tensor:
        if self.bias is None:
            return op.matmul(x, op.permute_dims(self.weight), out_dtype=self.out_dtype)
        xt, wt, bt = _raw(x), _raw(self.weight), _raw(self.bias)
        _same(xt, wt, "linear")
        _same(xt, bt, "linear bias")
        out = _DT[self.out_dtype] if self.out_dtype else xt.dtype
        return Tensor((torch.matmul(xt.float(), wt.float().t()) + bt.float()).to(out))


class Embedding(Module):
    def __init__(self, num: int, dim: int, dtype: str = "float32"):
        self.weight = Parameter((num, dim), dtype)

    def forward(self, x: Tensor) -> Tensor:
        return op.take(self.weight, x, axis=0)


class ExternModule(Module):
    pass


class RMSNorm(Module):  # named by the module, not used by the model's graph
    pass


def _same(a: torch.Tensor, b: torch.Tensor, name: str) -> None:
    if a.dtype != b.dtype:
        raise TypeError(f"{name}: operand dtypes differ ({a.dtype} vs {b.dtype})")


def _binary(fn, name):
    def f(a, b):
        x, y = _raw(a), _raw(b)
        _same(x, y, name)
        if _low(x):
            return Tensor(fn(x.float(), y.float()).to(x.dtype))
        return Tensor(fn(x, y))
    f.__name__ = name
    return f


def _unary(fn, name):
    def f(a, *args, **kwargs):
        x = _raw(a)
        if _low(x):
            return Tensor(fn(x.float(), *args, **kwargs).to(x.dtype))
        return Tensor(fn(x, *args, **kwargs))
    f.__name__ = name
    return f


def _matmul(a, b, out_dtype: str | None = None) -> Tensor:
    x, y = _raw(a), _raw(b)
    _same(x, y, "matmul")
    out = _DT[out_dtype] if out_dtype else x.dtype
    return Tensor(torch.matmul(x.float(), y.float()).to(out) if _low(x) else torch.matmul(x, y).to(out))


def _split(x, indices_or_sections, axis: int = 0):
    t = _raw(x)
    if isinstance(indices_or_sections, int):
        parts = torch.tensor_split(t, indices_or_sections, dim=axis)
    else:
        parts = torch.tensor_split(t, list(indices_or_sections), dim=axis)
    return tuple(Tensor(p) for p in parts)


def _permute_dims(x, axes=None) -> Tensor:
    t = _raw(x)
    return Tensor(t.permute(*(axes if axes is not None else reversed(range(t.dim())))))


def _expand_dims(x, axis) -> Tensor:
    t = _raw(x)
    for a in sorted(axis if isinstance(axis, (list, tuple)) else [axis]):
        t = t.unsqueeze(a)
    return Tensor(t)


op = types.SimpleNamespace(
    add=_binary(torch.add, "add"),
    multiply=_binary(torch.mul, "multiply"),
    astype=lambda x, dtype: Tensor(_raw(x).to(_DT[dtype])),
    reshape=lambda x, shape: Tensor(_raw(x).reshape(tuple(int(s) for s in shape))),
    expand_dims=_expand_dims,
    permute_dims=_permute_dims,
    matmul=_matmul,
    split=_split,
    concat=lambda xs, dim=0: Tensor(torch.cat([_raw(x) for x in xs], dim=dim)),
    softmax=_unary(lambda t, axis=-1: torch.softmax(t, dim=axis), "softmax"),
    exp=_unary(torch.exp, "exp"),
    sin=_unary(torch.sin, "sin"),
    cos=_unary(torch.cos, "cos"),
    square=_unary(torch.square, "square"),
    sigmoid=_unary(torch.sigmoid, "sigmoid"),
    silu=_unary(torch.nn.functional.silu, "silu"),
    rsqrt=_unary(torch.rsqrt, "rsqrt"),
    repeat=lambda x, repeats, axis=None: Tensor(torch.repeat_interleave(_raw(x), repeats, dim=axis)),
    mean=_unary(lambda t, axis=None, keepdims=False: torch.mean(t, dim=axis, keepdim=keepdims), "mean"),
    take=lambda x, idx, axis=0: Tensor(torch.index_select(_raw(x), axis, _raw(idx).reshape(-1).long())
                                       .reshape(tuple(_raw(idx).shape) + tuple(_raw(x).shape[1:]))),
    arange=lambda start, end=None, step=1, dtype="float32": Tensor(
        torch.arange(start, end, step, dtype=_DT[dtype]) if end is not None else torch.arange(start, dtype=_DT[dtype])),
)


def wrap_nested(expr, name: str = ""):
    if isinstance(expr, (tuple, list)):
        return tuple(Tensor(e) for e in expr)
    return Tensor(expr)


def install(tvm) -> None:
    """Point tvm.relax's graph-building names and tvm.relax.frontend.nn at this module (in this
    process only), keeping the stand-in's runtime pieces (global functions, tensors)."""
    rx = tvm.relax

    def _rx_unary(fn):
        return lambda x: _e(_unary(fn, "rx")(x)._expr)

    def call_inplace_packed(func_name, *args, inplace_indices=None, sinfo_args=None):
        f = tvm.get_global_func(func_name)
        conv = [tvm.runtime.from_dlpack(_raw(a)) if isinstance(a, torch.Tensor) else a for a in args]
        res = f(*conv)
        res = res if isinstance(res, (tuple, list)) else (res,)
        return tuple(_e(torch.from_dlpack(r)) if hasattr(r, "__dlpack__") else r for r in res)

    rx.op = types.SimpleNamespace(
        cos=_rx_unary(torch.cos), sin=_rx_unary(torch.sin), exp=_rx_unary(torch.exp), rsqrt=_rx_unary(torch.rsqrt),
        astype=lambda x, dtype: _e(_raw(x).to(_DT[dtype])),
        arange=lambda start, end=None, step=1, dtype="float32": _e(op.arange(start, end, step, dtype)._expr),
        expand_dims=lambda x, axis: _e(_expand_dims(x, axis)._expr),
        concat=lambda xs, axis=0: _e(torch.cat([_raw(x) for x in xs], dim=axis)),
        add=lambda a, b: _e(op.add(a, b)._expr),
        mean=lambda x, axis=None, keepdims=False: _e(op.mean(x, axis=axis, keepdims=keepdims)._expr),
        call_inplace_packed=call_inplace_packed,
    )
    rx.const = lambda value, dtype="float32": _e(torch.tensor(value, dtype=_DT[dtype]))
    rx.PrimValue = lambda v: int(v)
    rx.ShapeExpr = lambda v: list(v)
    rx.TensorStructInfo = lambda *a, **k: None

    nn = types.ModuleType("tvm.relax.frontend.nn")
    core = types.ModuleType("tvm.relax.frontend.nn.core")
    core.wrap_nested = wrap_nested
    for name in ("Tensor", "Parameter", "Module", "ModuleList", "Linear", "Embedding", "ExternModule", "RMSNorm"):
        setattr(nn, name, globals()[name])
    nn.op = op
    nn.core = core
    nn.spec = types.SimpleNamespace(Tensor=None, ModuleSpec=None)
    frontend = types.ModuleType("tvm.relax.frontend")
    frontend.nn = nn
    rx.frontend = frontend
    sys.modules.update({"tvm.relax.frontend": frontend, "tvm.relax.frontend.nn": nn,
                        "tvm.relax.frontend.nn.core": core})
