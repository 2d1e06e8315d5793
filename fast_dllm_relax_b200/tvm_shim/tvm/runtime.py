"""tvm.runtime stand-in: device tensors are PyTorch tensors behind TVM's tensor API."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

try:  # registers numpy's bfloat16 (the reference's runners import it too)
    import ml_dtypes as _ml_dtypes
except ImportError:  # pragma: no cover
    _ml_dtypes = None

_KDL = {"cpu": 1, "cuda": 2, "metal": 8}
_TORCH_DTYPES = {
    "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
    "int32": torch.int32, "int64": torch.int64, "uint8": torch.uint8, "int8": torch.int8,
    "bool": torch.bool, "float64": torch.float64,
}
_DTYPE_NAMES = {v: k for k, v in _TORCH_DTYPES.items()}


class Device:
    """TVM device handle: kind + index, with `sync()` and the DLPack device type."""

    def __init__(self, kind: str, index: int = 0):
        kind = {"gpu": "cuda"}.get(kind, kind)
        if kind not in _KDL:
            raise ValueError(f"unsupported device kind {kind!r}")
        self.kind = kind
        self.index = int(index)

    @property
    def device_type(self) -> int:
        return _KDL[self.kind]

    @property
    def device_id(self) -> int:
        return self.index

    def dlpack_device_type(self) -> int:
        return _KDL[self.kind]

    @property
    def exist(self) -> bool:
        if self.kind == "cpu":
            return True
        if self.kind == "cuda":
            return torch.cuda.is_available() and self.index < torch.cuda.device_count()
        return False

    @property
    def torch_device(self) -> torch.device:
        if self.kind == "cuda":
            return torch.device("cuda", self.index)
        if self.kind == "cpu":
            return torch.device("cpu")
        raise RuntimeError(f"device kind {self.kind} has no PyTorch backing")

    def sync(self) -> None:
        if self.kind == "cuda":
            torch.cuda.synchronize(self.index)

    def __repr__(self) -> str:
        return f"{self.kind}({self.index})"

    def __eq__(self, other) -> bool:
        return isinstance(other, Device) and (self.kind, self.index) == (other.kind, other.index)

    def __hash__(self) -> int:
        return hash((self.kind, self.index))


def device(kind, index: int = 0) -> Device:
    if isinstance(kind, Device):
        return kind
    if isinstance(kind, str) and ":" in kind:
        kind, idx = kind.split(":", 1)
        index = int(idx)
    return Device(kind, index)


def cuda(index: int = 0) -> Device:
    return Device("cuda", index)


def cpu(index: int = 0) -> Device:
    return Device("cpu", index)


def metal(index: int = 0) -> Device:
    return Device("metal", index)


def _device_of(t: torch.Tensor) -> Device:
    if t.device.type == "cuda":
        return Device("cuda", t.device.index or 0)
    return Device("cpu", 0)


class ShapeTuple(tuple):
    """Host integer tuple (TVM's runtime.ShapeTuple)."""

    def __new__(cls, values=()):
        return super().__new__(cls, (int(v) for v in values))


class Tensor:
    """A device tensor with TVM's Python surface, backed by a torch tensor (`.torch`)."""

    __slots__ = ("torch",)

    def __init__(self, t: torch.Tensor):
        self.torch = t

    @property
    def shape(self) -> ShapeTuple:
        return ShapeTuple(self.torch.shape)

    @property
    def ndim(self) -> int:
        return self.torch.dim()

    @property
    def dtype(self) -> str:
        return _DTYPE_NAMES[self.torch.dtype]

    @property
    def device(self) -> Device:
        return _device_of(self.torch)

    def numpy(self) -> np.ndarray:
        t = self.torch.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        if t.dtype == torch.bfloat16:
            bits = t.contiguous().view(torch.int16).numpy().view(np.uint16)
            return bits.view(_ml_dtypes.bfloat16) if _ml_dtypes is not None else bits
        return t.contiguous().numpy()

    def copyfrom(self, source) -> "Tensor":
        src = _as_torch(source, like=self.torch)
        if tuple(src.shape) != tuple(self.torch.shape):
            raise ValueError(f"copyfrom shape mismatch: {tuple(src.shape)} vs {tuple(self.torch.shape)}")
        self.torch.copy_(src)
        return self

    def copyto(self, target):
        if isinstance(target, Device):
            return Tensor(self.torch.to(target.torch_device, copy=True))
        target.copyfrom(self)
        return target

    def __dlpack__(self, *args, **kwargs):
        return self.torch.__dlpack__(*args, **kwargs)

    def __dlpack_device__(self):
        return self.torch.__dlpack_device__()

    def __repr__(self) -> str:
        return f"tvm.runtime.Tensor(shape={tuple(self.shape)}, dtype={self.dtype}, device={self.device})"


NDArray = Tensor


def _as_torch(source, like: torch.Tensor | None = None) -> torch.Tensor:
    if isinstance(source, Tensor):
        t = source.torch
    elif isinstance(source, torch.Tensor):
        t = source
    else:
        arr = np.asarray(source)
        if like is not None and like.dtype == torch.bfloat16 and arr.dtype in (np.uint16, np.int16):
            t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16)
        elif _ml_dtypes is not None and arr.dtype == _ml_dtypes.bfloat16:
            t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16)
        else:
            t = torch.from_numpy(np.ascontiguousarray(arr))
    if like is not None:
        t = t.to(device=like.device, dtype=like.dtype)
    return t


def tensor(source, device=None, dtype=None) -> Tensor:
    dev = globals()["device"](device) if isinstance(device, str) else (device or cpu(0))
    t = _as_torch(source)
    if dtype is not None:
        t = t.to(_TORCH_DTYPES[str(dtype)])
    return Tensor(t.to(dev.torch_device).contiguous())


def empty(shape, dtype="float32", device=None) -> Tensor:
    dev = device or cpu(0)
    return Tensor(torch.empty(tuple(int(s) for s in shape), dtype=_TORCH_DTYPES[str(dtype)],
                              device=dev.torch_device))


def from_dlpack(obj) -> Tensor:
    if isinstance(obj, Tensor):
        return obj
    if isinstance(obj, torch.Tensor):
        return Tensor(obj)
    return Tensor(torch.from_dlpack(obj))


def _reshape(t, shape) -> Tensor:
    """vm.builtin.reshape: a view with a new shape (runtime.py:326-330)."""
    return Tensor(_as_torch(t).reshape(tuple(int(s) for s in shape)))


def load_module(path: str, fmt: str = "") -> object:
    """Load an artifact library written by fast_dllm_relax_b200.artifacts (its `.so` is the
    sm_100a library; the model config is read from `<stem>_config.json` beside it)."""
    from fast_dllm_relax_b200.vm_backend import ArtifactModule  # noqa: PLC0415

    return ArtifactModule(Path(path))
