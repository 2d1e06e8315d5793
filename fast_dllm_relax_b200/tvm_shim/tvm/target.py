"""tvm.target stand-in."""

from ._inert import _Inert

Target = _Inert("tvm.target.Target")
