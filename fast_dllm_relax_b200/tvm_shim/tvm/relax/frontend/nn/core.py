"""tvm.relax.frontend.nn.core stand-in."""

from ...._inert import _Inert

wrap_nested = _Inert("tvm.relax.frontend.nn.core.wrap_nested")
