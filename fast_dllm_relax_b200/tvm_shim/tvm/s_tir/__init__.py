"""tvm.s_tir stand-in: dlight schedules are never applied with the sm_100a library."""

from .._inert import _Inert

dlight = _Inert("tvm.s_tir.dlight")
T = _Inert("tvm.s_tir.T")
