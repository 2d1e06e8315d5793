"""tvm.relax.frontend stand-in (inert; see tvm/__init__.py)."""

from . import nn  # noqa: F401
