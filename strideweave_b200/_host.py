"""The StrideWeave framework this package plugs into.

The CUDA carrier is a sibling ``strideweave.Carrier`` implementation, so the
reference framework itself must be importable.  An installed ``strideweave``
is used as is; a source checkout of this repository may instead carry an
installed copy under ``baseline/_ref`` (the layout the benchmark driver
uses), which is added to ``sys.path`` when nothing else provides it.
"""

from __future__ import annotations

import sys
from pathlib import Path

try:
    import strideweave  # noqa: F401
except ImportError:  # pragma: no cover - depends on the environment
    _candidate = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (_candidate / "strideweave").is_dir():
        raise ImportError(
            "strideweave_b200 plugs into the StrideWeave framework; install "
            "strideweave (patrickk1998/strideweave) first"
        ) from None
    sys.path.append(str(_candidate))
    import strideweave  # noqa: F401

import strideweave as sw
from strideweave import Carrier, Layout, Shape, Stride, Swizzle, Tensor
from strideweave.carriers.dtype import DType, SimpleDType
from strideweave.carriers.operation_capability import (
    OperationCapability,
    UnsupportedOperationPlan,
    register_operation_capabilities,
    require_capability,
)
from strideweave.carriers.operation_helpers import Operation
from strideweave.carriers.operation_policy import resolve_operation_plan
from strideweave.core._representation import Subtensor, TensorRepresentation


def _bfloat16() -> SimpleDType:
    """The BFloat16 storage dtype (an extension dtype; the reference has none)."""
    try:
        found = DType.from_name("BFloat16")
    except (KeyError, ValueError, LookupError):
        found = None
    if found is not None:
        return found
    return SimpleDType("BFloat16", bits=16, supertype=DType.Floating)


BFloat16 = _bfloat16()

__all__ = [
    "BFloat16", "Carrier", "DType", "Layout", "Operation", "OperationCapability", "Shape", "SimpleDType", "Stride",
    "Subtensor", "Swizzle", "Tensor", "TensorRepresentation", "UnsupportedOperationPlan",
    "register_operation_capabilities", "require_capability", "resolve_operation_plan", "sw",
]
