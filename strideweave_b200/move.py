"""CPU <-> CUDA moves for ``sw.move``.

The reference dispatches ``sw.move(tensor, destination)`` on the exact
(source class, destination class) pair and falls back to an elementwise copy
through Python indexing for unregistered pairs
(src/strideweave/carriers/move/ops.py:171-291).  Registering this pair makes
``sw.move(t, CUDA(n))`` a single host-to-device copy of the tensor's physical
span (layout holes included, as the reference's bulk CPU <-> FileBacked
moves do) and ``sw.move(t, CPU(n))`` the device-to-host copy back.

A carrier-level swizzle on the CUDA side is honoured: flat index f is stored
at swizzle(f), so the span is permuted on the host on the way.  Storage
dtypes without a bulk path between the two carriers take the reference's
elementwise copy.
"""

from __future__ import annotations

from ctypes import c_void_p
from typing import Any, ClassVar

import numpy as np

from . import _native as N
from ._host import DType  # makes `strideweave` importable (installed or baseline/_ref) first
from .layout_plan import swizzle_stages

from strideweave import CPU  # noqa: E402  (after _host)
from strideweave.carriers.move import (  # noqa: E402
    ElementwiseMoveOperation,
    MoveOperation,
    dispatch_move,
    register_move_operation,
)

from .carrier import CUDA  # noqa: E402  (carrier imports this module once CUDA exists)

_HOST_DTYPES = {DType.Float32: np.float32, DType.Int32: np.int32}


def _host_view(pointer: int, dtype: Any, count: int) -> np.ndarray:
    """The CPU carrier's storage at `pointer` as a numpy array (no copy)."""
    import ctypes

    np_dtype = np.dtype(_HOST_DTYPES[dtype])
    buf = (ctypes.c_char * (count * np_dtype.itemsize)).from_address(pointer)
    return np.frombuffer(buf, dtype=np_dtype, count=count)


def _permute(src_ptr: int, src_size: int, src_offset: int, src_swizzle: list, dst_ptr: int, dst_size: int,
             dst_offset: int, dst_swizzle: list) -> None:
    """dst flat index (dst_offset + i, through dst_swizzle) = src flat index
    (src_offset + i, through src_swizzle) for every i of the span: one
    32-bit view copy on the device."""
    from . import kernels

    count = min(src_size - src_offset, dst_size - dst_offset)
    kernels.copy_view_f32(src_ptr, src_size, src_offset, [(count, 1)], [(1, 0)], dst_ptr, dst_size, dst_offset,
                          [(count, 1)], [(1, 0)], swizzle=src_swizzle, dst_swizzle=dst_swizzle)


class CpuToCudaMoveOperation(MoveOperation):
    """Host-to-device move of a CPU tensor's physical span."""

    source_class: ClassVar[type | None] = CPU
    destination_class: ClassVar[type | None] = CUDA

    def _copy(self, tensor: Any, destination: Any, output: Any, element_count: int) -> None:
        dtype = destination.dtype()
        if dtype not in _HOST_DTYPES:
            ElementwiseMoveOperation._copy(self, tensor, destination, output, element_count)
            return
        src = _host_view(tensor.carrier.pointer() + tensor.offset * 4, dtype, element_count)
        if destination.swizzle is not None:
            # upload the span as it is, then permute it on the device into the
            # swizzled placement (positions outside the span keep their values)
            staged = N.DeviceBuffer(src.nbytes)
            staged.upload(src)
            _permute(staged.ptr, element_count, 0, [], destination.data_ptr, destination.size(), 0,
                     swizzle_stages(destination))
            N.synchronize()
            staged.free()
        else:
            N.check(N.lib.sw_memcpy_h2d(c_void_p(destination.data_ptr), c_void_p(src.ctypes.data), src.nbytes, None))
        N.synchronize()  # the source is released as soon as this returns
        destination._increment_version()


class CudaToCpuMoveOperation(MoveOperation):
    """Device-to-host move of a CUDA tensor's physical span."""

    source_class: ClassVar[type | None] = CUDA
    destination_class: ClassVar[type | None] = CPU

    def _copy(self, tensor: Any, destination: Any, output: Any, element_count: int) -> None:
        dtype = destination.dtype()
        if dtype not in _HOST_DTYPES:
            ElementwiseMoveOperation._copy(self, tensor, destination, output, element_count)
            return
        dst = _host_view(destination.pointer(), dtype, element_count)
        src = tensor.carrier
        if src.swizzle is not None:
            # gather the span out of the swizzled placement on the device, then
            # one copy to the host
            staged = N.DeviceBuffer(dst.nbytes)
            _permute(src.data_ptr, src.size(), tensor.offset, swizzle_stages(src), staged.ptr, element_count, 0, [])
            staged.download(dst)
            staged.free()
        else:
            N.check(N.lib.sw_memcpy_d2h(c_void_p(dst.ctypes.data), c_void_p(src.data_ptr + tensor.offset * 4),
                                        dst.nbytes, None))
        destination._increment_version()


def register() -> None:
    """Register the pair in the reference's move registry (once per process)."""
    if dispatch_move(CPU, CUDA) is not CpuToCudaMoveOperation:
        register_move_operation(CPU, CUDA, CpuToCudaMoveOperation)
    if dispatch_move(CUDA, CPU) is not CudaToCpuMoveOperation:
        register_move_operation(CUDA, CPU, CudaToCpuMoveOperation)


__all__ = ["CpuToCudaMoveOperation", "CudaToCpuMoveOperation", "register"]
