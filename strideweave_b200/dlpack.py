"""DLPack import and export for CUDA carriers.

The reference exports a tensor through ``Tensor.__dlpack__`` for Float32 and
Int32 only (src/strideweave/core/native/_tensor.cpp:180-188,412-435) and has
no import path.  This module adds both directions for device tensors:

- ``from_dlpack(obj)`` wraps any producer of a CUDA DLPack capsule (a torch
  CUDA tensor, for example) as a ``Tensor`` on a ``CUDA`` carrier without a
  copy.  The carrier keeps the producer's memory alive and hands it back
  through the capsule's deleter when it is released.  The producer is asked
  to make its data ready on the legacy default stream (``stream=1``), the
  stream every carrier operation is ordered on.
- ``to_dlpack(t)`` / ``DLPackExport(t)`` export a CUDA-carrier tensor of any
  carrier dtype, the narrow MX planes included (E4M3, E8M0, packed E2M1,
  BFloat16), as a strided DLPack view.  The device is synchronised before the
  capsule is handed out, so the consumer may read it on any stream.

DLPack dtype codes (DLPack 1.x): Int 0, UInt 1, Float 2, Bfloat 4, Bool 6,
Float8_e4m3fn 10, Float8_e8m0fnu 14, Float4_e2m1fn 17 (4 bits, 2 lanes per
byte as torch's ``float4_e2m1fn_x2``).
"""

from __future__ import annotations

import ctypes
from ctypes import CFUNCTYPE, POINTER, Structure, c_char_p, c_int, c_int64, c_uint8, c_uint16, c_uint64, c_void_p
from typing import Any

import numpy as np

from . import _native as N
from ._host import BFloat16, DType, Layout, Shape, Stride, Tensor

KDL_CUDA = 2
_CODES = {  # (code, bits, lanes) -> carrier dtype
    (2, 32, 1): DType.Float32,
    (0, 32, 1): DType.Int32,
    (6, 8, 1): DType.Bool,
    (4, 16, 1): BFloat16,
    (10, 8, 1): DType.E4M3,
    (14, 8, 1): DType.E8M0,
    (17, 4, 2): DType.E2M1,
}
_DTYPE_CODES = {v: k for k, v in _CODES.items()}


class DLDevice(Structure):
    _fields_ = [("device_type", c_int), ("device_id", c_int)]


class DLDataType(Structure):
    _fields_ = [("code", c_uint8), ("bits", c_uint8), ("lanes", c_uint16)]


class DLTensor(Structure):
    _fields_ = [("data", c_void_p), ("device", DLDevice), ("ndim", c_int), ("dtype", DLDataType),
                ("shape", POINTER(c_int64)), ("strides", POINTER(c_int64)), ("byte_offset", c_uint64)]


class DLManagedTensor(Structure):
    pass


_DELETER = CFUNCTYPE(None, POINTER(DLManagedTensor))
DLManagedTensor._fields_ = [("dl_tensor", DLTensor), ("manager_ctx", c_void_p), ("deleter", _DELETER)]

_api = ctypes.pythonapi
_api.PyCapsule_GetPointer.restype = c_void_p
_api.PyCapsule_GetPointer.argtypes = [ctypes.py_object, c_char_p]
_api.PyCapsule_IsValid.restype = c_int
_api.PyCapsule_IsValid.argtypes = [ctypes.py_object, c_char_p]
_api.PyCapsule_SetName.restype = c_int
_api.PyCapsule_SetName.argtypes = [ctypes.py_object, c_char_p]
# A capsule destructor runs while the capsule is being deallocated: it gets
# the raw object pointer and must not take a reference to it, so it uses
# bindings of the capsule API that pass the object as a plain pointer.
_CAPSULE_DESTRUCTOR = CFUNCTYPE(None, c_void_p)
_api.PyCapsule_New.restype = ctypes.py_object
_api.PyCapsule_New.argtypes = [c_void_p, c_char_p, _CAPSULE_DESTRUCTOR]
_raw_is_valid = ctypes.PYFUNCTYPE(c_int, c_void_p, c_char_p)(("PyCapsule_IsValid", ctypes.pythonapi))
_raw_get_pointer = ctypes.PYFUNCTYPE(c_void_p, c_void_p, c_char_p)(("PyCapsule_GetPointer", ctypes.pythonapi))


# ---- import -------------------------------------------------------------------------


class _ExternalBuffer:
    """Device memory owned by a DLPack producer, seen through the interface
    the carrier uses for its own allocations (ptr, nbytes, upload, download,
    free).  ``free`` returns the memory to the producer once."""

    __slots__ = ("ptr", "nbytes", "_managed", "_producer")

    def __init__(self, ptr: int, nbytes: int, managed: int, producer: Any) -> None:
        self.ptr = ptr
        self.nbytes = nbytes
        self._managed = managed
        self._producer = producer  # keeps the exporting object alive too

    def upload(self, host: np.ndarray, stream: int | None = None) -> None:
        if host.nbytes > self.nbytes:
            raise ValueError("host array larger than the device buffer")
        N.check(N.lib.sw_memcpy_h2d(c_void_p(self.ptr), c_void_p(host.ctypes.data), host.nbytes,
                                    c_void_p(stream or 0)))

    def download(self, host: np.ndarray, stream: int | None = None) -> None:
        if host.nbytes > self.nbytes:
            raise ValueError("host array larger than the device buffer")
        N.check(N.lib.sw_memcpy_d2h(c_void_p(host.ctypes.data), c_void_p(self.ptr), host.nbytes,
                                    c_void_p(stream or 0)))

    def free(self) -> None:
        if self._managed:
            N.synchronize()  # no carrier work may still read the producer's memory
            managed = DLManagedTensor.from_address(self._managed)
            self._managed = 0
            if managed.deleter:
                managed.deleter(ctypes.cast(ctypes.addressof(managed), POINTER(DLManagedTensor)))
        self.ptr = 0
        self.nbytes = 0
        self._producer = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.free()
        except Exception:
            pass


def from_dlpack(obj: Any, *, mutable: bool = True) -> Tensor:
    """Wrap a CUDA DLPack producer as a Tensor on a CUDA carrier, zero-copy.

    The carrier's flat index space is the span the producer's strides reach
    (from its first element); the tensor's layout is the producer's shape
    and strides, so element (i, j, ...) reads what the producer holds there.
    Negative strides are refused.  Packed E2M1 (``float4_e2m1fn_x2``) must be
    one-dimensional and contiguous; its logical size is twice the bytes.
    """
    from .carrier import CUDA, storage_bytes

    if hasattr(obj, "__dlpack_device__"):
        dev_type, dev_id = obj.__dlpack_device__()
        if int(dev_type) != KDL_CUDA:
            raise BufferError("from_dlpack needs a CUDA device tensor")
    if not hasattr(obj, "__dlpack__"):
        raise TypeError("object does not implement __dlpack__")
    try:
        capsule = obj.__dlpack__(stream=1)  # ready on the legacy default stream
    except TypeError:
        capsule = obj.__dlpack__()
    if not _api.PyCapsule_IsValid(capsule, b"dltensor"):
        raise BufferError("expected an unconsumed 'dltensor' capsule")
    managed_ptr = _api.PyCapsule_GetPointer(capsule, b"dltensor")
    dl = DLManagedTensor.from_address(managed_ptr).dl_tensor
    if dl.device.device_type != KDL_CUDA:
        raise BufferError("from_dlpack needs a CUDA device tensor")
    key = (dl.dtype.code, dl.dtype.bits, dl.dtype.lanes)
    dtype = _CODES.get(key)
    if dtype is None:
        raise BufferError(f"no CUDA carrier dtype for DLPack dtype {key}")
    ndim = dl.ndim
    shape = [dl.shape[i] for i in range(ndim)]
    if dl.strides:
        strides = [dl.strides[i] for i in range(ndim)]
    else:
        strides, acc = [0] * ndim, 1
        for i in reversed(range(ndim)):
            strides[i] = acc
            acc *= shape[i]
    if any(s < 0 for s in strides):
        raise BufferError("negative DLPack strides are not supported")
    n = 1
    for e in shape:
        n *= e
    span = 1 + sum((e - 1) * s for e, s in zip(shape, strides)) if n else 0
    if dtype is DType.E2M1:
        if ndim != 1 or (shape[0] > 1 and strides[0] != 1):
            raise BufferError("packed E2M1 import must be one-dimensional and contiguous")
        shape, strides, span = [2 * shape[0]], [1], 2 * span
    # take ownership: the capsule is consumed, its deleter runs at release
    _api.PyCapsule_SetName(capsule, b"used_dltensor")
    data = (dl.data or 0) + dl.byte_offset
    current = N.current_device()
    if dl.device.device_id != current:
        N.set_device(dl.device.device_id)
    carrier = CUDA(0, dtype=dtype, mutable=mutable, empty=True, device=dl.device.device_id)
    carrier._buffer.free()
    carrier._buffer = _ExternalBuffer(data, storage_bytes(dtype, span), managed_ptr, obj)
    carrier._size = span
    carrier._nbytes = storage_bytes(dtype, span)
    if ndim == 0:
        return Tensor(carrier, 0, Layout(Shape(1), Stride(1)))
    return Tensor(carrier, 0, Layout(Shape(list(shape)), Stride(list(strides))))


# ---- export -------------------------------------------------------------------------

_LIVE: dict[int, tuple[Any, ...]] = {}  # managed-tensor address -> objects it keeps alive


@_DELETER
def _release_export(managed: Any) -> None:
    _LIVE.pop(ctypes.addressof(managed.contents), None)


@_CAPSULE_DESTRUCTOR
def _capsule_destructor(capsule: int) -> None:
    # an exported capsule nobody consumed: drop what it keeps alive (a
    # consumer renames the capsule and calls the deleter itself)
    if _raw_is_valid(capsule, b"dltensor"):
        ptr = _raw_get_pointer(capsule, b"dltensor")
        _LIVE.pop(ptr, None)


def _export_strides(t: Tensor) -> tuple[list[int], list[int]]:
    from .layout_plan import mode_leaves

    shape, strides = [], []
    for m in range(len(t.layout)):
        leaves = [(e, s) for e, s in mode_leaves(t.layout, m) if e != 1]
        if not leaves:
            shape.append(1)
            strides.append(0)
            continue
        ext, st = leaves[0]
        for e, s in leaves[1:]:
            if s != st * ext:
                raise BufferError("a hierarchical mode that is not one stride has no DLPack view")
            ext *= e
        shape.append(ext)
        strides.append(st)
    return shape, strides


def to_dlpack(t: Tensor) -> Any:
    """A 'dltensor' capsule viewing a CUDA-carrier tensor (see module doc)."""
    from .carrier import CUDA

    if not isinstance(t, Tensor) or not isinstance(t.carrier, CUDA):
        raise TypeError("to_dlpack needs a Tensor on a CUDA carrier")
    t._require_single_subtensor("DLPack export")
    carrier = t.carrier
    if carrier.swizzle is not None:
        raise BufferError("a swizzled carrier has no strided DLPack view")
    shape, strides = _export_strides(t)
    dtype = carrier.dtype()
    code, bits, lanes = _DTYPE_CODES[dtype]
    offset_bytes = t.offset * bits // 8
    if dtype is DType.E2M1:
        if len(shape) != 1 or (shape[0] > 1 and strides[0] != 1) or shape[0] % 2 or t.offset % 2:
            raise BufferError("packed E2M1 export needs an even, contiguous, one-dimensional view")
        shape, strides, offset_bytes = [shape[0] // 2], [1], t.offset // 2
    N.synchronize()  # every carrier operation so far is complete on the device
    ndim = len(shape)
    shape_arr = (c_int64 * max(ndim, 1))(*shape)
    strides_arr = (c_int64 * max(ndim, 1))(*strides)
    managed = DLManagedTensor()
    managed.dl_tensor.data = carrier.data_ptr + offset_bytes
    managed.dl_tensor.device = DLDevice(KDL_CUDA, carrier.device)
    managed.dl_tensor.ndim = ndim
    managed.dl_tensor.dtype = DLDataType(code, bits, lanes)
    managed.dl_tensor.shape = ctypes.cast(shape_arr, POINTER(c_int64))
    managed.dl_tensor.strides = ctypes.cast(strides_arr, POINTER(c_int64))
    managed.dl_tensor.byte_offset = 0
    managed.manager_ctx = None
    managed.deleter = _release_export
    _LIVE[ctypes.addressof(managed)] = (managed, shape_arr, strides_arr, t, carrier)
    return _api.PyCapsule_New(ctypes.addressof(managed), b"dltensor", _capsule_destructor)


class DLPackExport:
    """A CUDA-carrier tensor seen through the DLPack protocol, so consumers
    such as ``torch.from_dlpack`` can take it without a copy."""

    def __init__(self, t: Tensor) -> None:
        self._t = t

    def __dlpack_device__(self) -> tuple[int, int]:
        return (KDL_CUDA, self._t.carrier.device)

    def __dlpack__(self, *, stream: Any = None, max_version: Any = None, dl_device: Any = None,
                   copy: Any = None) -> Any:
        if copy:
            raise BufferError("DLPackExport never copies")
        return to_dlpack(self._t)


__all__ = ["DLPackExport", "from_dlpack", "to_dlpack"]
