"""The CUDA carrier: a StrideWeave ``Carrier`` whose flat index space lives in
the HBM of one B200.

It is a sibling of the reference's closed carriers (``CPU``, ``Generic``,
``FileBacked``, ``Evictable``), implementing the ``Carrier`` interface of
src/strideweave/core/native/_carrier.hpp:19-196: ``size``, ``dtype``,
``get_value``, ``new_like``, ``allocate_like``, ``scatter``, ``_dispatch_op``,
``_is_mutable``, ``_supports_storage_dtype``, ``set_value``, ``_release`` and
``dlpack_info``.  Ownership, versioning and release are inherited from the
native base.

Storage is one ``sw_alloc`` allocation of one simple dtype: Float32, Int32,
Bool (1 byte), the MX plane dtypes E4M3 / E8M0 (1 byte) and E2M1 (two elements
per byte, even index in the low nibble), and the BFloat16 extension dtype.
A carrier may store its flat index space through a StrideWeave ``Swizzle``:
element ``f`` then lives at ``swizzle(f)``, which every access and every kernel
applies.  Tensor placement stays a ``Layout``, as the reference requires
(src/strideweave/core/index_map.py:143-144).

All work is enqueued on the legacy default stream of the carrier's device, so
operations are ordered with each other and with copies; host reads
(``get_value``, ``to_numpy``) and DLPack export synchronise first.
"""

from __future__ import annotations

import math
from collections.abc import Iterable
from ctypes import c_void_p
from operator import index as operator_index
from typing import Any

import numpy as np

from . import _native as N
from ._host import BFloat16, Carrier, DType, Swizzle
from .layout_plan import swizzle_map, swizzle_stages

FLOAT32 = DType.Float32
INT32 = DType.Int32
BOOL = DType.Bool
E4M3 = DType.E4M3
E8M0 = DType.E8M0
E2M1 = DType.E2M1

_BITS = {FLOAT32: 32, INT32: 32, BOOL: 8, E4M3: 8, E8M0: 8, E2M1: 4, BFloat16: 16}
_NUMPY = {FLOAT32: np.float32, INT32: np.int32, BOOL: np.uint8, E4M3: np.uint8, E8M0: np.uint8, E2M1: np.uint8,
          BFloat16: np.uint16}
STORAGE_DTYPES = tuple(_BITS)


def _decode_table(dtype: Any) -> np.ndarray:
    """Float value of every code of a narrow floating dtype (exact)."""
    if dtype is E4M3:
        codes = np.arange(256)
        s, f, m = codes >> 7, (codes >> 3) & 15, codes & 7
        v = np.where(f == 0, m * 2.0 ** -9, (1 + m / 8.0) * np.exp2(f - 7.0))
        v = np.where((f == 15) & (m == 7), np.nan, v)
        return np.where(s == 1, -v, v)
    if dtype is E2M1:
        codes = np.arange(16)
        s, f, m = codes >> 3, (codes >> 1) & 3, codes & 1
        v = np.where(f == 0, m * 0.5, (1 + m / 2.0) * np.exp2(f - 1.0))
        return np.where(s == 1, -v, v)
    if dtype is E8M0:
        codes = np.arange(256)
        return np.where(codes == 255, np.nan, np.exp2(codes - 127.0))
    raise TypeError(dtype)


_TABLES: dict[Any, np.ndarray] = {}


def _table(dtype: Any) -> np.ndarray:
    if dtype not in _TABLES:
        _TABLES[dtype] = _decode_table(dtype)
    return _TABLES[dtype]


def storage_bytes(dtype: Any, size: int) -> int:
    return (size * _BITS[dtype] + 7) // 8


def _encode_exact(dtype: Any, values: np.ndarray) -> np.ndarray:
    """Codes of values that are exactly representable in a narrow dtype."""
    table = _table(dtype)
    out = np.empty(values.shape, dtype=np.uint8)
    for i, v in enumerate(values.ravel()):
        v = float(v)
        if math.isnan(v):
            hits = np.flatnonzero(np.isnan(table))
        else:
            hits = np.flatnonzero(table == v)
            if v == 0.0 and hits.size > 1:  # keep the sign of zero
                hits = hits[[1 if math.copysign(1.0, v) < 0 else 0]]
        if hits.size == 0:
            raise ValueError(f"{v!r} is not representable in {dtype.name}; create MX planes with "
                             "strideweave_b200.mx.quantize")
        out.ravel()[i] = hits[0]
    return out


def _host_array(dtype: Any, values: Iterable[Any]) -> np.ndarray:
    """Normalise Python values into this dtype's storage encoding."""
    vals = list(values)
    if dtype is FLOAT32:
        return np.asarray([0.0 if v is None else float(v) for v in vals], dtype=np.float32)
    if dtype is INT32:
        out = np.empty(len(vals), dtype=np.int32)
        for i, v in enumerate(vals):
            iv = 0 if v is None else operator_index(v)
            if not -(2 ** 31) <= iv < 2 ** 31:
                raise OverflowError("CUDA value is out of int32 range")
            out[i] = iv
        return out
    if dtype is BOOL:
        for v in vals:
            if v is not None and not isinstance(v, (bool, np.bool_)):
                raise TypeError("CUDA value must be a bool for Bool storage")
        return np.asarray([1 if v else 0 for v in vals], dtype=np.uint8)
    if dtype is BFloat16:
        f = np.asarray([0.0 if v is None else float(v) for v in vals], dtype=np.float32)
        bits = f.view(np.uint32).astype(np.uint64)
        rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)  # nearest-even
        rounded[np.isnan(f)] = 0x7FC0
        return rounded
    codes = _encode_exact(dtype, np.asarray([0.0 if v is None else float(v) for v in vals], dtype=np.float64))
    if dtype is E2M1:
        padded = np.zeros(len(codes) + (len(codes) & 1), dtype=np.uint8)
        padded[: len(codes)] = codes
        return (padded[0::2] | (padded[1::2] << 4)).astype(np.uint8)
    return codes


class CUDA(Carrier):
    """Device storage of one simple dtype on one B200.

    Args:
        size: Number of elements of the flat index space.
        mutable: Whether public interfaces may modify the storage.
        dtype: Storage dtype (Float32, Int32, Bool, E4M3, E8M0, E2M1, BFloat16).
        empty: Leave owned storage uninitialised instead of zero-filled.
        device: CUDA device ordinal (default: the current device).
        swizzle: Optional ``Swizzle`` over ``Shape(size)``; element ``f`` is
            stored at ``swizzle(f)``.
    """

    def __init__(self, size: int, *, mutable: bool = True, dtype: Any = FLOAT32, empty: bool = False,
                 device: int | None = None, swizzle: Swizzle | None = None) -> None:
        super().__init__()
        size = operator_index(size)
        if size < 0:
            raise ValueError("CUDA size must be non-negative")
        if dtype not in _BITS:
            raise TypeError(f"CUDA does not store dtype {getattr(dtype, 'name', dtype)!r}")
        if swizzle is not None:
            if not isinstance(swizzle, Swizzle):
                raise TypeError("swizzle must be a Swizzle")
            if swizzle.size != size:
                raise ValueError("a carrier swizzle must cover exactly the carrier's flat index space")
        self._size = size
        self._dtype = dtype
        self._mutable = bool(mutable)
        self._swizzle = swizzle
        current = N.current_device()
        self._device = current if device is None else int(device)
        if self._device != current:
            N.set_device(self._device)
        self._nbytes = storage_bytes(dtype, size)
        self._buffer: N.DeviceBuffer | None = N.DeviceBuffer(self._nbytes)
        if not empty and self._nbytes:
            N.check(N.lib.sw_memset(c_void_p(self._buffer.ptr), 0, self._nbytes, None))

    # ---- Carrier interface -----------------------------------------------------

    def size(self) -> int:
        return self._size

    def dtype(self) -> Any:
        return self._dtype

    def _is_mutable(self) -> bool:
        return self._mutable

    def _supports_storage_dtype(self, dtype: Any) -> bool:
        return any(dtype is d for d in STORAGE_DTYPES)

    def _release(self) -> None:
        if self._buffer is not None:
            self._buffer.free()
            self._buffer = None
        self._size = 0

    def get_value(self, index: int) -> Any:
        raw = self._read_raw(operator_index(index))
        return self._decode(raw)

    def set_value(self, index: int, value: Any) -> None:
        if not self.is_mutable():
            raise RuntimeError("Carrier is not mutable")
        index = operator_index(index)
        if not 0 <= index < self._size:
            raise IndexError("Carrier index out of range")
        p = self.physical_index(index)
        if self._dtype is E2M1:
            code = int(_encode_exact(E2M1, np.asarray([float(value)]))[0])
            byte = self._read_bytes(p // 2, 1)[0]
            byte = (byte & 0xF0) | code if p % 2 == 0 else (byte & 0x0F) | (code << 4)
            self._write_bytes(p // 2, np.asarray([byte], dtype=np.uint8))
        else:
            enc = _host_array(self._dtype, [value])
            self._write_bytes(p * (_BITS[self._dtype] // 8), enc.view(np.uint8))
        self._increment_version()

    def new_like(self, values: Iterable[Any], *, mutable: bool = True, dtype: Any = None) -> CUDA:
        target = self._dtype if dtype is None else dtype
        host = _host_array(target, values)
        size = len(host) if target is not E2M1 else None
        if target is E2M1:
            size = len(list(values)) if not hasattr(values, "__len__") else len(values)  # type: ignore[arg-type]
        out = CUDA(size, mutable=mutable, dtype=target, empty=True, device=self._device)
        if host.nbytes:
            out._buffer.upload(np.ascontiguousarray(host))
        return out

    def _allocate(self, size: int) -> None:
        """Give an empty carrier (``CUDA(0)``) storage for ``size`` elements;
        ``sw.move`` calls it to size a destination to the moved layout."""
        size = operator_index(size)
        if self._size != 0:
            raise RuntimeError("only an empty CUDA carrier can be allocated")
        if size < 0:
            raise ValueError("CUDA size must be non-negative")
        if self._swizzle is not None:
            raise ValueError("a swizzled carrier cannot change size")
        nbytes = storage_bytes(self._dtype, size)
        buffer = N.DeviceBuffer(nbytes)
        if nbytes:
            N.check(N.lib.sw_memset(c_void_p(buffer.ptr), 0, nbytes, None))
        if self._buffer is not None:
            self._buffer.free()
        self._buffer = buffer
        self._size = size
        self._nbytes = nbytes

    def allocate_like(self, size: int, *, mutable: bool = True, dtype: Any = None, empty: bool = False) -> CUDA:
        size = operator_index(size)
        if size < 0:
            raise ValueError("CUDA allocation size must be non-negative")
        return CUDA(size, mutable=mutable, dtype=self._dtype if dtype is None else dtype, empty=empty,
                    device=self._device)

    def scatter(self, to_scatter: Any, scatter_onto: Any, mapping: Any, mapping_offset: int = 0) -> None:
        from ._host import Layout, Tensor

        if not self.is_mutable():
            raise RuntimeError("Carrier is not mutable")
        if not isinstance(to_scatter, Tensor) or not isinstance(scatter_onto, Tensor):
            raise TypeError("to_scatter and scatter_onto must be Tensors")
        if not isinstance(mapping, Layout):
            raise TypeError("mapping must be a Layout")
        to_scatter._require_single_subtensor("scatter")
        scatter_onto._require_single_subtensor("scatter")
        if scatter_onto.carrier is not self:
            raise ValueError("scatter_onto must be backed by this carrier")
        if mapping.shape != to_scatter.layout.shape:
            raise ValueError("mapping shape must match to_scatter layout shape")
        offset = operator_index(mapping_offset)
        if offset < 0:
            raise ValueError("mapping_offset must be non-negative")
        if self._scatter_on_device(to_scatter, scatter_onto.offset + offset, mapping):
            return
        for logical in range(to_scatter.size()):
            self[scatter_onto.offset + offset + mapping.index(logical)] = to_scatter[logical]

    def _scatter_on_device(self, to_scatter: Any, base: int, mapping: Any) -> bool:
        """One view-copy launch: element i of to_scatter (its layout, through
        its carrier's swizzle) lands at flat index base + mapping(i) of this
        carrier (through this carrier's swizzle), as the reference's native
        loop does element by element (src/strideweave/carriers/cpu/native/
        _cpu_carrier.hpp:521-540).  32-bit dtypes on CUDA carriers of this
        device; anything else returns False and takes the element loop."""
        from . import kernels
        from .layout_plan import all_leaves, coalesce, swizzle_stages

        src = to_scatter.carrier
        if (not isinstance(src, CUDA) or src.device != self._device or _BITS[self._dtype] != 32
                or _BITS[src.dtype()] != 32 or src.dtype() is not self._dtype):
            return False
        src_leaves, dst_leaves = all_leaves(to_scatter.layout), all_leaves(mapping)
        if len(src_leaves) > N.SW_MAX_LEAVES or len(dst_leaves) > N.SW_MAX_LEAVES:
            src_leaves, dst_leaves = coalesce(src_leaves), coalesce(dst_leaves)
            if len(src_leaves) > N.SW_MAX_LEAVES or len(dst_leaves) > N.SW_MAX_LEAVES:
                return False
        if to_scatter.size() == 0:
            return True
        kernels.copy_view_f32(src.data_ptr, src.size(), to_scatter.offset, src_leaves or [(1, 0)], [(1, 0)],
                              self.data_ptr, self._size, base, dst_leaves or [(1, 0)], [(1, 0)],
                              swizzle=swizzle_stages(src), dst_swizzle=swizzle_stages(self))
        self._increment_version()
        return True

    def dlpack_info(self) -> dict:
        if self._dtype not in (FLOAT32, INT32):
            raise BufferError("DLPack export supports Float32 and Int32 carriers")
        if self._swizzle is not None:
            raise BufferError("a swizzled carrier has no strided DLPack view")
        N.synchronize()  # the reference exporter ignores the stream argument
        return {"pointer": self.data_ptr, "device_type": 2, "device_id": self._device}

    def _dispatch_op(self, operation_name: str) -> Any:
        from .ops import make_operation

        return make_operation(operation_name)

    # ---- CUDA-specific surface ---------------------------------------------------

    @property
    def swizzle(self) -> Swizzle | None:
        return self._swizzle

    @property
    def device(self) -> int:
        return self._device

    @property
    def nbytes(self) -> int:
        return self._nbytes

    @property
    def data_ptr(self) -> int:
        if self._buffer is None:
            raise RuntimeError("Carrier is released")
        return self._buffer.ptr

    def physical_index(self, index: int) -> int:
        if self._swizzle is None:
            return index
        return int(self._swizzle(index))

    def _read_bytes(self, byte_offset: int, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.uint8)
        N.check(N.lib.sw_memcpy_d2h(c_void_p(out.ctypes.data), c_void_p(self.data_ptr + byte_offset), count, None))
        return out

    def _write_bytes(self, byte_offset: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        N.check(N.lib.sw_memcpy_h2d(c_void_p(self.data_ptr + byte_offset), c_void_p(data.ctypes.data), data.nbytes,
                                    None))
        N.synchronize()

    def _read_raw(self, index: int) -> int:
        if not 0 <= index < self._size:
            raise IndexError("Carrier index out of range")
        p = self.physical_index(index)
        if self._dtype is E2M1:
            byte = int(self._read_bytes(p // 2, 1)[0])
            return (byte >> (4 * (p % 2))) & 0xF
        width = _BITS[self._dtype] // 8
        raw = self._read_bytes(p * width, width)
        return int.from_bytes(raw.tobytes(), "little", signed=self._dtype is INT32)

    def _decode(self, raw: int) -> Any:
        d = self._dtype
        if d is FLOAT32:
            return float(np.array([raw], dtype=np.uint32).view(np.float32)[0])
        if d is INT32:
            return int(raw)
        if d is BOOL:
            return raw != 0
        if d is BFloat16:
            return float(np.array([raw << 16], dtype=np.uint32).view(np.float32)[0])
        return float(_table(d)[raw])

    def to_numpy(self) -> np.ndarray:
        """The flat index space as a host array in logical order (decoded for
        narrow float dtypes; E8M0 as scale values)."""
        N.synchronize()
        d = self._dtype
        if self._swizzle is not None and _BITS[d] == 32 and self._size:
            # un-swizzle on the device (one view copy), then one download
            from . import kernels

            staged = N.DeviceBuffer(self._nbytes)
            kernels.copy_view_f32(self.data_ptr, self._size, 0, [(self._size, 1)], [(1, 0)], staged.ptr, self._size,
                                  0, [(self._size, 1)], [(1, 0)], swizzle=swizzle_stages(self))
            out = np.empty(self._size, dtype=_NUMPY[d])
            staged.download(out)
            staged.free()
            return out
        raw = np.empty(self._nbytes, dtype=np.uint8)
        if self._nbytes:
            self._buffer.download(raw)
        if d is E2M1:
            codes = np.empty(self._nbytes * 2, dtype=np.uint8)
            codes[0::2] = raw & 0xF
            codes[1::2] = raw >> 4
            phys = codes[: self._size]
        else:
            phys = raw.view(_NUMPY[d])[: self._size]
        if self._swizzle is not None:
            phys = phys[swizzle_map(swizzle_stages(self), self._size)]
        if d is FLOAT32 or d is INT32:
            return phys.copy()
        if d is BOOL:
            return phys.astype(bool)
        if d is BFloat16:
            return (phys.astype(np.uint32) << 16).view(np.float32)
        return _table(d)[phys].astype(np.float32)

    def raw_numpy(self) -> np.ndarray:
        """The physical storage bytes (swizzled order, packed nibbles)."""
        N.synchronize()
        raw = np.empty(self._nbytes, dtype=np.uint8)
        if self._nbytes:
            self._buffer.download(raw)
        return raw

    @classmethod
    def from_numpy(cls, array: np.ndarray, *, dtype: Any = None, mutable: bool = True, device: int | None = None,
                   swizzle: Swizzle | None = None) -> CUDA:
        """Upload a host array as the logical flat index space (Float32 /
        Int32 / Bool arrays; the swizzle, if any, is applied on the way)."""
        arr = np.ascontiguousarray(array).ravel()
        if dtype is None:
            dtype = {np.dtype(np.float32): FLOAT32, np.dtype(np.int32): INT32, np.dtype(bool): BOOL}.get(arr.dtype)
            if dtype is None:
                raise TypeError(f"no CUDA storage dtype for numpy dtype {arr.dtype}")
        if dtype is FLOAT32:
            host = arr.astype(np.float32)
        elif dtype is INT32:
            host = arr.astype(np.int32)
        elif dtype is BOOL:
            host = arr.astype(np.uint8)
        else:
            host = _host_array(dtype, arr.tolist())
        out = cls(arr.size, dtype=dtype, mutable=mutable, empty=True, device=device, swizzle=swizzle)
        if swizzle is not None:
            if dtype is E2M1:
                raise NotImplementedError("swizzled E2M1 storage")
            phys = np.empty_like(host)
            phys[swizzle_map([(int(s.bits), int(s.base), int(s.shift)) for s in swizzle.stages], arr.size)] = host
            host = phys
        if host.nbytes:
            out._buffer.upload(np.ascontiguousarray(host))
        return out

    def upload_raw(self, data: np.ndarray, byte_offset: int = 0, stream: int = 0) -> None:
        """Copy raw bytes into the storage (no encoding, no swizzle)."""
        data = np.ascontiguousarray(data)
        if byte_offset < 0 or byte_offset + data.nbytes > self._nbytes:
            raise ValueError("raw upload outside the carrier storage")
        N.check(N.lib.sw_memcpy_h2d(c_void_p(self.data_ptr + byte_offset), c_void_p(data.ctypes.data), data.nbytes,
                                    c_void_p(stream)))

    def __repr__(self) -> str:
        extra = f", swizzle={self._swizzle!r}" if self._swizzle is not None else ""
        return f"CUDA(size={self._size}, dtype={self._dtype.name}, device={self._device}{extra})"


def _declare_capabilities() -> None:
    """Declare, at import, the exact plan shapes the CUDA carrier executes
    (register_operation_capabilities, src/strideweave/carriers/
    operation_capability.py:567-655): Float32 reduce_sum / reduce_max / argmax
    and the Float32 matmul plan."""
    from ._host import OperationCapability, register_operation_capabilities
    from .ops import declared_plans

    register_operation_capabilities(CUDA, [OperationCapability.from_plan(p) for p in declared_plans()])


_declare_capabilities()


def _register_moves() -> None:
    """CPU <-> CUDA bulk moves in the reference's move registry."""
    from .move import register

    register()


_register_moves()
