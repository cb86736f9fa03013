"""ctypes binding of the B200 carrier library (``include/strideweave_b200.h``).

The library is the only compute path of this package: there is no CPU
fallback.  Importing this module on a machine where the library was never
built raises ``ImportError`` naming the build command.  Every wrapper checks
the returned status and raises the matching Python exception with the
library's own message, mirroring the reference's error behaviour
(``ValueError`` for shapes/strides, ``NotImplementedError`` for plans no kernel
implements, ``RuntimeError`` for device failures).
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libswb200.so"

SW_OK = 0
SW_ERR_INVALID = 1
SW_ERR_UNSUPPORTED = 2
SW_ERR_CUDA = 3
SW_ERR_TIMEOUT = 4
SW_ERR_NOMEM = 5

SW_MAX_LEAVES = 8
SW_MAX_SWIZZLE = 4

SW_REDUCE_SUM = 0
SW_REDUCE_MAX = 1
SW_REDUCE_ARGMAX = 2
SW_REDUCE_SUM_F64 = 3
SW_ACC_F32 = 0
SW_ACC_F64 = 1

SW_MX_E4M3 = 1
SW_MX_E2M1 = 2
SW_SCALES_ROWMAJOR = 0
SW_SCALES_TC128 = 1
SW_OUT_F32 = 0
SW_OUT_BF16 = 1
SW_EW_GELU = 0
SW_EW_GELU_GRAD = 1
SW_EW_AXPY = 2
SW_BIN_MUL = 0
SW_MAP_ADD = 0
SW_MAP_SUB = 1
SW_MAP_MUL = 2
SW_MAP_SCALE = 3
SW_MAP_POW = 4
SW_MAP_POW_GRAD = 5
SW_XF_NONE = 0
SW_XF_GELU = 1
SW_XF_GELU_GRAD = 2
SW_NCCL_ID_BYTES = 128
SW_IPC_HANDLE_BYTES = 64


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait gave up (the kernel unwound cleanly)."""


class ReducePlan(ctypes.Structure):
    """Mirror of ``sw_reduce_plan``."""

    _fields_ = [
        ("kind", c_int32),
        ("kept_rank", c_int32),
        ("reduced_rank", c_int32),
        ("swizzle_rank", c_int32),
        ("offset", c_int64),
        ("kept_shape", c_int64 * SW_MAX_LEAVES),
        ("kept_stride", c_int64 * SW_MAX_LEAVES),
        ("reduced_shape", c_int64 * SW_MAX_LEAVES),
        ("reduced_stride", c_int64 * SW_MAX_LEAVES),
        ("swizzle_bits", c_int32 * SW_MAX_SWIZZLE),
        ("swizzle_base", c_int32 * SW_MAX_SWIZZLE),
        ("swizzle_shift", c_int32 * SW_MAX_SWIZZLE),
    ]


# name -> (restype, argtypes); exactly the functions the header declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "sw_last_error": (c_char_p, []),
    "sw_abi_version": (c_int, []),
    "sw_device_count": (c_int, [POINTER(c_int)]),
    "sw_set_device": (c_int, [c_int]),
    "sw_get_device": (c_int, [POINTER(c_int)]),
    "sw_alloc": (c_int, [POINTER(c_void_p), c_int64]),
    "sw_free": (c_int, [c_void_p]),
    "sw_memcpy_h2d": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "sw_memcpy_d2h": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "sw_memcpy_d2h_async": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "sw_memcpy_d2d": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "sw_memset": (c_int, [c_void_p, c_int, c_int64, c_void_p]),
    "sw_host_alloc": (c_int, [POINTER(c_void_p), c_int64]),
    "sw_host_free": (c_int, [c_void_p]),
    "sw_stream_create": (c_int, [POINTER(c_void_p)]),
    "sw_stream_destroy": (c_int, [c_void_p]),
    "sw_stream_synchronize": (c_int, [c_void_p]),
    "sw_device_sm_count": (c_int, [POINTER(c_int)]),
    "sw_event_create": (c_int, [POINTER(c_void_p), c_int]),
    "sw_event_destroy": (c_int, [c_void_p]),
    "sw_event_record": (c_int, [c_void_p, c_void_p]),
    "sw_stream_wait_event": (c_int, [c_void_p, c_void_p]),
    "sw_event_elapsed_ms": (c_int, [c_void_p, c_void_p, POINTER(ctypes.c_float)]),
    "sw_probe_bounded_wait": (c_int, [c_int64, c_void_p]),
    "sw_nccl_get_unique_id": (c_int, [c_void_p]),
    "sw_nccl_comm_init": (c_int, [POINTER(c_void_p), c_int, c_int, c_void_p]),
    "sw_nccl_reduce_scatter_f32": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "sw_nccl_all_gather_f32": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "sw_nccl_comm_destroy": (c_int, [c_void_p]),
    "sw_graph_capture_begin": (c_int, [c_void_p]),
    "sw_graph_capture_end": (c_int, [c_void_p, POINTER(c_void_p)]),
    "sw_graph_launch": (c_int, [c_void_p, c_void_p]),
    "sw_graph_destroy": (c_int, [c_void_p]),
    "sw_device_status": (c_int, [POINTER(c_int)]),
    "sw_reduce_f32": (c_int, [POINTER(ReducePlan), c_void_p, c_int64, c_void_p, c_void_p]),
    "sw_reduce_f32_noalloc": (c_int, [POINTER(ReducePlan), c_void_p, c_int64, c_void_p, c_void_p]),
    "sw_reduce_backward_f32": (
        c_int, [POINTER(ReducePlan), c_void_p, c_int64, c_void_p, c_void_p, POINTER(ReducePlan), c_int64, c_void_p],
    ),
    "sw_copy_view_f32": (
        c_int, [POINTER(ReducePlan), c_void_p, c_int64, POINTER(ReducePlan), c_void_p, c_int64, c_void_p],
    ),
    "sw_elementwise_f32": (c_int, [c_int, c_int64, c_void_p, c_void_p, c_void_p, ctypes.c_float, c_void_p]),
    "sw_mse_f32": (c_int, [c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "sw_mx_scale_index": (c_int64, [c_int64, c_int64, c_int64]),
    "sw_mx_scale_bytes_tc128": (c_int64, [c_int64, c_int64]),
    "sw_mx_quantize": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p],
    ),
    "sw_mx_quantize_view": (
        c_int,
        [c_int, POINTER(ReducePlan), c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p],
    ),
    "sw_mx_scales_to_tc128": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "sw_mx_quantize_dual": (
        c_int,
        [c_int, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64,
         c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p],
    ),
    "sw_mx_dequantize": (
        c_int,
        [c_int, c_void_p, c_int64, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p],
    ),
    "sw_mx_gemm": (
        c_int,
        [
            c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int,
            c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p,
        ],
    ),
    "sw_mx_gemm_ex": (
        c_int,
        [
            c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int,
            c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int, c_void_p,
        ],
    ),
    "sw_mx_gemm_batched": (
        c_int,
        [
            c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int,
            c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p,
        ],
    ),
    "sw_matmul_f32": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_void_p],
    ),
    "sw_matmul_f32_batched_ex": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p],
    ),
    "sw_matmul_f32_batched": (
        c_int,
        [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64,
         c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p],
    ),
    "sw_binary_f32": (
        c_int,
        [c_int, c_int, POINTER(c_int64), c_void_p, c_int64, POINTER(c_int64), c_int64, c_void_p, c_int64,
         POINTER(c_int64), c_int64, c_void_p, c_int64, POINTER(c_int64), c_int64, c_void_p],
    ),
    "sw_ipc_alloc": (c_int, [POINTER(c_void_p), c_int64, c_void_p]),
    "sw_ipc_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "sw_ipc_close": (c_int, [c_void_p]),
    "sw_ipc_free": (c_int, [c_void_p]),
    "sw_peer_wait": (c_int, [c_void_p, c_int, ctypes.c_uint32, c_int64, c_void_p]),
    "sw_peer_signal": (c_int, [POINTER(c_void_p), c_int, ctypes.c_uint32, c_void_p]),
    "sw_sum_slots_f32": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "sw_mx_gemm_routed": (
        c_int,
        [c_int, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, POINTER(c_void_p), c_int, c_int64, c_int64,
         c_int, c_int64, c_int64, c_int64, c_int, c_void_p],
    ),
    "sw_map_f32": (
        c_int,
        [c_int, c_int, POINTER(c_int64), c_void_p, c_int64, POINTER(c_int64), c_int64, c_void_p, c_int64,
         POINTER(c_int64), c_int64, c_void_p, c_int64, POINTER(c_int64), c_int64, ctypes.c_float, c_void_p],
    ),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"B200 carrier library not built ({LIB_PATH}); run "
            "`python -m strideweave_b200.build` (needs nvcc with sm_100a support)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


def last_error() -> str:
    raw = lib.sw_last_error()
    return raw.decode("utf-8", "replace") if raw else ""


def check(rc: int, what: str = "") -> None:
    """Raise the exception matching a non-zero status code."""
    if rc == SW_OK:
        return
    message = last_error() or what or f"status {rc}"
    if rc == SW_ERR_INVALID:
        raise ValueError(message)
    if rc == SW_ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    if rc == SW_ERR_TIMEOUT:
        raise DeviceTimeout(message)
    if rc == SW_ERR_NOMEM:
        raise MemoryError(message)
    raise RuntimeError(message)


def device_count() -> int:
    n = c_int(0)
    check(lib.sw_device_count(ctypes.byref(n)))
    return n.value


def set_device(device: int) -> None:
    check(lib.sw_set_device(int(device)))


def current_device() -> int:
    d = c_int(0)
    check(lib.sw_get_device(ctypes.byref(d)))
    return d.value


def device_status() -> int:
    """Synchronise, then read and clear the device-side error word."""
    s = c_int(0)
    check(lib.sw_device_status(ctypes.byref(s)))
    return s.value


def raise_device_status() -> None:
    status = device_status()
    if status == SW_ERR_TIMEOUT:
        raise DeviceTimeout("a bounded device-side wait gave up")
    if status != SW_OK:
        raise RuntimeError(f"device-side check failed with status {status}")


class DeviceBuffer:
    """Owned device allocation (``sw_alloc`` / ``sw_free``)."""

    __slots__ = ("ptr", "nbytes", "__weakref__")

    def __init__(self, nbytes: int) -> None:
        if nbytes < 0:
            raise ValueError("allocation size must be non-negative")
        p = c_void_p(0)
        check(lib.sw_alloc(ctypes.byref(p), int(nbytes)))
        self.ptr = p.value or 0
        self.nbytes = int(nbytes)

    def free(self) -> None:
        if self.ptr:
            check(lib.sw_free(c_void_p(self.ptr)))
            self.ptr = 0
            self.nbytes = 0

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            if self.ptr:
                lib.sw_free(c_void_p(self.ptr))
                self.ptr = 0
        except Exception:
            pass

    def upload(self, host, stream: int | None = None) -> None:
        """Copy a C-contiguous numpy array into the start of the buffer."""
        n = host.nbytes
        if n > self.nbytes:
            raise ValueError("host array larger than the device buffer")
        check(lib.sw_memcpy_h2d(c_void_p(self.ptr), c_void_p(host.ctypes.data), n, c_void_p(stream or 0)))

    def download(self, host, stream: int | None = None) -> None:
        """Copy the start of the buffer into a C-contiguous numpy array."""
        n = host.nbytes
        if n > self.nbytes:
            raise ValueError("host array larger than the device buffer")
        check(lib.sw_memcpy_d2h(c_void_p(host.ctypes.data), c_void_p(self.ptr), n, c_void_p(stream or 0)))


def synchronize(stream: int | None = None) -> None:
    check(lib.sw_stream_synchronize(c_void_p(stream or 0)))


def sm_count() -> int:
    """SMs of the current device."""
    n = c_int(0)
    check(lib.sw_device_sm_count(ctypes.byref(n)))
    return n.value


class Stream:
    """A non-blocking stream of the current device (``sw_stream_create``);
    ``handle`` is the ``cudaStream_t`` the C entry points take."""

    __slots__ = ("handle", "__weakref__")

    def __init__(self) -> None:
        s = c_void_p(0)
        check(lib.sw_stream_create(ctypes.byref(s)))
        self.handle = s.value or 0

    def synchronize(self) -> None:
        synchronize(self.handle)

    def close(self) -> None:
        if self.handle:
            check(lib.sw_stream_destroy(c_void_p(self.handle)))
            self.handle = 0

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            if self.handle:
                lib.sw_stream_destroy(c_void_p(self.handle))
                self.handle = 0
        except Exception:
            pass


class Event:
    """A CUDA event (``sw_event_*``): orders one stream after another's work,
    or, created with ``timing=True``, times work on the device."""

    __slots__ = ("handle", "__weakref__")

    def __init__(self, timing: bool = False) -> None:
        e = c_void_p(0)
        check(lib.sw_event_create(ctypes.byref(e), int(bool(timing))))
        self.handle = e.value or 0

    def record(self, stream: int = 0) -> None:
        check(lib.sw_event_record(c_void_p(self.handle), c_void_p(stream or 0)))

    def wait(self, stream: int = 0) -> None:
        """Work enqueued on ``stream`` after this call waits for the event."""
        check(lib.sw_stream_wait_event(c_void_p(stream or 0), c_void_p(self.handle)))

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float(0.0)
        check(lib.sw_event_elapsed_ms(c_void_p(self.handle), c_void_p(end.handle), ctypes.byref(ms)))
        return float(ms.value)

    def close(self) -> None:
        if self.handle:
            check(lib.sw_event_destroy(c_void_p(self.handle)))
            self.handle = 0

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            if self.handle:
                lib.sw_event_destroy(c_void_p(self.handle))
                self.handle = 0
        except Exception:
            pass
