"""Python face of the CPU oracle (``oracle/sw_oracle.c``) - TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only as the checker.  The product package
``strideweave_b200`` never imports it.

The C file restates the reference CPU carrier's folds (reduce_sum, reduce_max,
argmax, matmul) and the OCP MX v1.0 quantiser; see its header for the
reference file:line each function follows.  Reductions and matmul are pinned
against the reference by ``tests/golden``; the quantiser is "parity
unpinned" against the reference (the reference has none) and is pinned by
exhaustive element-code known-answer tests instead.
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_uint32, c_void_p
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "sw_oracle.c"
BUILD_DIR = ORACLE_DIR / "_build"
LIB_PATH = BUILD_DIR / "libsworacle.so"

E4M3 = 1
E2M1 = 2


def build_oracle(force: bool = False) -> Path:
    """Compile the oracle with gcc (no fast-math, IEEE semantics)."""
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".tmp.so")
    subprocess.run(
        ["gcc", "-O2", "-std=gnu11", "-fPIC", "-shared", "-fno-fast-math", "-ffp-contract=off",
         str(SOURCE), "-o", str(tmp), "-lm"],
        check=True,
    )
    tmp.replace(LIB_PATH)
    return LIB_PATH


def _load() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build_oracle()))
    I64P = POINTER(c_int64)
    I32P = POINTER(c_int32)
    lib.sw_oracle_reduce.restype = c_int
    lib.sw_oracle_reduce.argtypes = [c_int, c_void_p, c_int64, c_int64, c_int, I64P, I64P, c_int, I64P, I64P,
                                     c_int, I32P, I32P, I32P, c_void_p]
    lib.sw_oracle_matmul.restype = None
    lib.sw_oracle_matmul.argtypes = [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64,
                                     c_int64, c_int64, c_int64, c_int64, c_int]
    lib.sw_oracle_mx_quantize.restype = c_int
    lib.sw_oracle_mx_quantize.argtypes = [c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64,
                                          c_void_p, c_int, c_int64]
    lib.sw_oracle_mx_dequantize.restype = c_int
    lib.sw_oracle_mx_dequantize.argtypes = [c_int, c_void_p, c_int64, c_void_p, c_int, c_int64, c_int64, c_int64,
                                            c_void_p, c_int64]
    lib.sw_oracle_scale_index_tc128.restype = c_int64
    lib.sw_oracle_scale_index_tc128.argtypes = [c_int64, c_int64, c_int64]
    lib.sw_oracle_encode_elem.restype = c_uint32
    lib.sw_oracle_encode_elem.argtypes = [c_int, c_float]
    lib.sw_oracle_decode_elem.restype = c_double
    lib.sw_oracle_decode_elem.argtypes = [c_int, c_uint32]
    return lib


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _arr64(values, n=8):
    a = (c_int64 * max(n, 1))()
    for i, v in enumerate(values):
        a[i] = int(v)
    return a


def _arr32(values, n=4):
    a = (c_int32 * max(n, 1))()
    for i, v in enumerate(values):
        a[i] = int(v)
    return a


KIND = {"sum": 0, "max": 1, "argmax": 2, "sum64": 3}


def reduce(kind: str, storage: np.ndarray, offset: int, kept: list[tuple[int, int]],
           reduced: list[tuple[int, int]], swizzle: list[tuple[int, int, int]] | None = None) -> np.ndarray:
    """Sequential fold over a (kept, reduced) leaf plan of a flat float32 carrier.

    ``kept`` / ``reduced`` are (shape, stride) leaves, first leaf fastest;
    ``swizzle`` is a list of (bits, base, shift) XOR stages applied to each
    flat index.
    """
    storage = np.ascontiguousarray(storage, dtype=np.float32)
    n = int(np.prod([s for s, _ in kept])) if kept else 1
    out = np.empty(n, dtype=np.int32 if kind == "argmax" else np.float32)
    swz = swizzle or []
    rc = lib().sw_oracle_reduce(
        KIND[kind], storage.ctypes.data, storage.size, offset,
        len(kept), _arr64([s for s, _ in kept]), _arr64([d for _, d in kept]),
        len(reduced), _arr64([s for s, _ in reduced]), _arr64([d for _, d in reduced]),
        len(swz), _arr32([b for b, _, _ in swz]), _arr32([b for _, b, _ in swz]), _arr32([s for _, _, s in swz]),
        out.ctypes.data)
    if rc == 1:
        raise ValueError("reduction fibers must be non-empty")
    if rc == 2:
        raise IndexError("view addresses outside the storage")
    return out


def matmul(a: np.ndarray, b: np.ndarray, *, acc64: bool = False) -> np.ndarray:
    """C[m, n] = sum_k A[m, k] * B[n, k] exactly as the reference CPU kernel."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    M, K = a.shape
    N, K2 = b.shape
    assert K == K2
    c = np.empty((M, N), dtype=np.float32)
    lib().sw_oracle_matmul(a.ctypes.data, a.strides[0] // 4, a.strides[1] // 4, b.ctypes.data, b.strides[0] // 4,
                           b.strides[1] // 4, c.ctypes.data, N, 1, M, N, K, int(acc64))
    return c


def scale_bytes_tc128(rows: int, kblocks: int) -> int:
    return ((rows + 127) // 128) * ((kblocks + 3) // 4) * 512


def mx_quantize(fmt: int, x: np.ndarray, *, scale_layout: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Quantise rows of ``x`` (blocks of 32 along axis 1).

    Returns (payload[rows, row_bytes] uint8, scales uint8) where scales is
    [rows, kblocks] for the row-major placement or the flat padded atom plane
    for the TC128 placement.
    """
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    kblocks = (cols + 31) // 32
    row_bytes = cols if fmt == E4M3 else (cols + 1) // 2
    payload = np.zeros((rows, row_bytes), dtype=np.uint8)
    if scale_layout == 1:
        scales = np.full(scale_bytes_tc128(rows, kblocks), 127, dtype=np.uint8)
        lds = 0
    else:
        scales = np.zeros((rows, kblocks), dtype=np.uint8)
        lds = kblocks
    rc = lib().sw_oracle_mx_quantize(fmt, x.ctypes.data, rows, cols, x.strides[0] // 4, x.strides[1] // 4,
                                     payload.ctypes.data, row_bytes, scales.ctypes.data, scale_layout, lds)
    assert rc == 0
    return payload, scales


def mx_dequantize(fmt: int, payload: np.ndarray, scales: np.ndarray, rows: int, cols: int, *,
                  scale_layout: int = 0) -> np.ndarray:
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    kblocks = (cols + 31) // 32
    rc = lib().sw_oracle_mx_dequantize(fmt, payload.ctypes.data, payload.shape[1], scales.ctypes.data,
                                       scale_layout, kblocks, rows, cols, out.ctypes.data, cols)
    assert rc == 0
    return out


def scale_index_tc128(r: int, kb: int, kblocks: int) -> int:
    return int(lib().sw_oracle_scale_index_tc128(r, kb, kblocks))


def encode_elem(fmt: int, value: float) -> int:
    return int(lib().sw_oracle_encode_elem(fmt, value))


def decode_elem(fmt: int, code: int) -> float:
    return float(lib().sw_oracle_decode_elem(fmt, code))


def swizzle_index(index: int, stages: list[tuple[int, int, int]]) -> int:
    """Python restatement of Swizzle._index_ordinal (core/swizzle.py:107-117)."""
    r = index
    for bits, base, shift in stages:
        mask = (1 << bits) - 1
        if shift > 0:
            r ^= ((r >> (base + shift)) & mask) << base
        else:
            r ^= ((r >> base) & mask) << (base - shift)
    return r
