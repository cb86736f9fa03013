"""Device-buffer helpers shared by the GPU tests (numpy in, numpy out)."""

from __future__ import annotations

import numpy as np

from strideweave_b200 import _native as N


def to_device(a: np.ndarray) -> N.DeviceBuffer:
    a = np.ascontiguousarray(a)
    buf = N.DeviceBuffer(max(a.nbytes, 16))
    buf.upload(a)
    return buf


def empty(nbytes: int, fill: int | None = None) -> N.DeviceBuffer:
    buf = N.DeviceBuffer(max(int(nbytes), 16))
    if fill is not None:
        N.check(N.lib.sw_memset(N.c_void_p(buf.ptr), int(fill), buf.nbytes, None))
    return buf


def to_host(buf: N.DeviceBuffer, shape, dtype) -> np.ndarray:
    out = np.empty(shape, dtype=dtype)
    N.synchronize()
    buf.download(out)
    return out


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32)


def rel_frobenius(got: np.ndarray, want: np.ndarray) -> float:
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))
