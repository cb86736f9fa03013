"""Scatter and moves of a config-2 sized swizzled CUDA carrier in bulk.

``CUDA.scatter`` lands a tensor on the carrier through a mapping layout in
one device copy (the reference's native loop,
src/strideweave/carriers/cpu/native/_cpu_carrier.hpp:521-540, element by
element), and the CPU <-> CUDA moves map a swizzled carrier's flat index
space with one vectorised index map.  On X[8192 x 4096] each takes well
under a second, and the results equal the reference CPU carrier's bit for
bit.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, DType, Layout, Shape, Stride, Swizzle, SwizzleStage, Tensor  # noqa: E402

pytestmark = pytest.mark.gpu

R, C = 8192, 4096
TILED = Layout(Shape([[128, 64], [32, 128]]), Stride([[32, 128 * 32 * 128], [1, 128 * 32]]))


def cpu_carrier(flat: np.ndarray) -> CPU:
    carrier = CPU(flat.size)
    np.ctypeslib.as_array((ctypes.c_float * flat.size).from_address(carrier.pointer()))[:] = flat
    return carrier


def cpu_flat(carrier: CPU) -> np.ndarray:
    n = carrier.size()
    return np.ctypeslib.as_array((ctypes.c_float * n).from_address(carrier.pointer())).copy()


def test_scatter_through_a_tiled_mapping_onto_a_swizzled_carrier():
    from strideweave_b200 import CUDA

    size = R * C
    swz = Swizzle(Shape(size), SwizzleStage(bits=3, base=2, shift=3))
    x = np.random.default_rng(5).uniform(-1, 1, size=size).astype(np.float32)
    # X row-major, seen through the tiled shape tree: (r0 + 128 r1, c0 + 32 c1)
    rowmajor = Layout(Shape([[128, 64], [32, 128]]), Stride([[C, 128 * C], [1, 32]]))
    src = Tensor(CUDA.from_numpy(x), 0, rowmajor)
    dst = CUDA.from_numpy(np.zeros(size, np.float32), swizzle=swz)
    version = dst.version
    t0 = time.perf_counter()
    dst.scatter(src, Tensor(dst, 0, TILED), TILED, 0)
    got = dst.to_numpy()  # synchronises; logical (unswizzled) order
    elapsed = time.perf_counter() - t0
    assert dst.version > version
    want_carrier = CPU(size)
    want_carrier.scatter(Tensor(cpu_carrier(x), 0, rowmajor), Tensor(want_carrier, 0, TILED), TILED, 0)
    np.testing.assert_array_equal(got.view(np.uint32), cpu_flat(want_carrier).view(np.uint32))
    assert elapsed < 1.0, elapsed


def test_moves_of_a_swizzled_carrier_in_bulk():
    from strideweave_b200 import CUDA

    size = R * C
    swz = Swizzle(Shape(size), SwizzleStage(bits=3, base=2, shift=3))
    x = np.random.default_rng(6).uniform(-1, 1, size=size).astype(np.float32)
    src = Tensor(cpu_carrier(x), 0, TILED)
    t0 = time.perf_counter()
    on_gpu = sw.move(src, CUDA(size, swizzle=swz))
    N_sync()
    t_in = time.perf_counter() - t0
    # the device storage really is permuted (a move releases its source, so
    # look before moving back)
    raw = on_gpu.carrier.raw_numpy().view(np.float32)
    f = np.arange(size, dtype=np.int64)
    np.testing.assert_array_equal(raw[f ^ (((f >> 5) & 7) << 2)], x)
    t0 = time.perf_counter()
    back = sw.move(on_gpu, CPU(size, dtype=DType.Float32))
    t_out = time.perf_counter() - t0
    np.testing.assert_array_equal(cpu_flat(back.carrier).view(np.uint32), x.view(np.uint32))
    assert t_in + t_out < 1.0, (t_in, t_out)


def N_sync() -> None:
    from strideweave_b200 import _native as N

    N.synchronize()
