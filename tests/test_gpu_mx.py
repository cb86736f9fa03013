"""MX quantise / dequantise kernels against the CPU restatement of OCP MX v1.0,
bit for bit, through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from strideweave_b200 import _native as N
from tests.gpu_util import empty, to_device, to_host

pytestmark = pytest.mark.gpu


def adversarial(rows: int, cols: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    # wide dynamic range per row, so every scale byte region is exercised
    x = rng.standard_normal((rows, cols)) * np.exp2(rng.integers(-140, 120, size=(rows, 1)))
    x = x.astype(np.float32)
    flat = x.reshape(-1)
    n = flat.size
    picks = rng.choice(n, size=min(n, 64), replace=False)
    specials = [np.nan, np.inf, -np.inf, 0.0, -0.0, 448.0, 464.0, 470.0, 6.0, 2.0 ** -149, -(2.0 ** -126),
                3.4e38, 1e-45]
    for i, p in enumerate(picks):
        flat[p] = specials[i % len(specials)]
    if rows > 3 and cols >= 32:
        x[1, :32] = 0.0
        x[2, :32] = -0.0
        x[3, :32] = np.float32(2.0 ** -128)
    return x


def gpu_quantize(fmt, x, scale_layout, transposed=False):
    rows, cols = x.shape
    kblocks = (cols + 31) // 32
    row_bytes = cols if fmt == O.E4M3 else (cols + 1) // 2
    if transposed:
        store = np.ascontiguousarray(x.T)  # element (r, c) at c*rows + r
        ld_row, ld_col = 1, rows
    else:
        store = np.ascontiguousarray(x)
        ld_row, ld_col = cols, 1
    dx = to_device(store)
    payload = empty(rows * row_bytes, fill=0)
    if scale_layout == N.SW_SCALES_TC128:
        sbytes = O.scale_bytes_tc128(rows, kblocks)
        lds = 0
    else:
        sbytes = rows * kblocks
        lds = kblocks
    scales = empty(sbytes, fill=0)
    from strideweave_b200 import kernels

    kernels.mx_quantize(fmt, dx.ptr, rows, cols, ld_row, ld_col, payload.ptr, row_bytes, scales.ptr,
                        scale_layout=scale_layout, ld_scales=lds)
    p = to_host(payload, (rows, row_bytes), np.uint8)
    s = to_host(scales, sbytes, np.uint8)
    if scale_layout == N.SW_SCALES_ROWMAJOR:
        s = s.reshape(rows, kblocks)
    return p, s


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("scale_layout", [N.SW_SCALES_ROWMAJOR, N.SW_SCALES_TC128])
# (132, 100) transposed: the staged column path with a partial row tile and a ragged last block
@pytest.mark.parametrize("shape", [(128, 256), (256, 1024), (130, 100), (132, 100), (7, 33), (1, 32), (264, 2056)])
@pytest.mark.parametrize("transposed", [False, True])
def test_quantize_bit_exact(fmt, scale_layout, shape, transposed):
    x = adversarial(*shape, seed=shape[0] * 131 + shape[1])
    p, s = gpu_quantize(fmt, x, scale_layout, transposed)
    pw, sw_ = O.mx_quantize(fmt, x, scale_layout=scale_layout)
    np.testing.assert_array_equal(s, sw_)
    np.testing.assert_array_equal(p, pw)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("transposed", [False, True])
def test_quantize_full_size_8192(fmt, transposed):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((8192, 8192)).astype(np.float32)
    p, s = gpu_quantize(fmt, x, N.SW_SCALES_TC128, transposed)
    pw, sw_ = O.mx_quantize(fmt, x, scale_layout=N.SW_SCALES_TC128)
    np.testing.assert_array_equal(s, sw_)
    np.testing.assert_array_equal(p, pw)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("scale_layout", [N.SW_SCALES_ROWMAJOR, N.SW_SCALES_TC128])
def test_dequantize_bit_exact(fmt, scale_layout):
    rows, cols = 256, 320
    rng = np.random.default_rng(9)
    row_bytes = cols if fmt == O.E4M3 else cols // 2
    payload = rng.integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
    kblocks = cols // 32
    if scale_layout == N.SW_SCALES_TC128:
        scales = rng.integers(0, 256, size=O.scale_bytes_tc128(rows, kblocks), dtype=np.uint8)
        lds = 0
    else:
        scales = rng.integers(0, 256, size=(rows, kblocks), dtype=np.uint8)
        lds = kblocks
    want = O.mx_dequantize(fmt, payload, scales, rows, cols, scale_layout=scale_layout)
    dp, ds = to_device(payload), to_device(scales)
    out = empty(rows * cols * 4)
    from strideweave_b200 import kernels

    kernels.mx_dequantize(fmt, dp.ptr, row_bytes, ds.ptr, rows, cols, out.ptr, cols, scale_layout=scale_layout,
                          ld_scales=lds)
    got = to_host(out, (rows, cols), np.float32)
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_round_trip_is_idempotent(fmt):
    # quantise(dequantise(quantise(x))) == quantise(x): the dequantised values
    # are exactly representable, so a second pass changes nothing.
    x = adversarial(256, 512, seed=4)
    x[~np.isfinite(x)] = 1.0
    p, s = gpu_quantize(fmt, x, N.SW_SCALES_TC128)
    d = O.mx_dequantize(fmt, p, s, 256, 512, scale_layout=N.SW_SCALES_TC128)
    p2, s2 = gpu_quantize(fmt, d, N.SW_SCALES_TC128)
    np.testing.assert_array_equal(p2, p)
    np.testing.assert_array_equal(s2, s)
