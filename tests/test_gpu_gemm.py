"""Block-scaled MX contraction on the tensor cores against the CPU oracle.

The oracle is the reference contraction (cpu.matmul restated: binary32
products, Float32 accumulation) applied to the exactly dequantised MX
operands.  The tolerance of the path is 2e-3 relative Frobenius error.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from strideweave_b200 import _native as N
from tests.gpu_util import empty, rel_frobenius, to_device, to_host

pytestmark = pytest.mark.gpu

TOL = 2e-3


def quantize_on_gpu(fmt, store, rows, cols, ld_row, ld_col):
    from strideweave_b200 import kernels

    kblocks = cols // 32
    row_bytes = cols if fmt == O.E4M3 else cols // 2
    dx = to_device(store)
    payload = empty(rows * row_bytes)
    scales = empty(O.scale_bytes_tc128(rows, kblocks))
    kernels.mx_quantize(fmt, dx.ptr, rows, cols, ld_row, ld_col, payload.ptr, row_bytes, scales.ptr)
    return payload, scales, row_bytes


def operands(fmt, M, N_, K, seed=0, b_kn=False, b_sigma=1.0):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K)).astype(np.float32)
    if b_kn:
        # B given as K x N row-major (config 1): quantise its columns along K
        b_kn_arr = (rng.standard_normal((K, N_)) * b_sigma).astype(np.float32)
        b = np.ascontiguousarray(b_kn_arr.T)
        pb, sb, rb = quantize_on_gpu(fmt, b_kn_arr, N_, K, 1, N_)
    else:
        b = (rng.standard_normal((N_, K)) * b_sigma).astype(np.float32)
        pb, sb, rb = quantize_on_gpu(fmt, b, N_, K, K, 1)
    pa, sa, ra = quantize_on_gpu(fmt, a, M, K, K, 1)
    # the oracle's own quantisation must agree with the device's (bit-exact)
    pa_h, sa_h = O.mx_quantize(fmt, a, scale_layout=1)
    pb_h, sb_h = O.mx_quantize(fmt, b, scale_layout=1)
    np.testing.assert_array_equal(to_host(pa, pa_h.shape, np.uint8), pa_h)
    np.testing.assert_array_equal(to_host(sb, sb_h.shape, np.uint8), sb_h)
    da = O.mx_dequantize(fmt, pa_h, sa_h, M, K, scale_layout=1)
    db = O.mx_dequantize(fmt, pb_h, sb_h, N_, K, scale_layout=1)
    return (pa, sa, ra), (pb, sb, rb), da, db


def run_gemm(fmt, A, B, M, N_, K, *, out_bf16=False, col_major=False, c_init=None):
    from strideweave_b200 import kernels

    (pa, sa, ra), (pb, sb, rb) = A, B
    esize = 2 if out_bf16 else 4
    c = empty(M * N_ * esize, fill=0)
    if c_init is not None:
        c.upload(np.ascontiguousarray(c_init))
    ldc_m, ldc_n = (1, M) if col_major else (N_, 1)
    kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, M, N_, K, out_bf16=out_bf16,
                    ldc_m=ldc_m, ldc_n=ldc_n, beta_one=c_init is not None)
    N.raise_device_status()
    if out_bf16:
        raw = to_host(c, M * N_, np.uint16).astype(np.uint32) << 16
        flat = raw.view(np.float32)
    else:
        flat = to_host(c, M * N_, np.float32)
    return flat.reshape(N_, M).T if col_major else flat.reshape(M, N_)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_config1_512x1024x512(fmt):
    # config 1: A[512x1024], B[1024x512] ~ N(0,1), seed 0, quantised along K
    M, K, N_ = 512, 1024, 512
    A, B, da, db = operands(fmt, M, N_, K, seed=0, b_kn=True)
    got = run_gemm(fmt, A, B, M, N_, K)
    want = O.matmul(da, db)
    assert rel_frobenius(got, want) <= TOL
    # the tensor-core path computes exact products: it is far inside the tolerance
    assert rel_frobenius(got, want) <= 1e-5


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_narrow_tile_path_and_layouts(fmt):
    # N = 384 is not a multiple of 256: exercises the 128-wide tile
    M, N_, K = 256, 384, 512
    A, B, da, db = operands(fmt, M, N_, K, seed=3)
    want = O.matmul(da, db)
    assert rel_frobenius(run_gemm(fmt, A, B, M, N_, K), want) <= 1e-5
    assert rel_frobenius(run_gemm(fmt, A, B, M, N_, K, col_major=True), want) <= 1e-5
    got16 = run_gemm(fmt, A, B, M, N_, K, out_bf16=True)
    assert rel_frobenius(got16, want) <= 4e-3  # bf16 rounding of the output
    init = np.random.default_rng(1).standard_normal((M, N_)).astype(np.float32)
    acc = run_gemm(fmt, A, B, M, N_, K, c_init=init)
    assert rel_frobenius(acc, want + init) <= 1e-5


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("col_major", [False, True])
def test_many_tiles_persistent_schedule(fmt, col_major):
    # more tiles than SMs, several K stages per tile, activations N(0,1) and
    # weights N(0, 0.02) as in the large contraction configs; fp32 C in either
    # order goes through the staged epilogue's rotating chunk buffers
    M, N_, K = 2048, 2560, 1024
    A, B, da, db = operands(fmt, M, N_, K, seed=5, b_sigma=0.02)
    got = run_gemm(fmt, A, B, M, N_, K, col_major=col_major)
    want = da.astype(np.float64) @ db.astype(np.float64).T
    assert rel_frobenius(got, want) <= 1e-5


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("col_major", [False, True])
def test_staged_fp32_epilogue_equals_the_direct_stores(fmt, col_major):
    # pitched fp32 C: the staged TMA-store epilogue (no accumulation) against
    # the register-store epilogue (accumulation onto zeros), bit for bit
    from strideweave_b200 import kernels

    M, N_, K = 384, 512, 512
    (pa, sa, ra), (pb, sb, rb), _, _ = operands(fmt, M, N_, K, seed=12)
    ldc_m, ldc_n = (1, M + 32) if col_major else (N_ + 64, 1)
    span = (N_ - 1) * ldc_n + (M - 1) * ldc_m + 1
    outs = []
    for beta_one in (False, True):
        c = empty(4 * span, fill=0)
        kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, M, N_, K, ldc_m=ldc_m, ldc_n=ldc_n,
                        beta_one=beta_one)
        N.raise_device_status()
        outs.append(to_host(c, span, np.float32) + np.float32(0.0))  # +0 folds a -0 sum into +0
    np.testing.assert_array_equal(outs[0], outs[1])
    idx = np.arange(M)[:, None] * ldc_m + np.arange(N_)[None, :] * ldc_n
    untouched = np.ones(span, bool)
    untouched[idx.ravel()] = False
    assert not outs[0][untouched].any()  # the pitch gaps are not written


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_full_size_8192_sampled_rows(fmt):
    M = N_ = K = 8192
    A, B, da, db = operands(fmt, M, N_, K, seed=0, b_sigma=0.02)
    got = run_gemm(fmt, A, B, M, N_, K, out_bf16=(fmt == O.E2M1))
    rows = np.random.default_rng(0).choice(M, size=64, replace=False)
    want = da[rows].astype(np.float64) @ db.astype(np.float64).T
    assert rel_frobenius(got[rows], want) <= (4e-3 if fmt == O.E2M1 else 1e-5)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_staged_bf16_epilogue_rounds_the_fp32_result(fmt):
    # bf16 row-major results go through the shared-memory staged TMA-store
    # epilogue; they must be exactly the fp32 accumulator rounded to nearest even
    torch = pytest.importorskip("torch")
    M, N_, K = 512, 768, 1024
    A, B, _, _ = operands(fmt, M, N_, K, seed=9)
    f32 = run_gemm(fmt, A, B, M, N_, K)
    b16 = run_gemm(fmt, A, B, M, N_, K, out_bf16=True)
    want = torch.from_numpy(f32).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(b16, want)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
def test_cta_cap_changes_the_schedule_not_the_result(fmt):
    # sw_mx_gemm_ex on 7 and on 1 SMs: every tile still computed, bit-identical
    from strideweave_b200 import kernels

    M, N_, K = 512, 768, 512
    (pa, sa, ra), (pb, sb, rb), _, _ = operands(fmt, M, N_, K, seed=21)
    outs = []
    for cap in (0, 7, 1):
        c = empty(4 * M * N_, fill=0)
        kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, M, N_, K, max_ctas=cap)
        N.raise_device_status()
        outs.append(to_host(c, M * N_, np.float32))
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    with pytest.raises(ValueError):
        kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, pa.ptr, M, N_, K, max_ctas=-1)
