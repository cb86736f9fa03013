"""MX quantisation of hierarchical and swizzled Float32 views, and contractions
of ragged shapes, against the CPU oracle and the reference CPU carrier.

The reference contracts any extents and any hierarchical strides
(src/strideweave/carriers/cpu/native/ops/matmul.cpp:45-113,
src/strideweave/core/layout.py:1520-1546) and places tensors through a
Swizzle's flat-index map (src/strideweave/core/swizzle.py:107-117).  Here:

* ``sw_mx_quantize_view`` quantises a tiled or swizzled view where it lies;
  its planes must equal the oracle's quantisation of the view's logical
  values bit for bit;
* ``sw_mx_gemm`` takes any M and N and any K that is a whole number of
  32-element MX blocks (the last tile row / column is clipped, the K tail is
  zero-filled); results stay within the path's 2e-3 relative Frobenius
  tolerance of the reference contraction on the dequantised operands (the
  tensor cores' products are exact, so they measure ~1e-7).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, Layout, Shape, Stride, Swizzle, SwizzleStage, Tensor  # noqa: E402

from oracle import oracle as O  # noqa: E402
from strideweave_b200 import _native as N  # noqa: E402
from tests.gpu_util import empty, rel_frobenius, to_device, to_host  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3
EXACT = 1e-5  # exact products, Float32 accumulation: far inside TOL
FORMATS = [("MXFP8_E4M3", O.E4M3), ("MXFP4", O.E2M1)]


def quantize_rows(fmt, a):
    """Device planes of a [rows, K] row-major operand (atom-placed scales)."""
    from strideweave_b200 import kernels

    rows, K = a.shape
    rb = K if fmt == O.E4M3 else K // 2
    pay, sc = empty(rows * rb), empty(O.scale_bytes_tc128(rows, K // 32))
    x = to_device(a)
    kernels.mx_quantize(fmt, x.ptr, rows, K, K, 1, pay.ptr, rb, sc.ptr)
    return pay, sc, rb


def dequantized(fmt, a):
    rows, K = a.shape
    p, s = O.mx_quantize(fmt, a, scale_layout=1)
    return O.mx_dequantize(fmt, p, s, rows, K, scale_layout=1).astype(np.float64)


RAGGED = [
    (200, 1000, 480),   # every extent ragged; N's last 256-wide tile 232 columns
    (129, 257, 32),     # one row / column past a tile; a single MX block of K
    (100, 300, 96),     # N % 256 = 44: 128-wide tiles, the last one 44 columns
    (1, 1, 64),
    (384, 640, 352),    # whole tiles; MXFP4's K tail takes one scale atom of the last stage
]


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("M,N_,K", RAGGED)
def test_ragged_contraction_matches_the_oracle(fmt, M, N_, K):
    from strideweave_b200 import kernels

    rng = np.random.default_rng(M * 31 + N_ * 7 + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = (rng.standard_normal((N_, K)) * 0.02).astype(np.float32)
    (pa, sa, ra), (pb, sb, rb) = quantize_rows(fmt, a), quantize_rows(fmt, b)
    want = dequantized(fmt, a) @ dequantized(fmt, b).T
    for order in ("rows", "cols"):
        ldc_m, ldc_n = (N_, 1) if order == "rows" else (1, M)
        guard = 64  # elements past the result that must stay untouched
        c = empty(4 * (M * N_ + guard), fill=0xFF)
        kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, M, N_, K, ldc_m=ldc_m, ldc_n=ldc_n)
        N.raise_device_status()
        flat = to_host(c, M * N_ + guard, np.float32)
        assert (flat[M * N_:].view(np.uint32) == 0xFFFFFFFF).all(), "stores past the result"
        got = flat[:M * N_].reshape(M, N_) if order == "rows" else flat[:M * N_].reshape(N_, M).T
        assert rel_frobenius(got, want) <= EXACT
    # bf16 row-major (staged epilogue when N's tiles are 256 wide) and accumulation into C
    c16 = empty(2 * M * N_, fill=0)
    kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c16.ptr, M, N_, K, out_bf16=True)
    N.raise_device_status()
    got16 = (to_host(c16, M * N_, np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(M, N_)
    assert rel_frobenius(got16, want) <= 4e-3  # bf16 rounding of each output
    init = rng.standard_normal((M, N_)).astype(np.float32)
    cacc = to_device(init)
    kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, cacc.ptr, M, N_, K, beta_one=True)
    N.raise_device_status()
    assert rel_frobenius(to_host(cacc, (M, N_), np.float32), want + init) <= EXACT


def logical(flat, layout):
    """Logical [rows, cols] values of a two-mode layout over an unswizzled store."""
    from strideweave_b200.layout_plan import mode_size

    rows, cols = mode_size(layout, 0), mode_size(layout, 1)
    out = np.empty((rows, cols), np.float32)
    for i in range(rows):
        for j in range(cols):
            out[i, j] = flat[layout((i, j))]
    return out


VIEWS = {
    # 128 x 32 tiles, rows of 32 contiguous floats, two tile rows and four tile columns
    "tiled": (Layout(Shape([[128, 2], [32, 4]]), Stride([[32, 128 * 32 * 4], [1, 128 * 32]])), None),
    # the same tiles stored through the config-2(c) swizzle (16-byte chunks XOR row % 8)
    "tiled_swizzled": (Layout(Shape([[128, 2], [32, 4]]), Stride([[32, 128 * 32 * 4], [1, 128 * 32]])),
                       (3, 2, 3)),
    # a swizzle that moves single elements (bits 1..2): the element-wise run walk
    "tiled_swizzled_fine": (Layout(Shape([[128, 2], [32, 4]]), Stride([[32, 128 * 32 * 4], [1, 128 * 32]])),
                            (2, 1, 4)),
    # blocks along a hierarchical, strided mode (a transposed tiled store)
    "transposed_tiled": (Layout(Shape([[32, 4], [128, 2]]), Stride([[1, 128 * 32], [32, 128 * 32 * 4]])), None),
    # runs of 16 columns: every block spans two runs (the per-element walk)
    "short_runs": (Layout(Shape([128, [16, 8]]), Stride([16, [1, 2048]])), None),
    "short_runs_swizzled": (Layout(Shape([128, [16, 8]]), Stride([16, [1, 2048]])), (2, 4, 3)),
    # the swizzled tiles again with an all-zero block, NaN and infinities
    "tiled_swizzled_special": (Layout(Shape([[128, 2], [32, 4]]), Stride([[32, 128 * 32 * 4], [1, 128 * 32]])),
                               (3, 2, 3)),
}


@pytest.mark.parametrize("fmt,code", FORMATS)
@pytest.mark.parametrize("view", list(VIEWS))
def test_view_quantiser_equals_the_oracle_on_logical_values(fmt, code, view):
    from strideweave_b200 import CUDA, mx

    layout, stage = VIEWS[view]
    size = layout.cosize
    flat = np.random.default_rng(len(view)).standard_normal(size).astype(np.float32)
    flat[::97] *= 300.0  # blocks with large spreads (saturation, tiny elements)
    if view.endswith("special"):
        flat[0:32] = 0.0  # logical row 0, block 0
        flat[32:64] = -0.0
        flat[100], flat[5000], flat[9000] = np.nan, np.inf, -np.inf
    swz = Swizzle(Shape(size), SwizzleStage(bits=stage[0], base=stage[1], shift=stage[2])) if stage else None
    t = Tensor(CUDA.from_numpy(flat, swizzle=swz), 0, layout)
    q = mx.quantize(t, fmt)
    vals = logical(flat, layout)
    rows, K = vals.shape
    scale_layout = 1 if rows % 128 == 0 and (K // 32) % 4 == 0 else 0
    pw, sw_ = O.mx_quantize(code, vals, scale_layout=scale_layout)
    rep = q._representation
    np.testing.assert_array_equal(rep.subtensors[0].carrier.raw_numpy(), pw.ravel())
    np.testing.assert_array_equal(rep.subtensors[1].carrier.raw_numpy(), sw_.ravel())


@pytest.mark.parametrize("fmt,code", FORMATS)
def test_view_quantiser_on_the_config2_layout_at_full_size(fmt, code):
    # X[8192 x 4096] in 128 x 32 tiles through the 3-bit swizzle, quantised
    # along mode 1 where it lies: equal to the strided kernel on the logical
    # row-major values, byte for byte
    from strideweave_b200 import kernels

    R, C = 8192, 4096
    x = np.random.default_rng(8).standard_normal((R, C)).astype(np.float32)
    t = x.reshape(64, 128, 128, 32).transpose(0, 2, 1, 3)
    flat = np.ascontiguousarray(t).ravel()
    f = np.arange(flat.size, dtype=np.int64)
    store = np.empty_like(flat)
    store[f ^ (((f >> 5) & 7) << 2)] = flat
    rb = C if code == O.E4M3 else C // 2
    outs = []
    for src, plan in ((store, "view"), (x.ravel(), "rows")):
        d = to_device(src)
        pay, sc = empty(R * rb), empty(O.scale_bytes_tc128(R, C // 32))
        if plan == "view":
            kernels.mx_quantize_view(code, d.ptr, src.size, 0, [(128, 32), (64, 128 * 32 * 128)],
                                     [(32, 1), (128, 128 * 32)], pay.ptr, rb, sc.ptr, swizzle=[(3, 2, 3)])
        else:
            kernels.mx_quantize(code, d.ptr, R, C, C, 1, pay.ptr, rb, sc.ptr)
        N.raise_device_status()
        outs.append((to_host(pay, R * rb, np.uint8), to_host(sc, O.scale_bytes_tc128(R, C // 32), np.uint8)))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("fmt,code", FORMATS)
@pytest.mark.parametrize("order", ["rows", "cols"])
def test_view_quantiser_on_plain_strided_matrices(fmt, code, order):
    # one leaf per mode, no swizzle: the view entry hands the matrix to the
    # dense kernels (the row walk, or the column tiles for a column-major
    # source at an offset); planes equal the oracle's on the logical values
    from strideweave_b200 import kernels

    R, C, off = 256, 512, 64
    store = np.random.default_rng(17).standard_normal(off + R * C).astype(np.float32)
    if order == "rows":
        rows, cols = [(R, C)], [(C, 1)]
        vals = store[off:].reshape(R, C)
    else:
        rows, cols = [(R, 1)], [(C, R)]
        vals = store[off:].reshape(C, R).T
    rb = C if code == O.E4M3 else C // 2
    d = to_device(store)
    pay, sc = empty(R * rb), empty(O.scale_bytes_tc128(R, C // 32))
    kernels.mx_quantize_view(code, d.ptr, store.size, off, rows, cols, pay.ptr, rb, sc.ptr)
    N.raise_device_status()
    pw, sw_ = O.mx_quantize(code, np.ascontiguousarray(vals), scale_layout=1)
    np.testing.assert_array_equal(to_host(pay, R * rb, np.uint8), pw.ravel())
    np.testing.assert_array_equal(to_host(sc, O.scale_bytes_tc128(R, C // 32), np.uint8), sw_.ravel())


def test_view_quantiser_refuses_views_outside_the_carrier():
    from strideweave_b200 import kernels

    d = to_device(np.zeros(1024, np.float32))
    pay, sc = empty(64 * 32), empty(64)
    with pytest.raises(ValueError, match="outside carrier"):
        kernels.mx_quantize_view(O.E4M3, d.ptr, 1024, 0, [(64, 32)], [(32, 1)], pay.ptr, 32, sc.ptr,
                                 scale_layout=0, ld_scales=1)
    with pytest.raises(ValueError, match="swizzle may address past"):
        kernels.mx_quantize_view(O.E4M3, d.ptr, 1000, 0, [(31, 32)], [(32, 1)], pay.ptr, 32, sc.ptr,
                                 swizzle=[(3, 4, 3)], scale_layout=0, ld_scales=1)


def cpu_tensor(flat, layout):
    flat = np.ascontiguousarray(flat, dtype=np.float32)
    carrier = CPU(flat.size)
    np.ctypeslib.as_array((ctypes.c_float * flat.size).from_address(carrier.pointer()))[:] = flat
    return Tensor(carrier, 0, layout)


@pytest.mark.parametrize("fmt,code", FORMATS)
def test_ragged_mx_matmul_through_the_carrier(fmt, code):
    # 200 x 480 and 1000 x 480 MX tensors keep row-major scale planes (not whole
    # atoms); the contraction rewrites them into the atom placement and matches
    # the reference CPU carrier's matmul on the dequantised operands
    from strideweave_b200 import BFloat16, CUDA, mx

    M, N_, K = 200, 1000, 480
    rng = np.random.default_rng(30)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N_, K)).astype(np.float32)
    qa = mx.quantize(Tensor(CUDA.from_numpy(a.ravel()), 0, Layout(Shape([M, K]), Stride([K, 1]))), fmt)
    qb = mx.quantize(Tensor(CUDA.from_numpy(b.ravel()), 0, Layout(Shape([N_, K]), Stride([K, 1]))), fmt)
    assert qa._representation.subtensors[1].layout == Layout(Shape([M, K // 32]), Stride([K // 32, 1]))
    c = mx.matmul(qa, qb)
    assert c.layout == Layout(Shape([M, N_]), Stride([1, M]))
    da, db = dequantized(code, a).astype(np.float32), dequantized(code, b).astype(np.float32)
    want = sw.matmul(cpu_tensor(da.ravel(), Layout(Shape([M, K]), Stride([K, 1]))),
                     cpu_tensor(db.ravel(), Layout(Shape([N_, K]), Stride([K, 1]))))
    want_np = np.ctypeslib.as_array((ctypes.c_float * (M * N_)).from_address(want.carrier.pointer()))
    want_np = want_np.reshape(N_, M).T
    assert rel_frobenius(c.carrier.to_numpy().reshape(N_, M).T, want_np) <= EXACT
    c16 = mx.matmul(qa, qb, out_dtype=BFloat16)
    assert rel_frobenius(c16.carrier.to_numpy().reshape(N_, M).T, want_np) <= TOL


@pytest.mark.parametrize("fmt,code", FORMATS)
def test_tiled_swizzled_operand_contracts_like_its_logical_values(fmt, code):
    # an MX operand quantised from a tiled, swizzled Float32 tensor contracts
    # exactly like the same values quantised from a row-major tensor
    from strideweave_b200 import CUDA, mx

    layout, stage = VIEWS["tiled_swizzled"]
    size = layout.cosize
    flat = np.random.default_rng(31).standard_normal(size).astype(np.float32)
    swz = Swizzle(Shape(size), SwizzleStage(bits=stage[0], base=stage[1], shift=stage[2]))
    qa = mx.quantize(Tensor(CUDA.from_numpy(flat, swizzle=swz), 0, layout), fmt)
    vals = logical(flat, layout)
    rows, K = vals.shape
    b = np.random.default_rng(32).standard_normal((192, K)).astype(np.float32)
    qb = mx.quantize(Tensor(CUDA.from_numpy(b.ravel()), 0, Layout(Shape([192, K]), Stride([K, 1]))), fmt)
    got = mx.matmul(qa, qb).carrier.to_numpy().reshape(192, rows).T
    want = dequantized(code, vals) @ dequantized(code, b).T
    assert rel_frobenius(got, want) <= EXACT


@pytest.mark.parametrize("fmt,code", FORMATS)
def test_mx_linear_on_extents_of_whole_blocks(fmt, code):
    # batch 96, 160 -> 224: multiples of 32 but of no tile
    from strideweave_b200 import CUDA, mx

    B, IN, OUT = 96, 160, 224
    rng = np.random.default_rng(33)
    x = rng.standard_normal((B, IN)).astype(np.float32)
    w = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    g = rng.standard_normal((B, OUT)).astype(np.float32)
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, IN]), Stride([IN, 1])))
    wt = Tensor(CUDA.from_numpy(w.ravel()), 0, Layout(Shape([OUT, IN]), Stride([IN, 1])))
    y = mx.linear(xt, wt, fmt=fmt)
    y.backward(Tensor(CUDA.from_numpy(g.T.ravel().copy()), 0, y.layout))
    want_y = dequantized(code, x) @ dequantized(code, w).T
    want_dx = dequantized(code, g) @ dequantized(code, np.ascontiguousarray(w.T)).T
    want_dw = dequantized(code, np.ascontiguousarray(g.T)) @ dequantized(code, np.ascontiguousarray(x.T)).T
    assert rel_frobenius(y.carrier.to_numpy().reshape(OUT, B).T, want_y) <= EXACT
    assert rel_frobenius(xt.grad.carrier.to_numpy().reshape(B, IN), want_dx) <= EXACT
    assert rel_frobenius(wt.grad.carrier.to_numpy().reshape(OUT, IN), want_dw) <= EXACT


@pytest.mark.parametrize("ndest,rows_per_dest", [(1, 128), (3, 256)])
@pytest.mark.parametrize("N_,pad", [(1024, 0), (200, 4), (128, 0), (100, 8)])
def test_routed_contraction_lands_each_row_block_at_its_destination(ndest, rows_per_dest, N_, pad):
    """sw_mx_gemm_routed (the contraction half of the peer K-split), here with
    every destination on this GPU: row block q equals rows
    [q rows_per_dest, (q + 1) rows_per_dest) of the plain contraction bit for
    bit, with pitch N + pad, and nothing past a block is written.  N = 1024
    and 200 take the staged epilogue (whole 128-byte row segments), 128 and
    100 the register one."""
    from strideweave_b200 import kernels

    fmt, K = O.E4M3, 256
    M = ndest * rows_per_dest
    rng = np.random.default_rng(N_ + ndest)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = (rng.standard_normal((N_, K)) * 0.02).astype(np.float32)
    (pa, sa, ra), (pb, sb, rb) = quantize_rows(fmt, a), quantize_rows(fmt, b)
    c = empty(4 * M * N_)
    kernels.mx_gemm(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, M, N_, K)
    want = to_host(c, (M, N_), np.float32)
    ldc, guard = N_ + pad, 64
    blocks = [empty(4 * (rows_per_dest * ldc + guard), fill=0xFF) for _ in range(ndest)]
    # the walk starts at the last block (the rotation a K-split rank uses)
    kernels.mx_gemm_routed(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, [d.ptr for d in blocks], rows_per_dest,
                           ldc, M, N_, K, first=ndest - 1)
    N.raise_device_status()
    for q, d in enumerate(blocks):
        flat = to_host(d, rows_per_dest * ldc + guard, np.float32)
        assert (flat[rows_per_dest * ldc:].view(np.uint32) == 0xFFFFFFFF).all(), "stores past the block"
        got = flat[:rows_per_dest * ldc].reshape(rows_per_dest, ldc)
        np.testing.assert_array_equal(got[:, :N_], want[q * rows_per_dest:(q + 1) * rows_per_dest])
        assert (got[:, N_:].view(np.uint32) == 0xFFFFFFFF).all(), "stores into the pitch padding"
