"""The CUDA carrier behind the reference's own API.

Tensors on ``strideweave_b200.CUDA`` go through ``sw.reduce_sum`` /
``sw.reduce_max`` / ``sw.argmax`` / ``sw.matmul`` / ``Tensor.backward`` /
DLPack exactly as CPU tensors do; every result is compared with the
reference CPU carrier (``strideweave.CPU``) on the same values, the way the
reference's own tests (tests/test_cpu.py:961-1044) state them.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, Layout, Shape, Stride, Swizzle, SwizzleStage, Tensor  # noqa: E402

from oracle import oracle as O  # noqa: E402
from tests.gpu_util import rel_frobenius  # noqa: E402

pytestmark = pytest.mark.gpu

SUM_TOL = 2e-3


@pytest.fixture(scope="module")
def CUDA():
    from strideweave_b200 import CUDA as cls

    return cls


def cpu_tensor(flat: np.ndarray, layout: Layout) -> Tensor:
    """A reference CPU-carrier tensor holding `flat` (copied into the
    carrier's own storage)."""
    flat = np.ascontiguousarray(flat, dtype=np.float32)
    carrier = CPU(flat.size)
    dst = np.ctypeslib.as_array((ctypes.c_float * flat.size).from_address(carrier.pointer()))
    dst[:] = flat
    return Tensor(carrier, 0, layout)


def values(t: Tensor) -> np.ndarray:
    return np.array([t[i] for i in range(t.size())])


def cuda_values(t: Tensor) -> np.ndarray:
    """Logical values of a CUDA tensor with a canonical (compact) layout."""
    raw = t.carrier.to_numpy()
    return np.array([raw[t.offset + t.layout.index(i)] for i in range(t.size())])


LAYOUTS = {
    name: (layout, layout.cosize)
    for name, layout in {
        "rowmajor": Layout(Shape([64, 96]), Stride([96, 1])),
        "colmajor": Layout(Shape([64, 96]), Stride([1, 64])),
        "hierarchical": Layout(Shape([[2, 2], [3, 2]]), Stride([[1, 5], [20, 7]])),
        "tiled": Layout(Shape([[16, 4], [32, 3]]), Stride([[32, 16 * 32 * 3], [1, 16 * 32]])),
    }.items()
}


@pytest.mark.parametrize("name", list(LAYOUTS))
@pytest.mark.parametrize("op", ["reduce_sum", "reduce_max", "argmax"])
def test_reductions_dispatch_to_the_gpu_and_match_the_cpu_carrier(CUDA, name, op):
    layout, cosize = LAYOUTS[name]
    rng = np.random.default_rng(hash(name) % 2**32)
    flat = rng.uniform(-1, 1, size=cosize).astype(np.float32)
    flat[3] = -0.0
    fn = getattr(sw, op)
    want = fn(cpu_tensor(flat, layout), "a b -> a")
    got = fn(Tensor(CUDA.from_numpy(flat), 0, layout), "a b -> a")
    assert type(got.carrier) is CUDA
    assert got.layout == want.layout
    assert got.dtype() is want.dtype()
    g, w = cuda_values(got), values(want)
    if op == "reduce_sum":
        assert rel_frobenius(g, w) <= SUM_TOL
    else:
        np.testing.assert_array_equal(np.asarray(g, dtype=np.float64), np.asarray(w, dtype=np.float64))


@pytest.mark.parametrize("op", ["reduce_sum", "reduce_max", "argmax"])
def test_swizzled_carrier_matches_the_cpu_carrier_on_logical_values(CUDA, op):
    # the CUDA carrier stores flat index f at swizzle(f); the reference reduces
    # the same logical values from an unswizzled CPU carrier
    layout = Layout(Shape([[16, 4], [32, 4]]), Stride([[32, 16 * 32 * 4], [1, 16 * 32]]))
    size = 64 * 128
    swz = Swizzle(Shape(size), SwizzleStage(bits=3, base=2, shift=3))
    flat = np.random.default_rng(4).uniform(-1, 1, size=size).astype(np.float32)
    fn = getattr(sw, op)
    want = values(fn(cpu_tensor(flat, layout), "a b -> a"))
    got = fn(Tensor(CUDA.from_numpy(flat, swizzle=swz), 0, layout), "a b -> a")
    g = cuda_values(got)
    if op == "reduce_sum":
        assert rel_frobenius(g, want) <= SUM_TOL
    else:
        np.testing.assert_array_equal(g, want)
    # the storage really is permuted
    t = CUDA.from_numpy(flat, swizzle=swz)
    assert t[40] == flat[40] and not np.array_equal(t.raw_numpy().view(np.float32), flat)


def test_reduce_sum_backpropagates_like_the_cpu_carrier(CUDA):
    layout = Layout(Shape([[2, 2], [3, 2]]), Stride([[1, 5], [20, 7]]))
    flat = np.arange(layout.cosize, dtype=np.float32)
    t = Tensor(CUDA.from_numpy(flat), 0, layout)
    result = sw.reduce_sum(t, "a b -> a")
    gradient = Tensor(CUDA.from_numpy(np.array([10.0, 20.0, 30.0, 40.0], np.float32)), 0, result.layout)
    result.backward(gradient)
    assert type(result.autograd_ctx).__name__ == "CudaReduceSum"
    ct = cpu_tensor(flat, layout)
    cr = sw.reduce_sum(ct, "a b -> a")
    cr.backward(cpu_tensor(np.array([10.0, 20.0, 30.0, 40.0]), cr.layout))
    assert t.grad is not None and type(t.grad.carrier) is CUDA
    np.testing.assert_array_equal(cuda_values(t.grad), values(ct.grad))
    np.testing.assert_array_equal(cuda_values(result), values(cr))


def test_reduce_max_backpropagates_with_tie_splitting(CUDA):
    layout = Layout(Shape([3, 4]), Stride([4, 1]))
    flat = np.array([1, 5, 5, 2, -0.0, 0.0, -1, -2, np.nan, 1, 2, 3], dtype=np.float32)
    t = Tensor(CUDA.from_numpy(flat), 0, layout)
    r = sw.reduce_max(t, "a b -> a")
    r.backward(Tensor(CUDA.from_numpy(np.array([2.0, 3.0, 4.0], np.float32)), 0, r.layout))
    ct = cpu_tensor(flat, layout)
    cr = sw.reduce_max(ct, "a b -> a")
    cr.backward(cpu_tensor(np.array([2.0, 3.0, 4.0]), cr.layout))
    np.testing.assert_array_equal(cuda_values(r), values(cr))
    np.testing.assert_array_equal(cuda_values(t.grad), values(ct.grad))


@pytest.mark.parametrize(
    "a_layout,b_layout",
    [
        (Layout(Shape([2, 3]), Stride([1, 2])), Layout(Shape([4, 3]), Stride([1, 4]))),
        (Layout(Shape([2, [2, 2]]), Stride([1, [7, 3]])), Layout(Shape([3, [2, 2]]), Stride([2, [11, 5]]))),
        (Layout(Shape([48, 80]), Stride([80, 1])), Layout(Shape([40, 80]), Stride([1, 40]))),
    ],
)
def test_matmul_forward_and_backward_match_the_cpu_carrier(CUDA, a_layout, b_layout):
    rng = np.random.default_rng(0)
    a_flat = rng.standard_normal(a_layout.cosize).astype(np.float32)
    b_flat = rng.standard_normal(b_layout.cosize).astype(np.float32)
    a = Tensor(CUDA.from_numpy(a_flat), 0, a_layout)
    b = Tensor(CUDA.from_numpy(b_flat), 0, b_layout)
    result = a @ b
    assert type(result.autograd_ctx).__name__ == "CudaMatmul"
    grad = rng.standard_normal(result.layout.cosize).astype(np.float32)
    result.backward(Tensor(CUDA.from_numpy(grad), 0, result.layout))
    ca, cb = cpu_tensor(a_flat, a_layout), cpu_tensor(b_flat, b_layout)
    cres = ca @ cb
    cres.backward(cpu_tensor(grad, cres.layout))
    assert result.layout == cres.layout
    assert rel_frobenius(cuda_values(result), values(cres)) <= 1e-5
    assert a.grad.layout == ca.grad.layout and b.grad.layout == cb.grad.layout
    assert rel_frobenius(cuda_values(a.grad), values(ca.grad)) <= 1e-5
    assert rel_frobenius(cuda_values(b.grad), values(cb.grad)) <= 1e-5


def test_views_and_element_access(CUDA):
    flat = np.arange(12, dtype=np.float32)
    t = Tensor(CUDA.from_numpy(flat), 0, Layout(Shape([3, 4]), Stride([4, 1])))
    p = sw.permute(t, 1, 0)
    assert p.carrier is t.carrier and p[2, 1] == 6.0
    assert t[1, 2] == 6.0
    t.carrier[5] = 50.0
    assert t[1, 1] == 50.0
    c = t.carrier.new_like([1.0, 2.0, 3.0])
    assert type(c) is CUDA and c.size() == 3 and c[2] == 3.0
    z = t.carrier.allocate_like(5, dtype=sw.DType.Int32)
    assert z.dtype() is sw.DType.Int32 and z[4] == 0
    assert t.carrier.supports_storage_dtype(sw.DType.E4M3)


def test_dlpack_export_to_torch(CUDA):
    torch = pytest.importorskip("torch")
    flat = np.arange(24, dtype=np.float32)
    t = Tensor(CUDA.from_numpy(flat), 0, Layout(Shape([4, 6]), Stride([6, 1])))
    tt = torch.from_dlpack(t)
    assert tt.device.type == "cuda" and tt.shape == (4, 6)
    np.testing.assert_array_equal(tt.cpu().numpy(), flat.reshape(4, 6))


# ---- MX tensors -------------------------------------------------------------------


@pytest.mark.parametrize("fmt,code", [("MXFP8_E4M3", O.E4M3), ("MXFP4", O.E2M1)])
def test_mx_quantize_builds_a_validated_two_plane_tensor(CUDA, fmt, code):
    from strideweave_b200 import mx

    rows, K = 256, 512
    x = np.random.default_rng(1).standard_normal((rows, K)).astype(np.float32)
    t = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([rows, K]), Stride([K, 1])))
    q = mx.quantize(t, fmt)
    rep = q._representation
    assert rep.logical_dtype is getattr(sw.DType, fmt)
    assert len(rep.subtensors) == 2 and all(type(s.carrier) is CUDA for s in rep.subtensors)
    pw, sw_ = O.mx_quantize(code, x, scale_layout=1)
    np.testing.assert_array_equal(rep.subtensors[0].carrier.raw_numpy(), pw.ravel())
    np.testing.assert_array_equal(rep.subtensors[1].carrier.raw_numpy(), sw_)
    d = mx.dequantize(q)
    np.testing.assert_array_equal(d.carrier.to_numpy().reshape(rows, K),
                                  O.mx_dequantize(code, pw, sw_, rows, K, scale_layout=1))
    # element access through the representation's placement
    assert q.carrier[5] == pytest.approx(O.decode_elem(code, int(pw.ravel()[5]) if code == 1 else
                                                       int(pw.ravel()[2] >> 4)))
    # layout views keep both planes
    v = sw.permute(q, 1, 0)
    assert len(v._representation.subtensors) == 2


@pytest.mark.parametrize("fmt,code", [("MXFP8_E4M3", O.E4M3), ("MXFP4", O.E2M1)])
def test_mx_matmul_matches_the_cpu_carrier_on_dequantised_operands(CUDA, fmt, code):
    from strideweave_b200 import BFloat16, mx

    M, N_, K = 256, 384, 512
    rng = np.random.default_rng(2)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N_, K)).astype(np.float32)
    qa = mx.quantize(Tensor(CUDA.from_numpy(a.ravel()), 0, Layout(Shape([M, K]), Stride([K, 1]))), fmt)
    qb = mx.quantize(Tensor(CUDA.from_numpy(b.ravel()), 0, Layout(Shape([N_, K]), Stride([K, 1]))), fmt)
    c = mx.matmul(qa, qb)
    assert c.layout == Layout(Shape([M, N_]), Stride([1, M]))  # the reference's canonical result
    da = O.mx_dequantize(code, *O.mx_quantize(code, a, scale_layout=1), M, K, scale_layout=1)
    db = O.mx_dequantize(code, *O.mx_quantize(code, b, scale_layout=1), N_, K, scale_layout=1)
    # the reference CPU carrier's own matmul on the dequantised operands
    want = sw.matmul(cpu_tensor(da.ravel(), Layout(Shape([M, K]), Stride([K, 1]))),
                     cpu_tensor(db.ravel(), Layout(Shape([N_, K]), Stride([K, 1]))))
    want_np = np.ctypeslib.as_array((ctypes.c_float * (M * N_)).from_address(want.carrier.pointer()))
    want_np = want_np.reshape(N_, M).T
    got = c.carrier.to_numpy().reshape(N_, M).T
    assert rel_frobenius(got, want_np) <= 1e-5
    c16 = mx.matmul(qa, qb, out_dtype=BFloat16)
    assert c16.carrier.dtype() is BFloat16
    assert rel_frobenius(c16.carrier.to_numpy().reshape(N_, M).T, want_np) <= SUM_TOL


def test_mx_operands_are_refused_by_ordinary_operations(CUDA):
    from strideweave_b200 import mx

    x = np.ones((128, 128), np.float32)
    q = mx.quantize(Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([128, 128]), Stride([128, 1]))))
    with pytest.raises(Exception):
        sw.reduce_sum(q, "a b -> a")


@pytest.mark.parametrize("fmt,code", [("MXFP8_E4M3", O.E4M3), ("MXFP4", O.E2M1)])
def test_mx_linear_forward_and_backward(CUDA, fmt, code):
    from strideweave_b200 import mx

    B, IN, OUT = 256, 512, 256
    rng = np.random.default_rng(3)
    x = rng.standard_normal((B, IN)).astype(np.float32)
    w = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    g = rng.standard_normal((B, OUT)).astype(np.float32)
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, IN]), Stride([IN, 1])))
    wt = Tensor(CUDA.from_numpy(w.ravel()), 0, Layout(Shape([OUT, IN]), Stride([IN, 1])))
    y = mx.linear(xt, wt, fmt=fmt)
    assert y.layout == Layout(Shape([B, OUT]), Stride([1, B]))
    y.backward(Tensor(CUDA.from_numpy(g.T.ravel().copy()), 0, y.layout))

    def dq(m):  # quantise along mode 1, dequantise
        return O.mx_dequantize(code, *O.mx_quantize(code, m, scale_layout=1), m.shape[0], m.shape[1],
                               scale_layout=1).astype(np.float64)

    want_y = dq(x) @ dq(w).T
    want_dx = dq(g) @ dq(np.ascontiguousarray(w.T)).T
    want_dw = dq(np.ascontiguousarray(g.T)) @ dq(np.ascontiguousarray(x.T)).T
    assert rel_frobenius(y.carrier.to_numpy().reshape(OUT, B).T, want_y) <= 1e-5
    assert xt.grad.layout == xt.layout and wt.grad.layout == wt.layout
    assert rel_frobenius(xt.grad.carrier.to_numpy().reshape(B, IN), want_dx) <= 1e-5
    assert rel_frobenius(wt.grad.carrier.to_numpy().reshape(OUT, IN), want_dw) <= 1e-5
