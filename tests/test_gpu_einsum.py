"""Batched einsum on the CUDA carrier: the reference's own lowering (union
product through the carrier's elementwise_mul, then reduce_sum) and the
batched-contraction fast path, against numpy and against each other, values,
result layouts and gradients.  Float32 contraction tolerance: 2e-3 relative
Frobenius (the path's stated bound); the two device paths agree far closer."""

from __future__ import annotations

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import Layout, Shape, Stride, Tensor  # noqa: E402

from tests.gpu_util import rel_frobenius  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3


def cuda_tensor(arr, strides=None):
    from strideweave_b200 import CUDA

    arr = np.ascontiguousarray(arr, dtype=np.float32)
    if strides is None:  # row-major element strides
        strides, acc = [], 1
        for n in reversed(arr.shape):
            strides.insert(0, acc)
            acc *= n
    return Tensor(CUDA.from_numpy(arr.ravel()), 0, Layout(Shape(list(arr.shape)), Stride(list(strides))))


def values(t, shape):
    out = np.empty(shape, dtype=np.float32)
    for idx in np.ndindex(*shape):
        out[idx] = t[idx]
    return out


def test_elementwise_mul_broadcasts_and_differentiates():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 4)).astype(np.float32)
    b = rng.standard_normal((3, 1)).astype(np.float32)
    ta, tb = cuda_tensor(a), cuda_tensor(b)
    prod = sw.elementwise_mul(ta, tb)
    assert type(prod.autograd_ctx).__name__ == "CudaElementwiseMul"
    np.testing.assert_array_equal(values(prod, (3, 4)), a * b)
    g = cuda_tensor(np.ones((3, 4), np.float32), strides=[1, 3])
    prod.backward(g)
    np.testing.assert_allclose(values(ta.grad, (3, 4)), np.broadcast_to(b, (3, 4)), rtol=0, atol=0)
    np.testing.assert_allclose(values(tb.grad, (3, 1)), a.sum(axis=1, keepdims=True), rtol=1e-6)


@pytest.mark.parametrize("desc,out_order", [("b i k, b j k -> b i j", "bij"), ("b i k, b j k -> j b i", "jbi")])
def test_reference_lowering_runs_on_the_device(desc, out_order):
    rng = np.random.default_rng(1)
    B, I, J, K = 3, 5, 4, 7
    a = rng.standard_normal((B, I, K)).astype(np.float32)
    b = rng.standard_normal((B, J, K)).astype(np.float32)
    r = sw.einsum(cuda_tensor(a), cuda_tensor(b), desc)  # the reference's union-product lowering
    want = np.einsum(f"bik,bjk->{out_order}", a.astype(np.float64), b.astype(np.float64))
    assert rel_frobenius(values(r, want.shape), want) <= TOL


@pytest.mark.parametrize("desc,out_order", [
    ("b i k, b j k -> b i j", "bij"),
    ("b i k, b j k -> i j b", "ijb"),
    ("i b k, k b j -> b i j", None),
])
def test_fast_path_matches_numpy_and_the_reference_lowering(desc, out_order):
    from strideweave_b200 import einsum

    rng = np.random.default_rng(2)
    B, I, J, K = 4, 33, 17, 65
    if out_order is None:  # lhs (i, b, k), rhs (k, b, j)
        a = rng.standard_normal((I, B, K)).astype(np.float32)
        b = rng.standard_normal((K, B, J)).astype(np.float32)
        want = np.einsum("ibk,kbj->bij", a.astype(np.float64), b.astype(np.float64))
    else:
        a = rng.standard_normal((B, I, K)).astype(np.float32)
        b = rng.standard_normal((B, J, K)).astype(np.float32)
        want = np.einsum(f"bik,bjk->{out_order}", a.astype(np.float64), b.astype(np.float64))
    fast = einsum.einsum(cuda_tensor(a), cuda_tensor(b), desc)
    assert type(fast.autograd_ctx).__name__ == "CudaBatchedContraction"
    ref = sw.einsum(cuda_tensor(a), cuda_tensor(b), desc)
    assert fast.layout == ref.layout
    got = values(fast, want.shape)
    assert rel_frobenius(got, want) <= TOL
    assert rel_frobenius(got, values(ref, want.shape)) <= 1e-5


def test_fast_path_gradients_match_the_reference_lowering():
    from strideweave_b200 import einsum

    rng = np.random.default_rng(3)
    B, I, J, K = 2, 6, 5, 9
    a = rng.standard_normal((B, I, K)).astype(np.float32)
    b = rng.standard_normal((B, J, K)).astype(np.float32)
    g = rng.standard_normal((B, I, J)).astype(np.float32)
    grads = []
    for fn in (einsum.einsum, sw.einsum):
        ta, tb = cuda_tensor(a), cuda_tensor(b)
        r = fn(ta, tb, "b i k, b j k -> b i j")
        gt = Tensor(r.carrier.new_like(np.zeros(r.carrier.size(), np.float32).tolist()), 0, r.layout)
        for idx in np.ndindex(B, I, J):
            gt[idx] = float(g[idx])
        r.backward(gt)
        grads.append((values(ta.grad, (B, I, K)), values(tb.grad, (B, J, K))))
    want_a = np.einsum("bij,bjk->bik", g.astype(np.float64), b.astype(np.float64))
    want_b = np.einsum("bij,bik->bjk", g.astype(np.float64), a.astype(np.float64))
    for (da, db) in grads:
        assert rel_frobenius(da, want_a) <= TOL
        assert rel_frobenius(db, want_b) <= TOL


def col_major_values(t, shape):
    """A result in the canonical column-major layout, read in one copy."""
    flat = t.carrier.to_numpy()
    strides, acc = [], 1
    for n in shape:
        strides.append(acc * 4)
        acc *= n
    return np.lib.stride_tricks.as_strided(flat, shape, strides).copy()


def dequantised(code, x):
    """x [rows, K] through the oracle's MX quantisation (bit-exact with the device's) and back."""
    from oracle import oracle as O

    p, s = O.mx_quantize(code, np.ascontiguousarray(x), scale_layout=1)
    return O.mx_dequantize(code, p, s, x.shape[0], x.shape[1], scale_layout=1).astype(np.float64)


@pytest.mark.parametrize("fmt", ["MXFP8_E4M3", "MXFP4"])
@pytest.mark.parametrize("desc", ["b i k, b j k -> b i j", "i b k, k b j -> i j b"])
def test_mx_fast_path_contracts_the_quantised_inputs(fmt, desc):
    # fmt= quantises both inputs along the contracted symbol and runs one
    # batched block-scaled contraction: the result is the contraction of the
    # dequantised operands, in the plain path's result layout
    from oracle import oracle as O
    from strideweave_b200 import einsum

    code = O.E4M3 if fmt == "MXFP8_E4M3" else O.E2M1
    rng = np.random.default_rng(4)
    B, I, J, K = 3, 256, 128, 512
    if desc.startswith("b"):
        a = rng.standard_normal((B, I, K)).astype(np.float32)
        b = (rng.standard_normal((B, J, K)) * 0.1).astype(np.float32)
        a_bik, b_bjk, out_shape = a, b, (B, I, J)
    else:  # lhs (i, b, k), rhs (k, b, j): strided views, one quantisation per problem
        a = rng.standard_normal((I, B, K)).astype(np.float32)
        b = (rng.standard_normal((K, B, J)) * 0.1).astype(np.float32)
        a_bik, b_bjk, out_shape = a.transpose(1, 0, 2), b.transpose(1, 2, 0), (I, J, B)
    ta, tb = cuda_tensor(a), cuda_tensor(b)
    mx = einsum.einsum(ta, tb, desc, fmt=fmt)
    assert type(mx.autograd_ctx).__name__ == "CudaMxBatchedContraction"
    plain = einsum.einsum(cuda_tensor(a), cuda_tensor(b), desc)
    assert mx.layout == plain.layout
    want = np.stack([dequantised(code, a_bik[q]) @ dequantised(code, b_bjk[q]).T for q in range(B)])
    if out_shape == (I, J, B):
        want = want.transpose(1, 2, 0)
    got = col_major_values(mx, out_shape)
    assert rel_frobenius(got, want) <= TOL


def test_mx_fast_path_gradients_pass_straight_through():
    # the gradients of the MX path are the plain path's (Float32 contractions
    # of the unquantised inputs), bit for bit
    from strideweave_b200 import einsum

    rng = np.random.default_rng(5)
    B, I, J, K = 2, 128, 256, 256
    a = rng.standard_normal((B, I, K)).astype(np.float32)
    b = rng.standard_normal((B, J, K)).astype(np.float32)
    g = rng.standard_normal((J, I, B)).astype(np.float32)  # canonical column-major (b, i, j)
    grads = []
    for kw in ({}, {"fmt": "MXFP8_E4M3"}):
        ta, tb = cuda_tensor(a), cuda_tensor(b)
        r = einsum.einsum(ta, tb, "b i k, b j k -> b i j", **kw)
        from strideweave_b200 import CUDA

        r.backward(Tensor(CUDA.from_numpy(g.ravel()), 0, r.layout))
        grads.append((ta.grad.carrier.to_numpy(), tb.grad.carrier.to_numpy()))
    np.testing.assert_array_equal(grads[0][0], grads[1][0])
    np.testing.assert_array_equal(grads[0][1], grads[1][1])


def test_mx_fast_path_refuses_what_it_cannot_tile():
    from strideweave_b200 import einsum

    a = np.zeros((2, 100, 256), np.float32)
    b = np.zeros((2, 128, 256), np.float32)
    with pytest.raises(NotImplementedError):
        einsum.einsum(cuda_tensor(a), cuda_tensor(b), "b i k, b j k -> b i j", fmt="MXFP8_E4M3")
    with pytest.raises(NotImplementedError):
        einsum.einsum(cuda_tensor(b), cuda_tensor(b), "b i k, b j k -> b i j", fmt="MXFP6")
    with pytest.raises(NotImplementedError):  # no batch symbol: not the batched shape
        einsum.einsum(cuda_tensor(b[0]), cuda_tensor(b[0]), "i k, j k -> i j", fmt="MXFP8_E4M3")
