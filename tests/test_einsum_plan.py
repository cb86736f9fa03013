"""Host-side resolution of the batched-einsum fast path (no GPU): which
descriptions it takes, and the strides and extents it hands the batched
contraction; everything else must fall back to the reference lowering."""

from __future__ import annotations

import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, DType, Layout, Shape, Stride, Tensor  # noqa: E402


def t(shape, stride):
    n = 1 + sum((e - 1) * s for e, s in zip(shape, stride))
    return Tensor(CPU(n, dtype=DType.Float32), 0, Layout(Shape(list(shape)), Stride(list(stride))))


def test_plan_of_a_batched_contraction():
    from strideweave_b200.einsum import _plan

    B, I, J, K = 2, 3, 4, 5
    lhs = t((B, I, K), (I * K, K, 1))
    rhs = t((B, J, K), (1, B * K, B))  # any single-stride modes
    p = _plan(lhs, rhs, "b i k, b j k -> b i j")
    assert (p["batch"], p["M"], p["N"], p["K"]) == (B, I, J, K)
    assert (p["sab"], p["sam"], p["sak"]) == (I * K, K, 1)
    assert (p["sbb"], p["sbn"], p["sbk"]) == (1, B * K, B)
    # the reference's result layout: canonical column-major over the output modes
    assert (p["scb"], p["scm"], p["scn"]) == (1, B, B * I)
    assert p["layout"] == Layout(Shape([B, I, J]), Stride([1, B, B * I]))
    q = _plan(lhs, rhs, "b i k, b j k -> j b i")
    assert (q["scn"], q["scb"], q["scm"]) == (1, J, J * B)


def test_plan_falls_back_outside_its_shape():
    from strideweave_b200.einsum import _plan

    lhs = t((2, 3, 5), (15, 5, 1))
    rhs = t((2, 4, 5), (20, 5, 1))
    assert _plan(lhs, rhs, "b i k, b j k -> b i j k") is None      # nothing contracted
    assert _plan(lhs, rhs, "b i k, c j k -> b c i j") is None      # no batch symbol
    assert _plan(lhs, rhs, "(b i) k, b j k -> b i j") is None      # grouped modes
    hier = Tensor(CPU(64, dtype=DType.Float32), 0, Layout(Shape([2, 3, [5, 1]]), Stride([15, 5, [1, 7]])))
    assert _plan(hier, rhs, "b i k, b j k -> b i j") is not None  # unit leaf ignored
    two = Tensor(CPU(200, dtype=DType.Float32), 0, Layout(Shape([2, 3, [2, 3]]), Stride([30, 10, [1, 5]])))
    rhs6 = t((2, 4, 6), (24, 6, 1))
    assert _plan(two, rhs6, "b i k, b j k -> b i j") is None       # k is two strides


def test_mx_format_requests_never_fall_back_silently():
    # einsum(..., fmt=...) asks for the block-scaled tensor cores: tensors that
    # cannot take that path (here host tensors) and unknown formats raise, and
    # nothing is computed by the reference lowering in their place
    from strideweave_b200.einsum import einsum

    lhs = t((2, 128, 256), (128 * 256, 256, 1))
    rhs = t((2, 128, 256), (128 * 256, 256, 1))
    with pytest.raises(NotImplementedError, match="CUDA tensors"):
        einsum(lhs, rhs, "b i k, b j k -> b i j", fmt="MXFP8_E4M3")
    with pytest.raises(NotImplementedError, match="MXFP6"):
        einsum(lhs, rhs, "b i k, b j k -> b i j", fmt="MXFP6")
    assert einsum(lhs, rhs, "b i k, b j k -> b i j").layout.shape == Shape([2, 128, 128])  # no fmt: reference
