"""The reference's own tensor-level cases for the operations this carrier
executes, run with CUDA-carrier tensors: the values, result layouts, gradient
placements, autograd nodes and errors its tests pin for the Generic and CPU
carriers (tests/test_tensor.py:778-885 and 1811-1875, extrema semantics from
tests/test_dtype_conformance.py:470-510)."""

from __future__ import annotations

import math
import struct

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import CPU, Layout, Shape, Stride, Tensor  # noqa: E402

pytestmark = pytest.mark.gpu


def cuda(values, layout):
    from strideweave_b200 import CUDA

    return Tensor(CUDA.from_numpy(np.asarray(values, dtype=np.float32)), 0, layout)


def values_of(t):
    """Logical values in the layout's colexicographic order (first mode fastest)."""
    return [t[i] for i in range(t.size())]


def bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def test_reduce_sum_sums_the_second_mode():
    t = cuda([1, 2, 3, 4, 5, 6], Layout(Shape([2, 3]), Stride([1, 2])))
    r = sw.reduce_sum(t, "a b -> a")
    assert r.layout == Layout(Shape(2), Stride(1))
    assert values_of(r) == [9, 12]
    assert type(r.autograd_ctx).__name__ == "CudaReduceSum"


def test_reduce_sum_keeps_a_hierarchical_first_mode():
    t = cuda(range(1, 13), Layout(Shape([[2, 2], 3]), Stride([[1, 2], 4])))
    r = sw.reduce_sum(t, "(a b) c -> (a b)")
    assert r.layout == Layout(Shape([[2, 2]]), Stride([[1, 2]]))
    assert values_of(r) == [15, 18, 21, 24]


def test_reduce_sum_backward_copies_the_gradient_over_the_second_mode():
    from strideweave_b200 import CUDA

    t = cuda([1, 2, 3, 4, 5, 6], Layout(Shape([2, 3]), Stride([1, 2])))
    r = sw.reduce_sum(t, "a b -> a")
    r.backward(cuda([10, 20], r.layout))
    assert values_of(t.grad) == [10, 20, 10, 20, 10, 20]
    assert type(t.grad.carrier) is CUDA


def test_reduce_sum_primitive_rejects_a_one_mode_tensor():
    one = cuda([1, 2], Layout(Shape(2), Stride(1)))
    with pytest.raises(ValueError, match="tensor must have a two-mode layout"):
        one.carrier.dispatch_op("reduce_sum").forward(one)


def _nk_mk():
    a = cuda([1, 2, 3, 4, 5, 6], Layout(Shape([2, 3]), Stride([1, 2])))
    b = cuda([1, 0, 0, 1, 0, 1, 0, 1, 0, 0, 1, 1], Layout(Shape([4, 3]), Stride([1, 4])))
    return a, b


def test_matmul_contracts_nk_by_mk_to_nm():
    a, b = _nk_mk()
    r = a @ b
    assert r.layout == Layout(Shape([2, 4]), Stride([1, 2]))
    assert values_of(r) == [1, 2, 3, 4, 5, 6, 9, 12]
    assert type(r.autograd_ctx).__name__ == "CudaMatmul"


def test_matmul_keeps_hierarchical_row_modes():
    a = cuda(range(1, 13), Layout(Shape([[2, 2], 3]), Stride([[1, 2], 4])))
    b = cuda([1, 0, 0, 1, 0, 0], Layout(Shape([[2, 1], 3]), Stride([[1, 2], 2])))
    r = sw.matmul(a, b)
    assert r.layout == Layout(Shape([[2, 2], [2, 1]]), Stride([[1, 2], [4, 8]]))
    assert values_of(r) == [1, 2, 3, 4, 5, 6, 7, 8]


def test_matmul_backward_computes_both_input_gradients():
    from strideweave_b200 import CUDA

    a, b = _nk_mk()
    r = a @ b
    r.backward(cuda([1] * 8, r.layout))
    assert values_of(a.grad) == [2, 2, 2, 2, 2, 2]
    assert values_of(b.grad) == [3, 3, 3, 3, 7, 7, 7, 7, 11, 11, 11, 11]
    assert type(a.grad.carrier) is CUDA and type(b.grad.carrier) is CUDA


def test_matmul_rejects_bad_shapes_and_a_foreign_carrier():
    a = cuda([1, 2, 3, 4], Layout(Shape([2, 2]), Stride([1, 2])))
    bad_k = cuda([1, 2, 3], Layout(Shape([1, 3]), Stride([1, 1])))
    one = cuda([1, 2], Layout(Shape(2), Stride(1)))
    cpu = Tensor(CPU(4), 0, a.layout)
    with pytest.raises(ValueError, match="Matmul inner dimensions must match"):
        _ = a @ bad_k
    with pytest.raises(ValueError, match="rhs must have a two-mode layout"):
        _ = a @ one
    with pytest.raises(TypeError):
        _ = cpu @ a


def test_matmul_with_a_broadcast_operand_matches_torch():
    torch = pytest.importorskip("torch")
    lhs_layout = Layout(Shape([2, 3]), Stride([1, 2]))
    lhs = cuda([1.0, 4.0, 2.0, 5.0, 3.0, 6.0], lhs_layout)
    src_layout = Layout(Shape([1, 3]), Stride([1, 1]))
    src = cuda([7.0, 8.0, 9.0], src_layout)
    rhs = sw.broadcast_to(src, Shape([2, 3]))
    r = sw.matmul(lhs, rhs)
    r.backward(cuda([1.0, 3.0, 2.0, 4.0], r.layout))

    t_lhs = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], requires_grad=True)
    t_src = torch.tensor([[7.0, 8.0, 9.0]], requires_grad=True)
    t_r = t_lhs @ t_src.expand(2, 3).T
    t_r.backward(torch.tensor([[1.0, 2.0], [3.0, 4.0]]))
    assert [r[i, j] for i in range(2) for j in range(2)] == pytest.approx(t_r.reshape(-1).tolist())
    assert src.grad.layout == src_layout
    assert values_of(src.grad) == pytest.approx(t_src.grad.reshape(-1).tolist())


def test_backward_refuses_an_input_modified_in_place_after_forward():
    layout = Layout(Shape([2, 2]), Stride([1, 2]))
    t = cuda([1, 2, 3, 4], layout)
    r = sw.elementwise_mul(t, t)
    t[0, 0] = 10
    with pytest.raises(RuntimeError, match="modified in-place"):
        r.backward(cuda([1, 1, 1, 1], layout))


NAN_A, NAN_B = from_bits(0x7FC00011), from_bits(0x7FC00022)


@pytest.mark.parametrize(
    "values,expected_bits,expected_gradient",
    [
        ((NAN_A, 5.0, NAN_B), 0x7FC00011, (math.nan,) * 3),
        ((-0.0, 0.0), 0x00000000, (2.0, 2.0)),
        ((3.0, 3.0, -1.0), 0x40400000, (2.0, 2.0, 0.0)),
        ((math.inf, -math.inf, 5.0), 0x7F800000, (4.0, 0.0, 0.0)),
    ],
)
def test_reduce_max_payload_ties_infinity_signed_zero_and_vjp(values, expected_bits, expected_gradient):
    t = cuda(values, Layout(Shape([1, len(values)]), Stride([1, 1])))
    r = sw.reduce_max(t, "a b -> a")
    assert bits(r[0]) == expected_bits
    r.backward(cuda([4.0], r.layout))
    got = values_of(t.grad)
    for g, w in zip(got, expected_gradient):
        assert (math.isnan(g) and math.isnan(w)) or g == w
