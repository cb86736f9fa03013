"""The widened accumulator (``accumulator_dtype=DType.Float64``) of
reduce_sum and matmul on the CUDA carrier, following the behaviour the
reference pins for its CPU carrier (tests/test_cpu_plan.py:125-215): the
binary32 terms (2^24, 1, 1, -2^24) cancel to 0 when summed left to right in
binary32 and to exactly 2 in binary64; the widening changes only the
accumulation, is local to one call, and a widened matmul's backward keeps the
forward's accumulator.  Plus the capability declaration: one floating
capability per accumulator, and an undeclared accumulator refused before any
allocation."""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
from strideweave import DType, Layout, Shape, Stride, Tensor  # noqa: E402

CANCELLING = (2.0 ** 24, 1.0, 1.0, -(2.0 ** 24))


def cuda_row(values):
    from strideweave_b200 import CUDA

    arr = np.asarray(values, dtype=np.float32)
    return Tensor(CUDA.from_numpy(arr), 0, Layout(Shape([1, len(values)]), Stride([1, 1])))


def test_capabilities_declare_both_floating_accumulators():
    from strideweave.carriers.operation_capability import capabilities_for_carrier_class

    from strideweave_b200 import CUDA

    for operation in ("reduce_sum", "matmul"):
        accs = {c.accumulator_dtype for c in capabilities_for_carrier_class(CUDA, operation)}
        assert accs == {DType.Float32, DType.Float64}, operation


def test_an_undeclared_accumulator_is_refused():
    from strideweave.carriers.operation_capability import require_capability, supports_operation_plan
    from strideweave.carriers.operation_policy import resolve_operation_plan

    from strideweave_b200 import CUDA
    from strideweave_b200.ops import UnsupportedOperationPlan

    plan = dataclasses.replace(resolve_operation_plan("reduce_sum", DType.Float32), accumulator_dtype=DType.Int32)
    assert not supports_operation_plan(CUDA, plan)
    with pytest.raises(UnsupportedOperationPlan):
        require_capability(CUDA, plan)


@pytest.mark.gpu
def test_widened_reduce_sum_changes_only_the_accumulation():
    t = cuda_row(CANCELLING)
    widened = sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float64)
    explicit = sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float32)
    default = sw.reduce_sum(t, "a b -> a")
    assert [t[0, i] for i in range(4)] == list(CANCELLING)
    assert t.dtype() is widened.dtype() is DType.Float32
    assert widened[0] == 2.0
    # the binary32 summation order is backend-defined (operation_policy.py:109-114);
    # both binary32 requests take the same kernel
    assert explicit[0] == default[0]


@pytest.mark.gpu
def test_widened_matmul_changes_only_the_accumulation():
    lhs, rhs = cuda_row(CANCELLING), cuda_row((1.0, 1.0, 1.0, 1.0))
    widened = sw.matmul(lhs, rhs, accumulator_dtype=DType.Float64)
    default = sw.matmul(lhs, rhs)
    assert widened.dtype() is default.dtype() is DType.Float32
    assert widened[0, 0] == 2.0
    assert default[0, 0] == 0.0  # the products of one output are summed in k order


@pytest.mark.gpu
def test_accumulator_selection_is_local_to_one_call():
    t = cuda_row(CANCELLING)
    assert sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float64)[0] == 2.0
    default = sw.reduce_sum(t, "a b -> a")[0]
    assert sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float64)[0] == 2.0
    assert default == sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float32)[0]


@pytest.mark.gpu
def test_widened_matmul_backward_keeps_the_forward_accumulator():
    from strideweave_b200 import CUDA

    lhs = Tensor(CUDA.from_numpy(np.ones(1, np.float32)), 0, Layout(Shape([1, 1]), Stride([1, 1])))
    rhs = Tensor(CUDA.from_numpy(np.asarray(CANCELLING, np.float32)), 0, Layout(Shape([4, 1]), Stride([1, 1])))
    result = sw.matmul(lhs, rhs, accumulator_dtype=DType.Float64)
    grad = Tensor(CUDA.from_numpy(np.ones(4, np.float32)), 0, result.layout)
    result.backward(grad)
    assert lhs.grad is not None and lhs.grad.dtype() is DType.Float32
    assert lhs.grad[0, 0] == 2.0


@pytest.mark.gpu
@pytest.mark.parametrize("shape,strides", [((300, 1000), (1000, 1)), ((300, 1000), (1, 300)), ((64, 70000), (70000, 1))])
def test_widened_reduce_sum_against_a_binary64_sum(shape, strides):
    from strideweave_b200 import CUDA

    rng = np.random.default_rng(4)
    vals = (rng.standard_normal(shape) * np.exp2(rng.integers(-20, 20, size=shape))).astype(np.float32)
    store = vals.ravel() if strides[1] == 1 else np.ascontiguousarray(vals.T).ravel()
    t = Tensor(CUDA.from_numpy(store), 0, Layout(Shape(list(shape)), Stride(list(strides))))
    got = sw.reduce_sum(t, "a b -> a", accumulator_dtype=DType.Float64).carrier.to_numpy()
    want = vals.astype(np.float64).sum(axis=1)
    # binary64 partial sums in another order: far inside one binary32 rounding of the result
    np.testing.assert_allclose(got, want.astype(np.float32), rtol=1e-6, atol=0)
