"""The reference's own ``strideweave.nn`` modules on CUDA-carrier tensors.

``Linear`` (with its broadcast bias), ``GELU``, ``MSELoss`` and ``SGD``
(src/strideweave/nn/modules.py:40-176,273-302, nn/optim.py:17-80) run
unchanged: their contraction, elementwise arithmetic, reduction and
autograd dispatch to the CUDA carrier's operations.  A two-layer step on
CUDA parameters is compared with the same step of the same modules on the
reference CPU carrier: the loss, every parameter gradient and every updated
parameter agree within the path's 2e-3 relative Frobenius tolerance (the
CUDA contraction sums in another order; elementwise results are the same
binary32 operations).
"""

from __future__ import annotations

import ctypes
import random

import numpy as np
import pytest

sw = pytest.importorskip("strideweave")
import strideweave.nn as snn  # noqa: E402
from strideweave import Layout, Shape, Stride, Tensor  # noqa: E402
from strideweave.module import Parameter  # noqa: E402

from tests.gpu_util import rel_frobenius  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3
B, IN, HID, OUT = 64, 48, 96, 40


def cpu_values(t: Tensor) -> np.ndarray:
    """The flat storage of a tensor on the reference CPU carrier."""
    n = t.carrier.size()
    return np.ctypeslib.as_array((ctypes.c_float * n).from_address(t.carrier.pointer())).copy()


def logical(t: Tensor) -> np.ndarray:
    """Logical values of a two-mode tensor, on either carrier."""
    from strideweave_b200 import CUDA

    flat = t.carrier.to_numpy() if isinstance(t.carrier, CUDA) else cpu_values(t)
    rows, cols = int(t.layout.shape[0]), int(t.layout.shape[1])
    out = np.empty((rows, cols), np.float64)
    for i in range(rows):
        for j in range(cols):
            out[i, j] = flat[t.offset + t.layout((i, j))]
    return out


def model(on_cuda: bool):
    from strideweave_b200 import CUDA

    layers = [snn.Linear(IN, HID, rng=random.Random(0)), snn.Linear(HID, OUT, rng=random.Random(1))]
    if on_cuda:
        for layer in layers:
            for name in ("weight", "bias"):
                p = getattr(layer, name)
                setattr(layer, name, Parameter(Tensor(CUDA.from_numpy(cpu_values(p)), 0, p.layout)))
    return layers


def data(on_cuda: bool):
    from strideweave_b200 import CUDA

    rng = np.random.default_rng(7)
    x = rng.standard_normal((B, IN)).astype(np.float32)
    t = rng.standard_normal((B, OUT)).astype(np.float32)
    lay_x = Layout(Shape([B, IN]), Stride([1, B]))  # the nn convention: column-major
    lay_t = Layout(Shape([B, OUT]), Stride([1, B]))
    flat_x, flat_t = x.T.ravel().copy(), t.T.ravel().copy()
    if on_cuda:
        return Tensor(CUDA.from_numpy(flat_x), 0, lay_x), Tensor(CUDA.from_numpy(flat_t), 0, lay_t)
    from strideweave import CPU

    cx, ct = CPU(flat_x.size), CPU(flat_t.size)
    for carrier, flat in ((cx, flat_x), (ct, flat_t)):
        np.ctypeslib.as_array((ctypes.c_float * flat.size).from_address(carrier.pointer()))[:] = flat
    return Tensor(cx, 0, lay_x), Tensor(ct, 0, lay_t)


def step(on_cuda: bool):
    l1, l2 = model(on_cuda)
    x, t = data(on_cuda)
    gelu, mse = snn.GELU(), snn.MSELoss()
    loss = mse(l2(gelu(l1(x))), t)
    loss.backward()
    params = [l1.weight, l1.bias, l2.weight, l2.bias]
    grads = [logical(p.grad) for p in params]
    snn.SGD(params, lr=0.1).step()
    return float(loss[0]), grads, [logical(p) for p in params], loss


def test_reference_modules_train_on_the_cuda_carrier():
    from strideweave_b200 import CUDA, ops

    cuda_loss, cuda_grads, cuda_params, loss_t = step(True)
    cpu_loss, cpu_grads, cpu_params, _ = step(False)
    assert isinstance(loss_t.carrier, CUDA)
    # the loss node is the CUDA carrier's scalar multiply (friendly.mean)
    assert isinstance(loss_t.autograd_ctx, ops.CudaMul)
    assert abs(cuda_loss - cpu_loss) <= TOL * abs(cpu_loss)
    for g, want in zip(cuda_grads, cpu_grads):
        assert rel_frobenius(g, want) <= TOL
    for p, want in zip(cuda_params, cpu_params):
        assert rel_frobenius(p, want) <= TOL


def test_elementwise_arithmetic_matches_the_cpu_carrier():
    """add, sub, mul (tensor and scalar), pow and neg with a broadcast
    operand: the CPU carrier's binary32 results bit for bit (pow within one
    unit in the last place of the host's powf), and the same gradients."""
    from strideweave import CPU

    from strideweave_b200 import CUDA

    rng = np.random.default_rng(11)
    a = rng.standard_normal(6 * 5).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    lay_a = Layout(Shape([6, 5]), Stride([5, 1]))
    lay_b = Layout(Shape([1, 5]), Stride([5, 1]))

    def on(carrier_cls, flat, layout):
        if carrier_cls is CUDA:
            return Tensor(CUDA.from_numpy(flat), 0, layout)
        c = CPU(flat.size)
        np.ctypeslib.as_array((ctypes.c_float * flat.size).from_address(c.pointer()))[:] = flat
        return Tensor(c, 0, layout)

    results, grads = {}, {}
    for cls in (CUDA, CPU):
        ta, tb = on(cls, a, lay_a), on(cls, b, lay_b)
        wide = sw.broadcast_to(tb, ta.layout.shape)
        outs = [ta + wide, ta - wide, ta * 0.37, ta ** 2.0, -ta, sw.mul(ta, wide)]
        results[cls] = [logical(o).astype(np.float32) for o in outs]
        total = sw.reduce_sum(sw.reduce_sum(outs[1] * 1.5 + outs[3] - outs[5], "a b -> a"), "a -> 1")
        total.backward()
        grads[cls] = (logical(ta.grad).astype(np.float32), logical(tb.grad).astype(np.float32))
    for k, (got, want) in enumerate(zip(results[CUDA], results[CPU])):
        if k == 3:  # pow
            assert np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32)).max() <= 1
        else:
            np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    for got, want in zip(grads[CUDA], grads[CPU]):
        assert rel_frobenius(got, want) <= 1e-6
