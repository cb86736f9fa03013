"""One MX MLP training step on the CUDA carrier (forward, reference autograd
backward with MX re-quantisation, SGD) against a float64 numpy emulation
that quantises every contraction operand with the CPU oracle."""

from __future__ import annotations

import math
import os

import numpy as np
import pytest
from scipy.special import erf

sw = pytest.importorskip("strideweave")
from strideweave import Layout, Shape, Stride, Tensor  # noqa: E402

from oracle import oracle as O  # noqa: E402
from tests.gpu_util import rel_frobenius  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-3  # relative Frobenius error of the contraction path


def dq(m: np.ndarray, code: int) -> np.ndarray:
    """Quantise rows of m (blocks along axis 1) and dequantise, exactly.
    Rows are independent, so row blocks run on host threads (the oracle's C
    calls release the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    m = np.ascontiguousarray(m, dtype=np.float32)
    rows, cols = m.shape
    out = np.empty((rows, cols), np.float64)

    def part(r0: int, r1: int) -> None:
        p, s = O.mx_quantize(code, m[r0:r1], scale_layout=0)
        out[r0:r1] = O.mx_dequantize(code, p, s, r1 - r0, cols, scale_layout=0)

    step = max(1, -(-rows // 32))
    with ThreadPoolExecutor(min(32, os.cpu_count() or 1)) as pool:
        list(pool.map(lambda r0: part(r0, min(rows, r0 + step)), range(0, rows, step)))
    return out


def gelu(x):
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def gelu_grad(x):
    return 0.5 * (1.0 + erf(x / math.sqrt(2.0))) + x * np.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)


def emulate(x, t, Ws, code, lr):
    f32 = lambda a: a.astype(np.float32)  # noqa: E731  (device keeps activations in Float32)
    h, a = [], [x]
    for i, W in enumerate(Ws):
        z = f32(dq(a[-1], code) @ dq(W, code).T)
        h.append(z)
        a.append(f32(gelu(z.astype(np.float64))) if i + 1 < len(Ws) else z)
    y = a[-1]
    n = y.size
    loss = float(np.mean((y.astype(np.float64) - t) ** 2))
    g = f32(2.0 * (y.astype(np.float64) - t) / n)
    dWs = [None] * len(Ws)
    for i in reversed(range(len(Ws))):
        dWs[i] = dq(g.T, code) @ dq(a[i].T, code).T
        if i > 0:
            da = f32(dq(g, code) @ dq(Ws[i].T, code).T)
            g = f32(da.astype(np.float64) * gelu_grad(h[i - 1].astype(np.float64)))
    new = [W - lr * dW for W, dW in zip(Ws, dWs)]
    return loss, dWs, new


@pytest.mark.parametrize("fmt,code", [("MXFP8_E4M3", O.E4M3), ("MXFP4", O.E2M1)])
def test_mlp_training_step_matches_the_emulation(fmt, code):
    from strideweave_b200 import CUDA, nn

    B, dims, lr = 256, [256, 512, 512, 256], 0.1
    rng = np.random.default_rng(0)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    model = nn.MLP(dims, fmt=fmt, seed=1)
    Ws = [layer.weight.carrier.to_numpy().reshape(layer.out_features, layer.in_features) for layer in model.layers]
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, dims[0]]), Stride([dims[0], 1])))
    # targets in the canonical result layout of the last contraction ([B, out] : (1, B))
    tt = Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, Layout(Shape([B, dims[-1]]), Stride([1, B])))
    opt = nn.SGD(model.parameters(), lr=lr)
    loss = nn.MSELoss()(model(xt), tt)
    loss.backward()
    grads = [layer.weight.grad.carrier.to_numpy().reshape(layer.out_features, layer.in_features)
             for layer in model.layers]
    opt.step()
    new = [layer.weight.carrier.to_numpy().reshape(layer.out_features, layer.in_features) for layer in model.layers]

    want_loss, want_grads, want_new = emulate(x, t.astype(np.float64), [W.astype(np.float64) for W in Ws], code, lr)
    assert abs(loss[0] - want_loss) <= TOL * abs(want_loss)
    errs = [rel_frobenius(g, w) for g, w in zip(grads, want_grads)]
    assert max(errs) <= TOL, f"weight-gradient errors {errs}"
    for a, b in zip(new, want_new):
        assert rel_frobenius(a, b) <= TOL
    opt.zero_grad()
    assert all(p.grad is None for p in model.parameters())


def test_config4_full_size_step_stage_by_stage():
    """Config 4 at full size: batch 8192, 1024 -> 4096 -> 4096 -> 1024, GELU,
    MSE, SGD, MXFP8, master weights N(0, 0.02), inputs and targets N(0, 1) -
    the step the benchmark times (MLP.train_step, the two-way quantiser path).

    Every stage is checked at 2e-3 against the float64 emulation of that
    stage fed the device's own Float32 inputs: each pre-activation, the MSE
    gradient, each input gradient and each weight gradient, then the updated
    weights and the loss.  (A free-running emulation drifts at depth: a code
    that rounds the other way in one re-quantisation moves whole rows of the
    next contraction by ~1e-3, which flips many codes of the next
    re-quantisation; the first layer's weight gradient then sits ~3e-3 from
    the emulation's while every stage is within tolerance.)"""
    from strideweave_b200 import CUDA, nn

    B, dims, lr = 8192, [1024, 4096, 4096, 1024], 1e-3
    L = len(dims) - 1
    rng = np.random.default_rng(0)
    model = nn.MLP(dims, fmt="MXFP8_E4M3", seed=0, std=0.02)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    Ws = [layer.weight.carrier.to_numpy().reshape(layer.out_features, layer.in_features) for layer in model.layers]
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, dims[0]]), Stride([dims[0], 1])))
    tt = Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, Layout(Shape([B, dims[-1]]), Stride([1, B])))
    loss = model.train_step(xt, tt, lr=lr)
    plan = nn._dual_step_for(model, xt, tt)
    assert plan is not None  # the fused step ran, not the separate kernels

    def colmajor(tensor, cols):  # [B, cols] from the canonical (1, B) placement
        return tensor.carrier.to_numpy().reshape(cols, B).T.astype(np.float64)

    h = [colmajor(plan.h[i], dims[i + 1]) for i in range(L)]
    g = colmajor(plan.g, dims[-1])
    dx = [None] + [colmajor(plan.dx[i], dims[i]) for i in range(1, L)]
    dw = [plan.dw[i].carrier.to_numpy().reshape(dims[i + 1], dims[i]) for i in range(L)]
    new = [layer.weight.carrier.to_numpy().reshape(layer.out_features, layer.in_features) for layer in model.layers]
    f32 = lambda a: a.astype(np.float32)  # noqa: E731
    acts = [x] + [f32(gelu(h[i])) for i in range(L - 1)]
    errs = {}
    for i in range(L):
        errs[f"h{i}"] = rel_frobenius(h[i], dq(acts[i], O.E4M3) @ dq(Ws[i], O.E4M3).T)
    errs["g"] = rel_frobenius(g, f32(2.0 * (h[-1] - t) / h[-1].size))
    for i in reversed(range(L)):
        gi = f32(g) if i == L - 1 else f32(dx[i + 1] * gelu_grad(h[i]))
        want_dw = dq(gi.T, O.E4M3) @ dq(np.ascontiguousarray(acts[i].T), O.E4M3).T
        errs[f"dw{i}"] = rel_frobenius(dw[i], want_dw)
        if i > 0:
            errs[f"dx{i}"] = rel_frobenius(dx[i], dq(gi, O.E4M3) @ dq(np.ascontiguousarray(Ws[i].T), O.E4M3).T)
        errs[f"w{i}"] = rel_frobenius(new[i], Ws[i].astype(np.float64) - lr * want_dw)
    assert max(errs.values()) <= TOL, f"stage errors {errs}"
    want_loss = float(np.mean((h[-1] - t) ** 2))
    assert abs(loss[0] - want_loss) <= 1e-5 * want_loss


def test_gelu_and_mse_operations_through_autograd():
    from strideweave_b200 import CUDA, nn

    x = np.linspace(-4, 4, 64, dtype=np.float32)
    lay = Layout(Shape([8, 8]), Stride([1, 8]))
    xt = Tensor(CUDA.from_numpy(x), 0, lay)
    y = nn.gelu(xt)
    assert type(y.autograd_ctx).__name__ == "CudaGelu"
    np.testing.assert_allclose(y.carrier.to_numpy(), gelu(x.astype(np.float64)), rtol=2e-6, atol=2e-7)
    target = Tensor(CUDA.from_numpy(np.zeros(64, np.float32)), 0, lay)
    loss = nn.mse_loss(y, target)
    loss.backward()
    want = 2.0 * gelu(x.astype(np.float64)) / 64 * gelu_grad(x.astype(np.float64))
    np.testing.assert_allclose(xt.grad.carrier.to_numpy(), want, rtol=1e-5, atol=1e-7)


def test_gelu_and_its_derivative_over_the_whole_range():
    """The device GELU and GELU' (the elementwise kernels; the two-way
    quantiser applies the same device functions) against the float64 erf
    formula of the reference's CPU operation over [-12, 12] and at +-0,
    +-inf and NaN: 2e-6 relative, 2e-7 absolute for GELU and 5e-7 absolute
    for GELU' (which crosses zero near x = -0.75)."""
    from strideweave_b200 import _native as N
    from tests.gpu_util import empty, to_device, to_host

    x = np.concatenate([np.linspace(-12, 12, 240001, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 30.0, -30.0], np.float32)])
    n = x.size
    dx, ones = to_device(x), to_device(np.ones(n, np.float32))
    out = empty(4 * n)
    N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU, n, N.c_void_p(dx.ptr), None, N.c_void_p(out.ptr), 0.0, None))
    got = to_host(out, n, np.float32).astype(np.float64)
    want = gelu(x.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-7)
    assert np.signbit(got[x.size - 5]) and got[x.size - 5] == 0.0  # gelu(-0) = -0
    N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU_GRAD, n, N.c_void_p(dx.ptr), N.c_void_p(ones.ptr),
                                     N.c_void_p(out.ptr), 0.0, None))
    np.testing.assert_allclose(to_host(out, n, np.float32).astype(np.float64), gelu_grad(x.astype(np.float64)),
                               rtol=2e-6, atol=5e-7)
    special = np.array([np.inf, -np.inf, np.nan], np.float32)
    ds, so = to_device(special), empty(12)
    N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU, 3, N.c_void_p(ds.ptr), None, N.c_void_p(so.ptr), 0.0, None))
    g = to_host(so, 3, np.float32)
    assert g[0] == np.inf and np.isnan(g[1]) and np.isnan(g[2])  # inf * 1, -inf * 0, NaN
    N.raise_device_status()


def test_fused_train_step_equals_the_autograd_step():
    from strideweave_b200 import CUDA, nn

    B, dims = 256, [256, 384, 256]
    rng = np.random.default_rng(5)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    lay_x = Layout(Shape([B, dims[0]]), Stride([dims[0], 1]))
    lay_t = Layout(Shape([B, dims[-1]]), Stride([1, B]))
    a, b = nn.MLP(dims, seed=3), nn.MLP(dims, seed=3)
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, lay_x)
    tt = Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, lay_t)
    loss_a = nn.MSELoss()(a(xt), tt)
    loss_a.backward()
    nn.SGD(a.parameters(), lr=0.05).step()
    loss_b = b.train_step(xt, tt, lr=0.05)
    # the loss is an atomic sum over blocks: equal up to summation order
    assert abs(loss_a[0] - loss_b[0]) <= 1e-6 * abs(loss_a[0])
    for la, lb in zip(a.layers, b.layers):
        np.testing.assert_array_equal(la.weight.carrier.to_numpy(), lb.weight.carrier.to_numpy())


@pytest.mark.parametrize("fmt", ["MXFP8_E4M3", "MXFP4"])
def test_two_way_quantiser_step_equals_the_separate_kernels(fmt):
    """The step that quantises each activation, weight and gradient once, both
    ways, with the GELU (or its derivative) applied on the way in, leaves the
    same weights and loss as the step of separate kernels, bit for bit."""
    from strideweave_b200 import CUDA, nn

    B, dims = 256, [256, 512, 768, 256]
    rng = np.random.default_rng(9)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, dims[0]]), Stride([dims[0], 1])))
    tt = Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, Layout(Shape([B, dims[-1]]), Stride([1, B])))
    a, b = nn.MLP(dims, fmt=fmt, seed=4), nn.MLP(dims, fmt=fmt, seed=4)
    with sw.no_grad():
        for _ in range(2):
            la = nn._train_step_dual(a, xt, tt, 0.05)
            lb = nn._train_step_separate(b, xt, tt, 0.05)
            assert la is not None
            assert abs(la[0] - lb[0]) <= 1e-6 * abs(lb[0])
    for wa, wb in zip(a.layers, b.layers):
        np.testing.assert_array_equal(wa.weight.carrier.to_numpy(), wb.weight.carrier.to_numpy())


def test_untileable_batch_falls_back_to_the_separate_kernels():
    from strideweave_b200 import CUDA, nn

    B, dims = 128, [128, 256, 128]  # the batch is tileable, a 96-row input is not
    rng = np.random.default_rng(2)
    model = nn.MLP(dims, seed=1)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    xt = Tensor(CUDA.from_numpy(x.T.ravel().copy()), 0, Layout(Shape([B, dims[0]]), Stride([1, B])))
    tt = Tensor(CUDA.from_numpy(np.zeros(B * dims[-1], np.float32)), 0,
                Layout(Shape([B, dims[-1]]), Stride([1, B])))
    assert nn.MLP(dims, seed=1).train_step(xt, tt, lr=0.01)[0] > 0  # column-major input: the dual path reads it
    odd = Tensor(CUDA.from_numpy(np.zeros(96 * dims[0], np.float32)), 0,
                 Layout(Shape([96, dims[0]]), Stride([dims[0], 1])))
    with sw.no_grad():
        assert nn._train_step_dual(model, odd, tt, 0.01) is None


@pytest.mark.parametrize("fmt", ["MXFP8_E4M3", "MXFP4"])
def test_captured_step_replays_the_eager_step(fmt):
    """Three replays of the CUDA-graph step leave the weights and losses of
    three eager steps, bit for bit; new data written into x is read by the
    next replay."""
    from strideweave_b200 import CUDA, nn

    B, dims = 256, [256, 512, 256]
    rng = np.random.default_rng(13)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    lay_x = Layout(Shape([B, dims[0]]), Stride([dims[0], 1]))
    lay_t = Layout(Shape([B, dims[-1]]), Stride([1, B]))
    a, b = nn.MLP(dims, fmt=fmt, seed=2), nn.MLP(dims, fmt=fmt, seed=2)
    xa, ta = Tensor(CUDA.from_numpy(x.ravel()), 0, lay_x), Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, lay_t)
    xb, tb = Tensor(CUDA.from_numpy(x.ravel()), 0, lay_x), Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, lay_t)
    graph = b.capture_step(xb, tb, lr=0.05)
    x2 = rng.standard_normal((B, dims[0])).astype(np.float32)
    for k in range(3):
        if k == 2:  # new data: eager gets a new tensor, the graph gets it written into its input
            xa = Tensor(CUDA.from_numpy(x2.ravel()), 0, lay_x)
            xb.carrier.upload_raw(x2.ravel())
        la = a.train_step(xa, ta, lr=0.05)
        lb = graph.step()
        assert abs(la[0] - lb[0]) <= 1e-6 * abs(la[0])  # an atomic sum over blocks
    for wa, wb in zip(a.layers, b.layers):
        np.testing.assert_array_equal(wa.weight.carrier.to_numpy(), wb.weight.carrier.to_numpy())
    graph.close()



@pytest.mark.parametrize("n", [1 << 20, 1000003])
def test_mse_loss_and_gradient_in_one_pass(n):
    """sw_mse_f32 with loss and gradient and no upstream runs one fused pass:
    the gradient equals the gradient-only call bit for bit, the loss the
    loss-only call up to the order of its atomic sum."""
    from strideweave_b200 import _native as N
    from tests.gpu_util import empty, to_device, to_host

    rng = np.random.default_rng(n)
    p = rng.standard_normal(n).astype(np.float32)
    t = rng.standard_normal(n).astype(np.float32)
    dp, dt = to_device(p), to_device(t)
    loss_a, grad_a = empty(4), empty(4 * n)
    loss_b, grad_b = empty(4), empty(4 * n)
    N.check(N.lib.sw_mse_f32(n, N.c_void_p(dp.ptr), N.c_void_p(dt.ptr), N.c_void_p(loss_a.ptr), None,
                             N.c_void_p(grad_a.ptr), None))
    N.check(N.lib.sw_mse_f32(n, N.c_void_p(dp.ptr), N.c_void_p(dt.ptr), N.c_void_p(loss_b.ptr), None, None, None))
    N.check(N.lib.sw_mse_f32(n, N.c_void_p(dp.ptr), N.c_void_p(dt.ptr), None, None, N.c_void_p(grad_b.ptr), None))
    np.testing.assert_array_equal(to_host(grad_a, n, np.float32), to_host(grad_b, n, np.float32))
    la, lb = to_host(loss_a, 1, np.float32)[0], to_host(loss_b, 1, np.float32)[0]
    want = float(np.mean((p.astype(np.float64) - t) ** 2))
    assert abs(la - lb) <= 1e-5 * lb and abs(la - want) <= 1e-5 * want
