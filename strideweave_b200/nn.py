"""Training-step building blocks on the CUDA carrier.

These mirror the reference's `strideweave.nn` pieces:

- `Linear`: src/strideweave/nn/modules.py:40-127, weight [out, in] and
  y = x @ weight;
- `GELU`: modules.py:273-302, erf form;
- `MSELoss`: modules.py:129-200, mean of squared differences;
- `SGD`: src/strideweave/nn/optim.py:17-100, p -= lr * p.grad.

The autograd graph is still the reference's (`Tensor.backward`), but every
node runs on the GPU:

- `MXLinear` contracts through the differentiable MX contraction
  (`mx_linear`). The forward quantises x and the weight along `in`; the
  backward re-quantises along each gradient contraction's own K.
- `GELU` and `MSELoss` are fused elementwise kernels with their vector-Jacobian
  products.
- `SGD.step` is one fused update kernel per parameter. The reference updates
  one element at a time through carrier indexing.

Elementwise operations work on a tensor's whole storage range. That needs a
compact, injective layout, which the contraction results always have.
"""

from __future__ import annotations

from typing import Any, Iterable

import numpy as np

from . import _native as N
from ._host import DType, Layout, Operation, Shape, Stride, Tensor, require_capability, resolve_operation_plan
from .layout_plan import canonical_layout


def _compact(t: Any, name: str) -> tuple[int, int]:
    """(address, element count) of a Float32 CUDA tensor whose layout fills
    [offset, offset + size) exactly once."""
    from .carrier import CUDA

    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a Tensor")
    t._require_single_subtensor("CUDA elementwise operation")
    if not isinstance(t.carrier, CUDA) or t.carrier.dtype() is not DType.Float32:
        raise TypeError(f"{name} must be a Float32 tensor on a CUDA carrier")
    if t.carrier.swizzle is not None:
        raise NotImplementedError(f"{name}: swizzled carriers are not supported by elementwise operations")
    lay = t.layout
    if not lay.is_injective or lay.cosize != t.size():
        raise NotImplementedError(f"{name}: elementwise operations need a compact, injective layout")
    return t.carrier.data_ptr + 4 * t.offset, t.size()


def _like(t: Tensor) -> Tensor:
    from .carrier import CUDA

    return Tensor(CUDA(t.size(), dtype=DType.Float32, empty=True, device=t.carrier.device), 0, t.layout)


def _ptr(t: Tensor) -> int:
    return t.carrier.data_ptr + 4 * t.offset


class CudaGelu(Operation):
    """gelu(x) = x / 2 * (1 + erf(x / sqrt 2)) (the reference's Float32 plan,
    src/strideweave/carriers/cpu/native/_cpu_operation.hpp:33-40)."""

    def _forward(self, tensor: Any) -> Tensor:
        from .carrier import CUDA

        ptr, n = _compact(tensor, "tensor")
        require_capability(CUDA, resolve_operation_plan("gelu", tensor.carrier.dtype()))
        out = _like(tensor)
        N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU, n, N.c_void_p(ptr), None, N.c_void_p(_ptr(out)), 0.0, None))
        return out

    def backward(self, gradient: Any) -> tuple[Any]:
        (tensor,) = self.inputs()
        xp, n = _compact(tensor, "tensor")
        gp, gn = _compact(gradient, "gradient")
        if gradient.layout != tensor.layout:
            raise ValueError("Tensor layouts must match")
        out = _like(tensor)
        N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU_GRAD, n, N.c_void_p(xp), N.c_void_p(gp), N.c_void_p(_ptr(out)),
                                         0.0, None))
        return (out,)


SCALAR = Layout(Shape(1), Stride(1))


class CudaMSELoss(Operation):
    """mean((pred - target)^2) as one fused kernel, with both gradients."""

    def _forward(self, pred: Any, target: Any) -> Tensor:
        from .carrier import CUDA

        pp, n = _compact(pred, "pred")
        tp, tn = _compact(target, "target")
        if pred.layout != target.layout:
            raise ValueError("pred and target layouts must match")
        out = Tensor(CUDA(1, dtype=DType.Float32, empty=True, device=pred.carrier.device), 0, SCALAR)
        N.check(N.lib.sw_mse_f32(n, N.c_void_p(pp), N.c_void_p(tp), N.c_void_p(_ptr(out)), None, None, None))
        return out

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        pred, target = self.inputs()
        pp, n = _compact(pred, "pred")
        tp, _ = _compact(target, "target")
        up, _ = _compact(gradient, "gradient")
        dp, dt = _like(pred), _like(target)
        N.check(N.lib.sw_mse_f32(n, N.c_void_p(pp), N.c_void_p(tp), None, N.c_void_p(up), N.c_void_p(_ptr(dp)), None))
        N.check(N.lib.sw_mse_f32(n, N.c_void_p(tp), N.c_void_p(pp), None, N.c_void_p(up), N.c_void_p(_ptr(dt)), None))
        return (dp, dt)


def gelu(t: Tensor) -> Tensor:
    return t.carrier.dispatch_op("gelu").forward(t)


def mse_loss(pred: Tensor, target: Tensor) -> Tensor:
    return pred.carrier.dispatch_op("mse_loss").forward(pred, target)


# ---- modules ------------------------------------------------------------------------


def _parameter(values: np.ndarray, layout: Layout) -> Any:
    from strideweave.core.module import Parameter

    from .carrier import CUDA

    return Parameter(CUDA.from_numpy(np.ascontiguousarray(values, dtype=np.float32).ravel()), 0, layout)


class MXLinear:
    """y[b, o] = sum_i x[b, i] weight[o, i], MX-quantised on the tensor cores.

    `weight` is a Float32 master parameter [out, in] stored row-major (the
    K-major operand the contraction reads without a transpose).
    """

    def __init__(self, in_features: int, out_features: int, *, fmt: str = "MXFP8_E4M3",
                 init: np.ndarray | None = None, rng: np.random.Generator | None = None, std: float = 0.02) -> None:
        if init is None:
            rng = rng if rng is not None else np.random.default_rng()
            init = rng.standard_normal((out_features, in_features)) * std
        if init.shape != (out_features, in_features):
            raise ValueError("init must have shape [out_features, in_features]")
        self.in_features, self.out_features, self.fmt = in_features, out_features, fmt
        self.weight = _parameter(init, Layout(Shape([out_features, in_features]), Stride([in_features, 1])))

    def parameters(self) -> list[Any]:
        return [self.weight]

    def __call__(self, x: Tensor) -> Tensor:
        from . import mx

        return mx.linear(x, self.weight, fmt=self.fmt)


class GELU:
    def __call__(self, x: Tensor) -> Tensor:
        return gelu(x)


class MSELoss:
    def __call__(self, pred: Tensor, target: Tensor) -> Tensor:
        return mse_loss(pred, target)


class MLP:
    """MXLinear -> GELU -> ... -> MXLinear (no activation after the last)."""

    def __init__(self, dims: list[int], *, fmt: str = "MXFP8_E4M3", seed: int = 0, std: float = 0.02) -> None:
        rng = np.random.default_rng(seed)
        self.layers = [MXLinear(dims[i], dims[i + 1], fmt=fmt, rng=rng, std=std) for i in range(len(dims) - 1)]
        self.act = GELU()

    def parameters(self) -> list[Any]:
        return [p for layer in self.layers for p in layer.parameters()]

    def __call__(self, x: Tensor) -> Tensor:
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i + 1 < len(self.layers):
                x = self.act(x)
        return x

    def train_step(self, x: Tensor, target: Tensor, lr: float) -> Tensor:
        return train_step(self, x, target, lr)


def gelu_grad(x: Tensor, g: Tensor) -> Tensor:
    """g * gelu'(x) (same layout as x)."""
    xp, n = _compact(x, "x")
    gp, _ = _compact(g, "gradient")
    if g.layout != x.layout:
        raise ValueError("Tensor layouts must match")
    out = _like(x)
    N.check(N.lib.sw_elementwise_f32(N.SW_EW_GELU_GRAD, n, N.c_void_p(xp), N.c_void_p(gp), N.c_void_p(_ptr(out)),
                                     0.0, None))
    return out


def train_step(model: "MLP", x: Tensor, target: Tensor, lr: float) -> Tensor:
    """One training step of an MLP: forward, MSE loss, backward and SGD, with
    the same contractions and the same MX re-quantisation as the autograd path
    (MxLinear / CudaGelu / CudaMSELoss), scheduled explicitly.

    The reference's leaf-gradient accumulation copies a gradient element by
    element through `Tensor.__getitem__` (src/strideweave/core/native/
    _tensor.cpp:914-990).  That is harmless on a host carrier but would stall
    a device carrier for seconds per weight, so the full-size step runs here.

    Each activation, weight and gradient is read once by the two-way quantiser
    (``sw_mx_quantize_dual``): it applies the GELU (forward) or the GELU
    derivative (backward) on the way in and writes both operands the layer's
    contractions take from it.  The activations themselves are never stored,
    and the result is bit-identical to the autograd step.  Shapes that the
    quantiser cannot tile fall back to the separate kernels.  Returns the loss
    (a one-element CUDA tensor, read it after the step).
    """
    from strideweave import no_grad

    with no_grad():
        loss = _train_step_dual(model, x, target, lr)
        if loss is None:
            loss = _train_step_separate(model, x, target, lr)
    return loss


def _mse_and_grad(y: Tensor, target: Tensor) -> tuple[Tensor, Tensor]:
    from .carrier import CUDA

    pp, n = _compact(y, "pred")
    tp, _ = _compact(target, "target")
    if y.layout != target.layout:
        raise ValueError("pred and target layouts must match")
    loss = Tensor(CUDA(1, dtype=DType.Float32, empty=True, device=y.carrier.device), 0, SCALAR)
    g = _like(y)
    # unit upstream gradient: no host-to-device upload inside the step
    N.check(N.lib.sw_mse_f32(n, N.c_void_p(pp), N.c_void_p(tp), N.c_void_p(_ptr(loss)), None,
                             N.c_void_p(_ptr(g)), None))
    return loss, g


def _sgd_update(weight: Any, dw: Tensor, lr: float) -> None:
    wp, wn = _compact(weight, "weight")
    N.check(N.lib.sw_elementwise_f32(N.SW_EW_AXPY, wn, N.c_void_p(wp), N.c_void_p(_ptr(dw)), N.c_void_p(wp),
                                     -float(lr), None))
    weight.carrier._increment_version()


def _train_step_dual(model: "MLP", x: Tensor, target: Tensor, lr: float) -> Tensor | None:
    from . import kernels, mx
    from .carrier import CUDA
    from .layout_plan import injective_layout_for, mode_leaves, single_stride

    layers = model.layers
    codes = {mx.FORMATS[layer.fmt][2] for layer in layers}
    if len(codes) != 1:
        return None
    code = codes.pop()
    q = 256 if code == N.SW_MX_E2M1 else 128
    geo = mx.dual_geometry(x)
    if geo is None or any(mx.dual_geometry(layer.weight) is None for layer in layers):
        return None
    B = geo[2] if geo[4] else geo[1]
    if B % q or any(layer.in_features % q or layer.out_features % q for layer in layers):
        return None
    if x.layout.shape.top_level[1] != layers[0].in_features:
        raise ValueError("Matmul inner dimensions must match")
    dev = x.carrier.device

    def rb(k: int) -> int:
        return kernels.mx_row_bytes(code, k)

    def gemm(a: Any, b: Any, out: Tensor, M: int, Nn: int, K: int) -> None:
        (_, s0), (_, s1) = single_stride(mode_leaves(out.layout, 0)), single_stride(mode_leaves(out.layout, 1))
        kernels.mx_gemm(code, a[0].data_ptr, rb(K), a[1].data_ptr, b[0].data_ptr, rb(K), b[1].data_ptr,
                        _ptr(out), M, Nn, K, ldc_m=s0, ldc_n=s1)

    # forward: the operands of each layer's input (x, then gelu(h)) and weights
    wq = [mx.quantize_both(layer.weight, code, need_tT=i > 0) for i, layer in enumerate(layers)]
    aq = [mx.quantize_both(x, code)]
    pres = []
    for i, layer in enumerate(layers):
        lay = canonical_layout(x.layout.shape.top_level[0], layer.weight.layout.shape.top_level[0])
        h = Tensor(CUDA(lay.cosize, dtype=DType.Float32, empty=True, device=dev), 0, lay)
        gemm(aq[i][0], wq[i][0], h, B, layer.out_features, layer.in_features)
        pres.append(h)
        if i + 1 < len(layers):
            aq.append(mx.quantize_both(h, code, transform=N.SW_XF_GELU))
            if aq[-1] is None:
                raise RuntimeError("the two-way quantiser refused a contraction result")
    loss, g = _mse_and_grad(pres[-1], target)
    g_h, xf = None, N.SW_XF_NONE
    for i in reversed(range(len(layers))):
        layer = layers[i]
        qg = mx.quantize_both(g, code, transform=xf, h=g_h, need_t=i > 0)
        if qg is None:
            raise RuntimeError("the two-way quantiser refused a gradient")
        dx = None
        if i > 0:
            # dx[b, k] = sum_o g[b, o] w[o, k], stored like the layer input
            lay = injective_layout_for(pres[i - 1].layout)
            dx = Tensor(CUDA(lay.cosize, dtype=DType.Float32, empty=True, device=dev), 0, lay)
            gemm(qg[0], wq[i][1], dx, B, layer.in_features, layer.out_features)
        # dw[o, k] = sum_b g[b, o] a[b, k]
        lay = injective_layout_for(layer.weight.layout)
        dw = Tensor(CUDA(lay.cosize, dtype=DType.Float32, empty=True, device=dev), 0, lay)
        gemm(qg[1], aq[i][1], dw, layer.out_features, layer.in_features, B)
        _sgd_update(layer.weight, dw, lr)
        if i > 0:
            g, g_h, xf = dx, pres[i - 1], N.SW_XF_GELU_GRAD
    return loss


def _train_step_separate(model: "MLP", x: Tensor, target: Tensor, lr: float) -> Tensor:
    """The same step with one kernel per elementwise operation and one
    quantisation per contraction operand."""
    from . import mx

    acts, pres = [x], []
    for i, layer in enumerate(model.layers):
        h = mx.linear_forward(acts[-1], layer.weight, layer.fmt)
        pres.append(h)
        acts.append(gelu(h) if i + 1 < len(model.layers) else h)
    loss, g = _mse_and_grad(acts[-1], target)
    for i in reversed(range(len(model.layers))):
        layer = model.layers[i]
        dx, dw = mx.linear_backward(acts[i], layer.weight, g, layer.fmt, need_dx=i > 0)
        _sgd_update(layer.weight, dw, lr)
        if i > 0:
            g = gelu_grad(pres[i - 1], dx)
    return loss


class SGD:
    """p -= lr * p.grad for every parameter with a gradient, one fused update
    kernel each (the reference's SGD.step, src/strideweave/nn/optim.py:45-80)."""

    def __init__(self, parameters: Iterable[Any], lr: float) -> None:
        self._parameters = tuple(parameters)
        if lr <= 0:
            raise ValueError("lr must be positive")
        self.lr = float(lr)

    def step(self) -> None:
        for p in self._parameters:
            g = p.grad
            if g is None:
                continue
            pp, n = _compact(p, "parameter")
            gp, gn = _compact(g, "gradient")
            if g.layout != p.layout or gn != n:
                raise ValueError("a gradient must share its parameter's layout")
            N.check(N.lib.sw_elementwise_f32(N.SW_EW_AXPY, n, N.c_void_p(pp), N.c_void_p(gp), N.c_void_p(pp),
                                             -self.lr, None))
            p.carrier._increment_version()

    def zero_grad(self) -> None:
        for p in self._parameters:
            p.grad = None


NN_OPERATIONS = {"gelu": CudaGelu, "mse_loss": CudaMSELoss}

__all__ = ["GELU", "MLP", "MSELoss", "MXLinear", "SGD", "gelu", "gelu_grad", "mse_loss", "train_step"]
