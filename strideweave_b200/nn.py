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

    def capture_step(self, x: Tensor, target: Tensor, lr: float) -> "CapturedTrainStep":
        """``train_step(x, target, lr)`` captured in a CUDA graph (see CapturedTrainStep)."""
        return CapturedTrainStep(self, x, target, lr)


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


class _DualStep:
    """The buffers and kernel arguments of one MLP training step through the
    two-way quantiser, built once for a model and an input / target placement
    and reused by every step, eager or captured in a CUDA graph.

    Per step: each weight, the input, each hidden pre-activation (with the
    GELU) and each gradient (with the GELU derivative) is quantised once into
    the operands both of its contractions take; eight contractions; the MSE
    loss and gradient; an in-place SGD update per weight.  Nothing is
    allocated after construction except the caller's loss."""

    @classmethod
    def build(cls, model: "MLP", x: Tensor, target: Tensor) -> "_DualStep | None":
        from . import mx

        layers = model.layers
        codes = {mx.FORMATS[layer.fmt][2] for layer in layers}
        if len(codes) != 1:
            return None
        code = next(iter(codes))
        q = 256 if code == N.SW_MX_E2M1 else 128
        geo = mx.dual_geometry(x)
        if geo is None or any(mx.dual_geometry(layer.weight) is None for layer in layers):
            return None
        B = geo[2] if geo[4] else geo[1]
        if B % q or any(layer.in_features % q or layer.out_features % q for layer in layers):
            return None
        if x.layout.shape.top_level[1] != layers[0].in_features:
            raise ValueError("Matmul inner dimensions must match")
        return cls(model, x, target, code, B)

    def __init__(self, model: "MLP", x: Tensor, target: Tensor, code: int, B: int) -> None:
        from . import kernels, mx
        from .carrier import CUDA
        from .layout_plan import injective_layout_for, mode_leaves, single_stride

        self.layers = model.layers
        self.code, self.B = code, B
        self.x, self.target = x, target
        dev = x.carrier.device
        elem = DType.E4M3 if code == N.SW_MX_E4M3 else DType.E2M1

        def planes(n: int, k: int) -> tuple[Any, Any]:
            return (CUDA(n * k, dtype=elem, empty=True, device=dev),
                    CUDA(kernels.scale_bytes_tc128(n, k // 32), dtype=DType.E8M0, empty=True, device=dev))

        def f32(layout: Layout) -> Tensor:
            return Tensor(CUDA(layout.cosize, dtype=DType.Float32, empty=True, device=dev), 0, layout)

        def strides(t: Tensor) -> tuple[int, int]:
            return single_stride(mode_leaves(t.layout, 0))[1], single_stride(mode_leaves(t.layout, 1))[1]

        L = len(self.layers)
        self.wq = [(planes(l.out_features, l.in_features), planes(l.in_features, l.out_features) if i > 0 else None)
                   for i, l in enumerate(self.layers)]
        self.aq = [(planes(B, l.in_features), planes(l.in_features, B)) for l in self.layers]
        self.h = [f32(canonical_layout(x.layout.shape.top_level[0], l.weight.layout.shape.top_level[0]))
                  for l in self.layers]
        if self.h[-1].layout != target.layout:
            raise ValueError("pred and target layouts must match")
        self.g = f32(self.h[-1].layout)
        self.qg = [(planes(B, l.out_features) if i > 0 else None, planes(l.out_features, B))
                   for i, l in enumerate(self.layers)]
        self.dx = [None] + [f32(injective_layout_for(self.h[i - 1].layout)) for i in range(1, L)]
        self.dw = [f32(injective_layout_for(l.weight.layout)) for l in self.layers]
        self.n_out = self.h[-1].size()
        # every call of a step, with its arguments resolved to integers
        self.calls: list[tuple[str, tuple]] = []
        for i, layer in enumerate(self.layers):
            self._dual(layer.weight, N.SW_XF_NONE, None, self.wq[i][0], self.wq[i][1])
        self._dual(x, N.SW_XF_NONE, None, self.aq[0][0], self.aq[0][1])
        for i, layer in enumerate(self.layers):
            self._gemm(self.aq[i][0], self.wq[i][0], self.h[i], B, layer.out_features, layer.in_features, strides)
            if i + 1 < L:
                self._dual(self.h[i], N.SW_XF_GELU, None, self.aq[i + 1][0], self.aq[i + 1][1])
        self.calls.append(("mse", (self.n_out, _ptr(self.h[-1]), _ptr(target), _ptr(self.g))))
        g, g_h, xf = self.g, None, N.SW_XF_NONE
        for i in reversed(range(L)):
            layer = self.layers[i]
            self._dual(g, xf, g_h, self.qg[i][0], self.qg[i][1])
            if i > 0:
                # dx[b, k] = sum_o g[b, o] w[o, k], stored like the layer input
                self._gemm(self.qg[i][0], self.wq[i][1], self.dx[i], B, layer.in_features, layer.out_features,
                           strides)
            # dw[o, k] = sum_b g[b, o] a[b, k]
            self._gemm(self.qg[i][1], self.aq[i][1], self.dw[i], layer.out_features, layer.in_features, B, strides)
            wp, wn = _compact(layer.weight, "weight")
            self.calls.append(("axpy", (wn, wp, _ptr(self.dw[i]))))
            if i > 0:
                g, g_h, xf = self.dx[i], self.h[i - 1], N.SW_XF_GELU_GRAD

    def _dual(self, t: Tensor, xf: int, h: Tensor | None, q_t: Any, q_tT: Any) -> None:
        from . import mx

        geo = mx.dual_geometry(t)
        if geo is None or (h is not None and (h.layout != t.layout or mx.dual_geometry(h) is None)):
            raise RuntimeError("the two-way quantiser cannot read a tensor of the step")
        ptr, rows, cols, ld, transposed = geo
        row_q, col_q = (q_tT, q_t) if transposed else (q_t, q_tT)
        self.calls.append(("dual", (xf, ptr, _ptr(h) if h is not None else 0, rows, cols, ld,
                                    (row_q[0].data_ptr, row_q[1].data_ptr) if row_q else None,
                                    (col_q[0].data_ptr, col_q[1].data_ptr) if col_q else None)))

    def _gemm(self, a: Any, b: Any, out: Tensor, M: int, Nn: int, K: int, strides: Any) -> None:
        s0, s1 = strides(out)
        self.calls.append(("gemm", (a[0].data_ptr, a[1].data_ptr, b[0].data_ptr, b[1].data_ptr, _ptr(out), M, Nn,
                                    K, s0, s1)))

    def run(self, loss_ptr: int, lr: float, stream: int = 0) -> None:
        """Enqueues one step on `stream`; the loss lands at loss_ptr."""
        from . import kernels

        code = self.code
        sp = N.c_void_p(stream or None)
        for kind, a in self.calls:
            if kind == "dual":
                xf, ptr, hp, rows, cols, ld, rq, cq = a
                kernels.mx_quantize_dual(code, xf, ptr, hp, rows, cols, ld, rq, cq, stream=stream)
            elif kind == "gemm":
                ap, asc, bp, bsc, cp, M, Nn, K, s0, s1 = a
                rb = kernels.mx_row_bytes(code, K)
                kernels.mx_gemm(code, ap, rb, asc, bp, rb, bsc, cp, M, Nn, K, ldc_m=s0, ldc_n=s1, stream=stream)
            elif kind == "mse":
                n, pp, tp, gp = a
                N.check(N.lib.sw_mse_f32(n, N.c_void_p(pp), N.c_void_p(tp), N.c_void_p(loss_ptr), None,
                                         N.c_void_p(gp), sp))
            else:
                wn, wp, dwp = a
                N.check(N.lib.sw_elementwise_f32(N.SW_EW_AXPY, wn, N.c_void_p(wp), N.c_void_p(dwp),
                                                 N.c_void_p(wp), -float(lr), sp))

    def bump_weight_versions(self) -> None:
        for layer in self.layers:
            layer.weight.carrier._increment_version()


def _dual_step_for(model: "MLP", x: Tensor, target: Tensor) -> _DualStep | None:
    """The model's cached step for this input / target placement (rebuilt when
    the placement or a weight's storage changes)."""
    key = (x.carrier.data_ptr + 4 * x.offset, str(x.layout), target.carrier.data_ptr + 4 * target.offset,
           str(target.layout), tuple(layer.weight.carrier.data_ptr for layer in model.layers))
    cached = getattr(model, "_dual_step", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    model._dual_step = None  # release the previous buffers first
    plan = _DualStep.build(model, x, target)
    if plan is not None:
        model._dual_step = (key, plan)
    return plan


def _train_step_dual(model: "MLP", x: Tensor, target: Tensor, lr: float) -> Tensor | None:
    from .carrier import CUDA

    plan = _dual_step_for(model, x, target)
    if plan is None:
        return None
    loss = Tensor(CUDA(1, dtype=DType.Float32, empty=True, device=x.carrier.device), 0, SCALAR)
    plan.run(_ptr(loss), lr)
    plan.bump_weight_versions()
    return loss


class CapturedTrainStep:
    """An MLP training step captured once in a CUDA graph and replayed.

    ``step()`` launches the graph on the legacy default stream, where it is
    ordered with every other carrier operation, and returns that step's loss.
    The graph holds the addresses of ``x``, ``target`` and the weights: to
    train on other data write it into ``x`` and ``target`` (the replay reads
    their current contents).  ``lr`` is fixed at capture.  The step is the one
    ``MLP.train_step`` runs (the two-way quantiser path), bit for bit.
    """

    def __init__(self, model: "MLP", x: Tensor, target: Tensor, lr: float) -> None:
        from .carrier import CUDA

        self._exec = None
        self._stream = None
        plan = _DualStep.build(model, x, target)
        if plan is None:
            raise NotImplementedError("CapturedTrainStep needs shapes the two-way quantiser tiles "
                                      "(batch and features multiples of 128, 256 for MXFP4)")
        self.plan = plan
        self.loss = Tensor(CUDA(1, dtype=DType.Float32, empty=True, device=x.carrier.device), 0, SCALAR)
        stream = N.c_void_p()
        N.check(N.lib.sw_stream_create(N.ctypes.byref(stream)))
        self._stream = stream.value
        N.check(N.lib.sw_graph_capture_begin(N.c_void_p(self._stream)))
        exec_ = N.c_void_p()
        try:
            plan.run(_ptr(self.loss), lr, self._stream)
        finally:
            rc = N.lib.sw_graph_capture_end(N.c_void_p(self._stream), N.ctypes.byref(exec_))
        N.check(rc)
        self._exec = exec_.value

    def step(self) -> Tensor:
        from .carrier import CUDA

        if self._exec is None:
            raise RuntimeError("the captured step was released")
        N.check(N.lib.sw_graph_launch(N.c_void_p(self._exec), None))
        self.plan.bump_weight_versions()
        out = Tensor(CUDA(1, dtype=DType.Float32, empty=True, device=self.loss.carrier.device), 0, SCALAR)
        N.check(N.lib.sw_memcpy_d2d(N.c_void_p(_ptr(out)), N.c_void_p(_ptr(self.loss)), 4, None))
        return out

    def close(self) -> None:
        if self._exec is not None:
            N.lib.sw_graph_destroy(N.c_void_p(self._exec))
            self._exec = None
        if self._stream is not None:
            N.lib.sw_stream_destroy(N.c_void_p(self._stream))
            self._stream = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


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

__all__ = ["CapturedTrainStep", "GELU", "MLP", "MSELoss", "MXLinear", "SGD", "gelu", "gelu_grad", "mse_loss",
           "train_step"]
