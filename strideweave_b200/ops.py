"""Operations the CUDA carrier dispatches.

Each class is a ``strideweave`` ``Operation`` (the Python face of
src/strideweave/core/native/_operation.hpp:44-242): ``_forward`` resolves the
shared operation plan and the carrier's capability before allocating anything
(the reference's CPP001 rule), lowers the operand layouts to flat leaf plans
and enqueues one kernel through the C ABI; ``backward`` returns the gradients
in the injective canonical layout of each input, as the CPU carrier does
(src/strideweave/carriers/cpu/native/_cpu_carrier.hpp:711-717).

Layout views (rearrange, permute, reshape, ...) are the reference's own
zero-copy shared operations; the CUDA carrier returns fresh instances of them.
"""

from __future__ import annotations

from typing import Any

from . import _native as N
from . import kernels
from ._host import (
    DType,
    Operation,
    Tensor,
    UnsupportedOperationPlan,
    require_capability,
    resolve_operation_plan,
)
from .layout_plan import canonical_layout, injective_layout_for, mode_leaves, mode_size, single_stride, swizzle_stages


def _cuda_tensor(value: Any, name: str) -> Tensor:
    from .carrier import CUDA

    if not isinstance(value, Tensor):
        raise TypeError(f"{name} must be a Tensor")
    value._require_single_subtensor("CUDA operation")
    if not isinstance(value.carrier, CUDA):
        raise TypeError(f"{name} must be backed by a CUDA carrier")
    if value.carrier.is_released():
        raise RuntimeError(f"{name} carrier is released")
    return value


def _two_mode(value: Any, name: str) -> Tensor:
    t = _cuda_tensor(value, name)
    if len(t.layout) != 2:
        raise ValueError(f"{name} must have a two-mode layout")
    return t


def _new_result(like: Any, layout: Any, dtype: Any, *, zero: bool = False) -> Tensor:
    from .carrier import CUDA

    carrier = CUDA(layout.cosize, dtype=dtype, empty=not zero, device=like.carrier.device)
    return Tensor(carrier, 0, layout)


class CudaOperation(Operation):
    """Common base: the executing carrier class for plan checks."""

    @staticmethod
    def _carrier_class() -> type:
        from .carrier import CUDA

        return CUDA


# ---- reductions -----------------------------------------------------------------


class CudaReduction(CudaOperation):
    """reduce_sum / reduce_max / argmax over mode 1 of a two-mode tensor.

    Replaces CpuReduceSumOperation (src/strideweave/carriers/cpu/native/ops/
    reduce_sum.cpp:30-118) and CpuFloatReductionOperation<Kind>
    (src/strideweave/carriers/cpu/native/_cpu_reduction.hpp:47-196).
    """

    kind = ""

    def _forward(self, tensor: Any) -> Tensor:
        tensor = _two_mode(tensor, "tensor")
        layout = tensor.layout
        n = mode_size(layout, 0)
        m = mode_size(layout, 1)
        if m <= 0 and self.kind != "reduce_sum":
            raise ValueError("reduction fibers must be non-empty")
        output_layout = canonical_layout(layout.shape.top_level[0])
        self.ctx["output_layout"] = output_layout
        plan = resolve_operation_plan(self.kind, tensor.carrier.dtype(), options=self._execution_options)
        require_capability(self._carrier_class(), plan)
        result = _new_result(tensor, output_layout, plan.output)
        # the widened plan (accumulator_dtype=Float64) sums in binary64
        kind = "reduce_sum_f64" if self.kind == "reduce_sum" and plan.accumulator_dtype is DType.Float64 else self.kind
        if n:
            kernels.reduce_f32(kind, tensor.carrier.data_ptr, tensor.carrier.size(), tensor.offset,
                               mode_leaves(layout, 0), mode_leaves(layout, 1), result.carrier.data_ptr,
                               swizzle=swizzle_stages(tensor.carrier))
        return result

    def backward(self, gradient: Any) -> tuple[Any, ...]:
        if self.kind == "argmax":
            return ()
        (tensor,) = self.inputs()
        gradient = _cuda_tensor(gradient, "gradient")
        if gradient.layout != self.ctx["output_layout"]:
            raise ValueError("Tensor layouts must match")
        grad_layout = injective_layout_for(tensor.layout)
        result = _new_result(tensor, grad_layout, DType.Float32)
        kernels.reduce_backward_f32(
            self.kind, tensor.carrier.data_ptr if self.kind == "reduce_max" else 0, tensor.carrier.size(),
            tensor.offset, mode_leaves(tensor.layout, 0), mode_leaves(tensor.layout, 1),
            swizzle_stages(tensor.carrier), gradient.carrier.data_ptr + 4 * gradient.offset,
            result.carrier.data_ptr, mode_leaves(grad_layout, 0), mode_leaves(grad_layout, 1),
            result.carrier.size())
        return (result,)


class CudaReduceSum(CudaReduction):
    kind = "reduce_sum"


class CudaReduceMax(CudaReduction):
    kind = "reduce_max"


class CudaArgmax(CudaReduction):
    kind = "argmax"


# ---- Float32 contraction ----------------------------------------------------------


def _strided(t: Tensor) -> tuple[int, int, int, Any]:
    """(address, stride of mode 0, stride of mode 1, keep-alive) of a Float32
    CUDA matrix; views that do not walk memory with one stride per mode (or
    that sit behind a swizzle) are first gathered into a row-major copy."""
    from .carrier import CUDA

    s0 = single_stride(mode_leaves(t.layout, 0))
    s1 = single_stride(mode_leaves(t.layout, 1))
    if s0 is not None and s1 is not None and not swizzle_stages(t.carrier):
        return t.carrier.data_ptr + 4 * t.offset, s0[1], s1[1], None
    n0, n1 = mode_size(t.layout, 0), mode_size(t.layout, 1)
    tmp = CUDA(max(n0 * n1, 1), dtype=DType.Float32, empty=True, device=t.carrier.device)
    kernels.copy_view_f32(t.carrier.data_ptr, t.carrier.size(), t.offset, mode_leaves(t.layout, 0),
                          mode_leaves(t.layout, 1), tmp.data_ptr, tmp.size(), 0, [(n0, n1)], [(n1, 1)],
                          swizzle=swizzle_stages(t.carrier))
    return tmp.data_ptr, n1, 1, tmp


def _output(layout: Any, like: Tensor) -> tuple[Tensor, int, int, Any]:
    """A fresh Float32 result placed by `layout` and the (address, strides) a
    kernel writes; hierarchical placements are written through a row-major
    staging copy that `_finish` scatters."""
    from .carrier import CUDA

    result = _new_result(like, layout, DType.Float32)
    s0 = single_stride(mode_leaves(layout, 0))
    s1 = single_stride(mode_leaves(layout, 1))
    if s0 is not None and s1 is not None:
        return result, result.carrier.data_ptr, s0[1], s1[1], None
    n0, n1 = mode_size(layout, 0), mode_size(layout, 1)
    tmp = CUDA(max(n0 * n1, 1), dtype=DType.Float32, empty=True, device=like.carrier.device)
    return result, tmp.data_ptr, n1, 1, tmp


def _finish(result: Tensor, staging: Any) -> Tensor:
    if staging is not None:
        lay = result.layout
        n0, n1 = mode_size(lay, 0), mode_size(lay, 1)
        kernels.copy_view_f32(staging.data_ptr, staging.size(), 0, [(n0, n1)], [(n1, 1)], result.carrier.data_ptr,
                              result.carrier.size(), result.offset, mode_leaves(lay, 0), mode_leaves(lay, 1))
    return result


class CudaMatmul(CudaOperation):
    """Float32 contraction out[i, j] = sum_k lhs[i, k] rhs[j, k].

    Replaces CpuMatmulOperation (src/strideweave/carriers/cpu/native/ops/
    matmul.cpp:45-191): the same BINARY32 / FLOATING / Float32 plan, the result
    in the canonical column-major layout of (lhs mode 0, rhs mode 0).
    """

    def _forward(self, lhs: Any, rhs: Any) -> Tensor:
        lhs = _two_mode(lhs, "lhs")
        rhs = _two_mode(rhs, "rhs")
        if type(lhs.carrier) is not type(rhs.carrier):
            raise TypeError("Tensor backing carriers must match")
        M, K = mode_size(lhs.layout, 0), mode_size(lhs.layout, 1)
        Nn, K2 = mode_size(rhs.layout, 0), mode_size(rhs.layout, 1)
        if K != K2:
            raise ValueError("Matmul inner dimensions must match")
        output_layout = canonical_layout(lhs.layout.shape.top_level[0], rhs.layout.shape.top_level[0])
        self.ctx["output_layout"] = output_layout
        plan = resolve_operation_plan("matmul", lhs.carrier.dtype(), rhs.carrier.dtype(),
                                      options=self._execution_options)
        require_capability(self._carrier_class(), plan)
        # the widened plan sums the binary32 products in binary64; the backward
        # contracts the same terms and keeps the forward's accumulator
        # (tests/test_cpu_plan.py:193 pins this for the CPU carrier)
        self.ctx["acc64"] = plan.accumulator_dtype is DType.Float64
        a, sam, sak, _ka = _strided(lhs)
        b, sbn, sbk, _kb = _strided(rhs)
        result = _new_result(lhs, output_layout, DType.Float32)
        kernels.matmul_f32(a, sam, sak, b, sbn, sbk, result.carrier.data_ptr, 1, M, M, Nn, K, acc64=self.ctx["acc64"])
        return result

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        lhs, rhs = self.inputs()
        gradient = _cuda_tensor(gradient, "gradient")
        if gradient.layout != self.ctx["output_layout"]:
            raise ValueError("Tensor layouts must match")
        M, K = mode_size(lhs.layout, 0), mode_size(lhs.layout, 1)
        Nn = mode_size(rhs.layout, 0)
        a, sam, sak, _ka = _strided(lhs)
        b, sbn, sbk, _kb = _strided(rhs)
        g, sgm, sgn, _kg = _strided(gradient)
        dl, dlp, dlm, dlk, dls = _output(injective_layout_for(lhs.layout), lhs)
        dr, drp, drn, drk, drs = _output(injective_layout_for(rhs.layout), rhs)
        acc64 = bool(self.ctx.get("acc64", False))
        # dlhs[m, k] = sum_n g[m, n] rhs[n, k]  (rhs viewed as [k, n])
        kernels.matmul_f32(g, sgm, sgn, b, sbk, sbn, dlp, dlm, dlk, M, K, Nn, acc64=acc64)
        # drhs[n, k] = sum_m g[m, n] lhs[m, k]  (g viewed as [n, m], lhs as [k, m])
        kernels.matmul_f32(g, sgn, sgm, a, sak, sam, drp, drn, drk, Nn, K, M, acc64=acc64)
        return (_finish(dl, dls), _finish(dr, drs))


# ---- elementwise product (the union step of batched einsum) ------------------------


def _map(op: int, a: Tensor, b: Tensor | None, out: Tensor, scalar: float = 0.0, name: str = "elementwise") -> None:
    """out = a (op) b, or (op)(a, scalar), elementwise over views sharing one
    shape tree (sw_map_f32)."""
    import ctypes

    from . import _native as N
    from .layout_plan import all_leaves

    views = [(a, "lhs"), (out, "output")] + ([(b, "rhs")] if b is not None else [])
    for t, role in views:
        if t.carrier.swizzle is not None:
            raise NotImplementedError(f"{role}: swizzled carriers are not supported by {name}")
    la, lo = all_leaves(a.layout), all_leaves(out.layout)
    lb = all_leaves(b.layout) if b is not None else la
    if not (len(la) == len(lb) == len(lo)) or any(x[0] != y[0] or x[0] != z[0] for x, y, z in zip(la, lb, lo)):
        raise ValueError(f"{name} operands must share one shape tree")
    keep = [i for i, (e, _) in enumerate(lo) if e != 1]
    rank = len(keep)
    arr = ctypes.c_int64 * max(rank, 1)
    shape = arr(*[lo[i][0] for i in keep])
    sa, sb, so = (arr(*[leaves[i][1] for i in keep]) for leaves in (la, lb, lo))
    bt = b if b is not None else a
    N.check(N.lib.sw_map_f32(
        op, rank, shape,
        N.c_void_p(a.carrier.data_ptr), a.offset, sa, a.carrier.size(),
        N.c_void_p(bt.carrier.data_ptr), bt.offset, sb, bt.carrier.size(),
        N.c_void_p(out.carrier.data_ptr), out.offset, so, out.carrier.size(), float(scalar), None))


def _binary_mul(a: Tensor, b: Tensor, out: Tensor) -> None:
    """out = a * b elementwise over three views sharing one shape tree."""
    from . import _native as N

    _map(N.SW_MAP_MUL, a, b, out, name="elementwise_mul")


class CudaElementwiseMul(CudaOperation):
    """Float32 elementwise product of two broadcast-compatible tensors.

    Replaces CpuElementwiseMulOperation (src/strideweave/carriers/cpu/native/
    ops/elementwise_mul.cpp:8-48): the operands are aligned by the reference's
    own ``_align_binary_operands`` (differentiable broadcast views,
    src/strideweave/carriers/operation_helpers.py:129-185), the result takes
    the canonical layout of the common shape and each product is rounded to
    binary32; the gradients are g * rhs and g * lhs in the injective canonical
    layout of each aligned operand.  With this the reference's batched
    ``einsum`` (union product, then reduce_sum) runs on the device unchanged.
    """

    def _forward(self, lhs: Any, rhs: Any) -> Tensor:
        from strideweave.carriers.operation_helpers import _align_binary_operands

        lhs = _cuda_tensor(lhs, "lhs")
        rhs = _cuda_tensor(rhs, "rhs")
        if type(lhs.carrier) is not type(rhs.carrier):
            raise TypeError("Tensor backing carriers must match")
        lhs, rhs, result_layout = _align_binary_operands(lhs, rhs)
        if len(self.inputs()) != 0:
            self.store_inputs(lhs, rhs)  # the gradient flows through the broadcast views
        plan = resolve_operation_plan("elementwise_mul", lhs.carrier.dtype(), rhs.carrier.dtype(),
                                      options=self._execution_options)
        require_capability(self._carrier_class(), plan)
        result = _new_result(lhs, result_layout, DType.Float32)
        _binary_mul(lhs, rhs, result)
        return result

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        lhs, rhs = self.inputs()
        gradient = _cuda_tensor(gradient, "gradient")
        if gradient.layout.shape != lhs.layout.shape:
            raise ValueError("Tensor shapes must match")
        dl = _new_result(lhs, injective_layout_for(lhs.layout), DType.Float32)
        dr = _new_result(rhs, injective_layout_for(rhs.layout), DType.Float32)
        _binary_mul(gradient, rhs, dl)
        _binary_mul(gradient, lhs, dr)
        return (dl, dr)


# ---- the elementwise arithmetic of the reference's nn modules ---------------------
#
# A Linear's bias add, an MSE loss's difference, square and mean scale
# (src/strideweave/nn/modules.py:40-176, friendly/ops.py:52) and their
# gradients, so the reference's own modules train on CUDA-carrier tensors.


def _copy(src: Tensor, dst: Tensor) -> None:
    """dst = src value for value (NaN payloads kept) over one shape tree."""
    from . import kernels
    from .layout_plan import all_leaves

    ls, ld = all_leaves(src.layout), all_leaves(dst.layout)
    if len(ls) > N.SW_MAX_LEAVES:
        raise NotImplementedError(f"more than {N.SW_MAX_LEAVES} leaves")
    kernels.copy_view_f32(src.carrier.data_ptr, src.carrier.size(), src.offset, ls or [(1, 0)], [(1, 0)],
                          dst.carrier.data_ptr, dst.carrier.size(), dst.offset, ld or [(1, 0)], [(1, 0)],
                          swizzle=swizzle_stages(src.carrier))


def _gradient_like(t: Tensor, gradient: Any) -> tuple[Tensor, Tensor]:
    gradient = _cuda_tensor(gradient, "gradient")
    if gradient.layout.shape != t.layout.shape:
        raise ValueError("Tensor shapes must match")
    return gradient, _new_result(t, injective_layout_for(t.layout), DType.Float32)


class _CudaBinaryArithmetic(CudaOperation):
    """Tensor (op) tensor, as the reference's cpu_binary_elementwise_forward
    (src/strideweave/carriers/cpu/native/_cpu_binary.hpp:85-130): operands
    aligned by ``_align_binary_operands`` (differentiable broadcast views),
    the canonical layout of the common shape, one binary32 operation per
    element."""

    _name = ""
    _op = -1

    def _forward(self, lhs: Any, rhs: Any) -> Tensor:
        from strideweave.carriers.operation_helpers import _align_binary_operands

        lhs = _cuda_tensor(lhs, "lhs")
        rhs = _cuda_tensor(rhs, "rhs")
        if type(lhs.carrier) is not type(rhs.carrier):
            raise TypeError("Tensor backing carriers must match")
        lhs, rhs, result_layout = _align_binary_operands(lhs, rhs)
        if len(self.inputs()) != 0:
            self.store_inputs(lhs, rhs)  # the gradient flows through the broadcast views
        plan = resolve_operation_plan(self._name, lhs.carrier.dtype(), rhs.carrier.dtype(),
                                      options=self._execution_options)
        require_capability(self._carrier_class(), plan)
        result = _new_result(lhs, result_layout, DType.Float32)
        _map(self._op, lhs, rhs, result, name=self._name)
        return result


class CudaAdd(_CudaBinaryArithmetic):
    """lhs + rhs (CpuAddOperation, ops/add.cpp); both gradients are g."""

    _name, _op = "add", N.SW_MAP_ADD

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        lhs, rhs = self.inputs()
        g, dl = _gradient_like(lhs, gradient)
        _, dr = _gradient_like(rhs, gradient)
        _copy(g, dl)
        _copy(g, dr)
        return (dl, dr)


class CudaSub(_CudaBinaryArithmetic):
    """lhs - rhs (CpuSubOperation, ops/sub.cpp:8-24); gradients g and -g."""

    _name, _op = "sub", N.SW_MAP_SUB

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        lhs, rhs = self.inputs()
        g, dl = _gradient_like(lhs, gradient)
        _, dr = _gradient_like(rhs, gradient)
        _copy(g, dl)
        _map(N.SW_MAP_SCALE, g, None, dr, -1.0, name="sub")
        return (dl, dr)


class CudaMul(CudaOperation):
    """mul: a tensor times a weak scalar (CpuScalarMulOperation,
    ops/scalar_mul.cpp), result and gradient g * scalar in the injective
    canonical layout of the tensor; tensor times tensor as elementwise_mul."""

    def _forward(self, tensor: Any, other: Any) -> Tensor:
        if isinstance(other, Tensor):
            self.ctx["tensor_rhs"] = True
            from strideweave.carriers.operation_helpers import _align_binary_operands

            lhs, rhs = _cuda_tensor(tensor, "lhs"), _cuda_tensor(other, "rhs")
            lhs, rhs, result_layout = _align_binary_operands(lhs, rhs)
            if len(self.inputs()) != 0:
                self.store_inputs(lhs, rhs)
            require_capability(self._carrier_class(), resolve_operation_plan(
                "mul", lhs.carrier.dtype(), rhs.carrier.dtype(), options=self._execution_options))
            result = _new_result(lhs, result_layout, DType.Float32)
            _map(N.SW_MAP_MUL, lhs, rhs, result, name="mul")
            return result
        tensor = _cuda_tensor(tensor, "tensor")
        require_capability(self._carrier_class(), resolve_operation_plan(
            "mul", tensor.carrier.dtype(), other, options=self._execution_options))
        scalar = float(other)
        self.ctx["scalar"] = scalar
        result = _new_result(tensor, injective_layout_for(tensor.layout), DType.Float32)
        _map(N.SW_MAP_SCALE, tensor, None, result, scalar, name="mul")
        return result

    def backward(self, gradient: Any) -> tuple[Any, ...]:
        inputs = self.inputs()
        if self.ctx.get("tensor_rhs"):
            lhs, rhs = inputs
            g, dl = _gradient_like(lhs, gradient)
            _, dr = _gradient_like(rhs, gradient)
            _map(N.SW_MAP_MUL, g, rhs, dl, name="mul")
            _map(N.SW_MAP_MUL, g, lhs, dr, name="mul")
            return (dl, dr)
        (tensor,) = inputs[:1]
        g, dt = _gradient_like(tensor, gradient)
        _map(N.SW_MAP_SCALE, g, None, dt, self.ctx["scalar"], name="mul")
        return (dt,)


class CudaPow(CudaOperation):
    """A tensor raised to a weak-scalar exponent (CpuPowOperation,
    ops/pow.cpp:66-101 forward, :160-175 gradient g * p * x^(p - 1)), in the
    injective canonical layout of the tensor."""

    def _forward(self, tensor: Any, exponent: Any) -> Tensor:
        if isinstance(exponent, Tensor):
            raise NotImplementedError("CUDA pow takes a scalar exponent")
        tensor = _cuda_tensor(tensor, "tensor")
        require_capability(self._carrier_class(), resolve_operation_plan(
            "pow", tensor.carrier.dtype(), exponent, options=self._execution_options))
        p = float(exponent)
        self.ctx["exponent"] = p
        result = _new_result(tensor, injective_layout_for(tensor.layout), DType.Float32)
        _map(N.SW_MAP_POW, tensor, None, result, p, name="pow")
        return result

    def backward(self, gradient: Any) -> tuple[Any]:
        (tensor,) = self.inputs()[:1]
        g, dt = _gradient_like(tensor, gradient)
        _map(N.SW_MAP_POW_GRAD, g, tensor, dt, self.ctx["exponent"], name="pow")
        return (dt,)


class CudaNeg(CudaOperation):
    """-tensor (ops/neg.cpp); gradient -g."""

    def _forward(self, tensor: Any) -> Tensor:
        tensor = _cuda_tensor(tensor, "tensor")
        require_capability(self._carrier_class(), resolve_operation_plan(
            "neg", tensor.carrier.dtype(), options=self._execution_options))
        result = _new_result(tensor, injective_layout_for(tensor.layout), DType.Float32)
        _map(N.SW_MAP_SCALE, tensor, None, result, -1.0, name="neg")
        return result

    def backward(self, gradient: Any) -> tuple[Any]:
        (tensor,) = self.inputs()[:1]
        g, dt = _gradient_like(tensor, gradient)
        _map(N.SW_MAP_SCALE, g, None, dt, -1.0, name="neg")
        return (dt,)


# ---- dispatch table ----------------------------------------------------------------


def _shared(name: str) -> Any:
    from strideweave.carriers import shared_ops
    from strideweave.carriers.generic.as_strided_ops import GenericAsStridedOperation

    table = {
        "broadcast_to": shared_ops.BroadcastOperation,
        "permute": shared_ops.PermuteOperation,
        "rearrange": shared_ops.RearrangeOperation,
        "reshape": shared_ops.ReshapeOperation,
        "squeeze": shared_ops.SqueezeOperation,
        "unsqueeze": shared_ops.UnsqueezeOperation,
        "view": shared_ops.GenericViewOperation,
        "as_strided": GenericAsStridedOperation,
    }
    return table.get(name)


_OPS = {
    "reduce_sum": CudaReduceSum,
    "reduce_max": CudaReduceMax,
    "argmax": CudaArgmax,
    "matmul": CudaMatmul,
    "elementwise_mul": CudaElementwiseMul,
    "add": CudaAdd,
    "sub": CudaSub,
    "mul": CudaMul,
    "pow": CudaPow,
    "neg": CudaNeg,
}


def make_operation(name: str) -> Any:
    """A fresh operation instance for ``name`` (``Carrier._dispatch_op``)."""
    if name in _OPS:
        return _OPS[name]()
    from .mx import MX_OPERATIONS
    from .nn import NN_OPERATIONS

    if name in MX_OPERATIONS:
        return MX_OPERATIONS[name]()
    if name in NN_OPERATIONS:
        return NN_OPERATIONS[name]()
    shared = _shared(name)
    if shared is not None:
        return shared()
    raise NotImplementedError(f"CUDA carrier does not support operation '{name}'")


def declared_plans() -> list[Any]:
    """The plan shapes this carrier executes (declared at import)."""
    f32 = DType.Float32
    return [
        resolve_operation_plan("reduce_sum", f32),
        resolve_operation_plan("reduce_sum", f32, accumulator_dtype=DType.Float64),
        resolve_operation_plan("reduce_max", f32),
        resolve_operation_plan("argmax", f32),
        resolve_operation_plan("matmul", f32, f32),
        resolve_operation_plan("matmul", f32, f32, accumulator_dtype=DType.Float64),
        resolve_operation_plan("gelu", f32),
        resolve_operation_plan("elementwise_mul", f32, f32),
        resolve_operation_plan("add", f32, f32),
        resolve_operation_plan("sub", f32, f32),
        resolve_operation_plan("mul", f32, f32),
        resolve_operation_plan("mul", f32, 1.0),
        resolve_operation_plan("pow", f32, 2.0),
        resolve_operation_plan("neg", f32),
    ]


__all__ = ["CudaAdd", "CudaArgmax", "CudaElementwiseMul", "CudaMatmul", "CudaMul", "CudaNeg", "CudaPow",
           "CudaReduceMax", "CudaReduceSum", "CudaSub", "UnsupportedOperationPlan", "declared_plans",
           "make_operation"]
