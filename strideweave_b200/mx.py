"""MX (OCP Microscaling v1.0) tensors on the CUDA carrier.

An MX tensor is the reference's multi-sub-tensor representation
(src/strideweave/core/_representation.py:38-173) of a block-scaled dtype
(``DType.MXFP8_E4M3`` or ``DType.MXFP4``, src/strideweave/carriers/_dtype/
builtins.py:39-52) with two planes on CUDA carriers:

  level 0, payload  ``L0 = ((rows), (32, K/32)) : ((ld), (1, 32))`` - one
           E4M3 byte or one E2M1 nibble per element, rows of K contiguous;
  level 1, scales   one E8M0 byte per 32-element block.  When rows % 128 == 0
           and K % 128 == 0 the plane uses the tensor-core atom placement
           ``((32, 4, rows/128), (4, K/128)) : ((16, 4, 512*K/128), (1, 512))``
           that tcgen05.cp copies straight into tensor memory; otherwise a
           row-major ``(rows, K/32) : (K/32, 1)`` placement;
  adjacent S0 = ((rows), (32, K/32)) : ((1), (0, rows)), which maps payload
           coordinate (r, (k0, k1)) to scale ordinal r + rows * k1, i.e. 32
           payload elements per scale (the LevelExtent(0, 32) rule).

The contraction kernel reads both planes exactly where this representation
places them.  MX dtypes are not differentiable in the reference
(src/strideweave/core/native/_operation.hpp:30-33); the differentiable path is
``mx_linear``, which takes Float32 operands and quantises inside its forward
and backward (re-quantising along each contraction's own K).
"""

from __future__ import annotations

from typing import Any

from . import _native as N
from . import kernels
from ._host import BFloat16, DType, Layout, Operation, Shape, Stride, Subtensor, Tensor, TensorRepresentation
from .layout_plan import mode_leaves, mode_size, single_stride, swizzle_stages

FORMATS = {
    "MXFP8_E4M3": (DType.MXFP8_E4M3, DType.E4M3, N.SW_MX_E4M3),
    "MXFP4": (DType.MXFP4, DType.E2M1, N.SW_MX_E2M1),
}
_BY_DTYPE = {v[0]: (k, v[1], v[2]) for k, v in FORMATS.items()}


def payload_layout(rows: int, K: int, ld: int | None = None) -> Layout:
    return Layout(Shape([rows, [32, K // 32]]), Stride([K if ld is None else ld, [1, 32]]))


def scale_layout_tc128(rows: int, kblocks: int) -> Layout:
    katoms = kblocks // 4
    return Layout(Shape([[32, 4, rows // 128], [4, katoms]]), Stride([[16, 4, 512 * katoms], [1, 512]]))


def scale_layout_rowmajor(rows: int, kblocks: int) -> Layout:
    return Layout(Shape([rows, kblocks]), Stride([kblocks, 1]))


def adjacent_layout(rows: int, kblocks: int) -> Layout:
    return Layout(Shape([rows, [32, kblocks]]), Stride([1, [0, rows]]))


def uses_tc128(rows: int, kblocks: int) -> bool:
    return rows % 128 == 0 and kblocks % 4 == 0


def _f32_operand(t: Any, name: str) -> tuple[int, int, int, int, int]:
    """(address, rows, cols, row stride, col stride) of a Float32 CUDA matrix."""
    from .carrier import CUDA

    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a Tensor")
    t._require_single_subtensor("MX quantisation")
    if not isinstance(t.carrier, CUDA) or t.carrier.dtype() is not DType.Float32:
        raise TypeError(f"{name} must be a Float32 tensor on a CUDA carrier")
    if len(t.layout) != 2:
        raise ValueError(f"{name} must have a two-mode layout")
    if swizzle_stages(t.carrier):
        raise NotImplementedError(f"{name}: quantising a swizzled carrier is not supported")
    r = single_stride(mode_leaves(t.layout, 0))
    c = single_stride(mode_leaves(t.layout, 1))
    if r is None or c is None:
        raise NotImplementedError(f"{name}: each mode must walk memory with a single stride")
    return t.carrier.data_ptr + 4 * t.offset, r[0], c[0], r[1], c[1]


def _f32_view(t: Any, name: str) -> tuple[Any, list[tuple[int, int]], list[tuple[int, int]], list]:
    """(carrier, row leaves, column leaves, swizzle stages) of a two-mode
    Float32 CUDA tensor, leaves first-fastest with unit leaves dropped."""
    from .carrier import CUDA
    from .layout_plan import coalesce

    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a Tensor")
    t._require_single_subtensor("MX quantisation")
    if not isinstance(t.carrier, CUDA) or t.carrier.dtype() is not DType.Float32:
        raise TypeError(f"{name} must be a Float32 tensor on a CUDA carrier")
    if len(t.layout) != 2:
        raise ValueError(f"{name} must have a two-mode layout")
    rows = coalesce(mode_leaves(t.layout, 0)) or [(1, 0)]
    cols = coalesce(mode_leaves(t.layout, 1)) or [(1, 0)]
    if len(rows) > N.SW_MAX_LEAVES or len(cols) > N.SW_MAX_LEAVES:
        raise NotImplementedError(f"{name}: more than {N.SW_MAX_LEAVES} leaves in one mode")
    return t.carrier, rows, cols, swizzle_stages(t.carrier)


def quantize(t: Tensor, fmt: str = "MXFP8_E4M3") -> Tensor:
    """Quantise a Float32 CUDA tensor [rows, K] into an MX tensor, blocks of 32
    along mode 1 (the mode a contraction sums over).  Any layout: modes that
    walk memory with one stride each take the strided kernels; hierarchical
    (tiled) modes and swizzled carriers are quantised where they lie through
    the view kernel, the same planes bit for bit."""
    from .carrier import CUDA

    if fmt not in FORMATS:
        raise NotImplementedError(f"no MX kernel for format {fmt!r}")
    mx_dtype, elem_dtype, code = FORMATS[fmt]
    carrier, row_leaves, col_leaves, swz = _f32_view(t, "tensor")
    rows, K = mode_size(t.layout, 0), mode_size(t.layout, 1)
    if K % 32 != 0:
        raise ValueError("MX quantisation needs the blocked mode to be a multiple of 32")
    kblocks = K // 32
    tc = uses_tc128(rows, kblocks)
    payload = CUDA(rows * K, dtype=elem_dtype, empty=True, device=t.carrier.device)
    scale_size = kernels.scale_bytes_tc128(rows, kblocks) if tc else rows * kblocks
    scales = CUDA(scale_size, dtype=DType.E8M0, empty=True, device=t.carrier.device)
    placement = dict(scale_layout=N.SW_SCALES_TC128 if tc else N.SW_SCALES_ROWMAJOR, ld_scales=0 if tc else kblocks)
    r1, c1 = single_stride(row_leaves), single_stride(col_leaves)
    if not swz and r1 is not None and c1 is not None:
        kernels.mx_quantize(code, carrier.data_ptr + 4 * t.offset, rows, K, r1[1], c1[1], payload.data_ptr,
                            kernels.mx_row_bytes(code, K), scales.data_ptr, **placement)
    else:
        kernels.mx_quantize_view(code, carrier.data_ptr, carrier.size(), t.offset, row_leaves, col_leaves,
                                 payload.data_ptr, kernels.mx_row_bytes(code, K), scales.data_ptr, swizzle=swz,
                                 **placement)
    rep = TensorRepresentation(
        mx_dtype,
        (Subtensor(elem_dtype, payload, 0, payload_layout(rows, K)),
         Subtensor(DType.E8M0, scales, 0, scale_layout_tc128(rows, kblocks) if tc else
                   scale_layout_rowmajor(rows, kblocks))),
        (adjacent_layout(rows, kblocks),),
    )
    return Tensor._from_representation(rep)


def dual_geometry(t: Tensor) -> tuple[int, int, int, int, bool] | None:
    """(address, rows, cols, pitch, transposed) of the memory matrix behind a
    Float32 CUDA matrix when ``sw_mx_quantize_dual`` can read it, else None.
    ``transposed`` means the memory rows are the tensor's columns (a
    column-major tensor)."""
    ptr, R, C, sr, sc = _f32_operand(t, "operand")
    if sc == 1 and R > 1:
        rows, cols, ld, transposed = R, C, sr, False
    elif sr == 1:
        rows, cols, ld, transposed = C, R, sc, True
    else:
        return None
    if rows % 32 or cols % 128 or ld % 4 or ptr % 16 or ld < cols:
        return None
    return ptr, rows, cols, ld, transposed


Planes = tuple[Any, Any]  # (payload carrier, scale carrier), TC128 scales, packed rows


def quantize_both(t: Tensor, code: int, *, transform: int = N.SW_XF_NONE, h: Tensor | None = None,
                  need_t: bool = True, need_tT: bool = True) -> tuple[Planes | None, Planes | None] | None:
    """The contraction operands t [R, C] (blocks along C) and t^T [C, R] (blocks
    along R) of S = t, gelu(t) or t * gelu'(h), from one read of t (and h,
    which shares t's layout).  The planes equal those of the elementwise
    kernel followed by two ``quantize`` calls, bit for bit.  Returns None when
    the fused quantiser cannot read t's layout."""
    from .carrier import CUDA

    geo = dual_geometry(t)
    if geo is None:
        return None
    ptr, rows, cols, ld, transposed = geo
    h_ptr = 0
    if transform == N.SW_XF_GELU_GRAD:
        if h is None or h.layout != t.layout:
            return None
        hgeo = dual_geometry(h)
        if hgeo is None:
            return None
        h_ptr = hgeo[0]
    R, C = (cols, rows) if transposed else (rows, cols)
    elem = DType.E4M3 if code == N.SW_MX_E4M3 else DType.E2M1
    dev = t.carrier.device

    def planes(n: int, k: int) -> Planes:
        return (CUDA(n * k, dtype=elem, empty=True, device=dev),
                CUDA(kernels.scale_bytes_tc128(n, k // 32), dtype=DType.E8M0, empty=True, device=dev))

    q_t = planes(R, C) if need_t else None
    q_tT = planes(C, R) if need_tT else None
    row_q, col_q = (q_tT, q_t) if transposed else (q_t, q_tT)
    kernels.mx_quantize_dual(code, transform, ptr, h_ptr, rows, cols, ld,
                             (row_q[0].data_ptr, row_q[1].data_ptr) if row_q else None,
                             (col_q[0].data_ptr, col_q[1].data_ptr) if col_q else None)
    return q_t, q_tT


class MXPlanes:
    """The two planes of a validated MX tensor, lowered for the kernels."""

    def __init__(self, mx: Tensor, name: str = "operand") -> None:
        from .carrier import CUDA

        rep = mx._representation
        if rep.logical_dtype not in _BY_DTYPE:
            raise TypeError(f"{name} must be an MX tensor (MXFP8_E4M3 or MXFP4), not {rep.logical_dtype.name}")
        self.fmt_name, _, self.code = _BY_DTYPE[rep.logical_dtype]
        pay, sc = rep.subtensors
        if not isinstance(pay.carrier, CUDA) or not isinstance(sc.carrier, CUDA):
            raise TypeError(f"{name} planes must live on CUDA carriers")
        self.rows = mode_size(pay.layout, 0)
        self.K = mode_size(pay.layout, 1)
        kblocks = self.K // 32
        self.kblocks = kblocks
        ld = single_stride(mode_leaves(pay.layout, 0))
        if ld is None or pay.layout != payload_layout(self.rows, self.K, ld[1]):
            raise NotImplementedError(f"{name}: payload placement must be rows of K contiguous elements")
        self.ld_elems = ld[1]
        self.payload = pay
        self.scales = sc
        self.tc128 = sc.layout == scale_layout_tc128(self.rows, kblocks) if uses_tc128(self.rows, kblocks) else False
        if not self.tc128 and sc.layout != scale_layout_rowmajor(self.rows, kblocks):
            raise NotImplementedError(f"{name}: unsupported scale placement {sc.layout}")
        if rep.adjacent_layouts[0] != adjacent_layout(self.rows, kblocks):
            raise NotImplementedError(f"{name}: unsupported adjacent layout {rep.adjacent_layouts[0]}")

    @property
    def payload_ptr(self) -> int:
        return self.payload.carrier.data_ptr + (self.payload.offset if self.code == N.SW_MX_E4M3
                                                else self.payload.offset // 2)

    @property
    def ld_bytes(self) -> int:
        return self.ld_elems if self.code == N.SW_MX_E4M3 else self.ld_elems // 2

    @property
    def scales_ptr(self) -> int:
        return self.scales.carrier.data_ptr + self.scales.offset


def _scale_atoms(pl: MXPlanes, dev: int) -> Any:
    """A row-major scale plane rewritten into the tensor-core atom placement,
    as a fresh CUDA carrier (released in stream order after its last use)."""
    from .carrier import CUDA

    tmp = CUDA(kernels.scale_bytes_tc128(pl.rows, pl.kblocks), dtype=DType.E8M0, empty=True, device=dev)
    kernels.mx_scales_to_tc128(pl.scales_ptr, pl.kblocks, pl.rows, pl.kblocks, tmp.data_ptr)
    return tmp


def _scales_ptr(source: Any) -> int:
    return source.scales_ptr if isinstance(source, MXPlanes) else source.data_ptr


def dequantize(mx: Tensor) -> Tensor:
    """Exact Float32 image of an MX tensor, [rows, K] row-major."""
    from .carrier import CUDA

    pl = MXPlanes(mx)
    out = CUDA(pl.rows * pl.K, dtype=DType.Float32, empty=True, device=pl.payload.carrier.device)
    kernels.mx_dequantize(pl.code, pl.payload_ptr, pl.ld_bytes, pl.scales_ptr, pl.rows, pl.K, out.data_ptr, pl.K,
                          scale_layout=N.SW_SCALES_TC128 if pl.tc128 else N.SW_SCALES_ROWMAJOR,
                          ld_scales=0 if pl.tc128 else pl.kblocks)
    return Tensor(out, 0, Layout(Shape([pl.rows, pl.K]), Stride([pl.K, 1])))


class MxMatmul(Operation):
    """Block-scaled contraction out[m, n] = sum_k A[m, k] B[n, k] of two MX
    tensors (both blocked along their mode 1), fp32 accumulation, Float32 or
    BFloat16 result in the canonical column-major layout - the reference's
    matmul contract (src/strideweave/carriers/cpu/native/ops/matmul.cpp:45-113)
    extended to MX operands, which the reference policy refuses
    (src/strideweave/carriers/operation_policy.py:1407-1440).

    MX tensors have two sub-tensors, which the native ``Operation.forward``
    preflight refuses for everything but layout views
    (src/strideweave/core/native/_operation.hpp:214-233); this operation
    overrides ``forward`` the way the reference's composite adapters do
    (src/strideweave/carriers/evictable/ops.py:66-90).  MX dtypes are not
    differentiable, so no autograd node is attached.
    """

    def forward(self, a: Any, b: Any, *, out_dtype: Any = None) -> Tensor:  # type: ignore[override]
        return self._forward(a, b, out_dtype=out_dtype)

    def _forward(self, a: Any, b: Any, *, out_dtype: Any = None) -> Tensor:
        from .carrier import CUDA
        from .layout_plan import canonical_layout

        pa, pb = MXPlanes(a, "lhs"), MXPlanes(b, "rhs")
        if pa.code != pb.code:
            raise NotImplementedError("mixed MX operand formats are not supported")
        if pa.K != pb.K:
            raise ValueError("Matmul inner dimensions must match")
        out_dtype = DType.Float32 if out_dtype is None else out_dtype
        if out_dtype is not DType.Float32 and out_dtype is not BFloat16:
            raise NotImplementedError("MX contraction produces Float32 or BFloat16")
        M, Nn, K = pa.rows, pb.rows, pa.K
        layout = canonical_layout(a.layout.shape.top_level[0], b.layout.shape.top_level[0])
        self.ctx["output_layout"] = layout
        dev = pa.payload.carrier.device
        out = CUDA(M * Nn, dtype=out_dtype, empty=True, device=dev)
        # Planes whose rows or blocks are not whole 128 x 4 atoms keep row-major
        # scales; the kernel reads the atom placement, so those are rewritten
        # into it first (1/32 of the payload bytes; released in stream order).
        atoms = [pl if pl.tc128 else _scale_atoms(pl, dev) for pl in (pa, pb)]
        kernels.mx_gemm(pa.code, pa.payload_ptr, pa.ld_bytes, _scales_ptr(atoms[0]), pb.payload_ptr, pb.ld_bytes,
                        _scales_ptr(atoms[1]), out.data_ptr, M, Nn, K, out_bf16=out_dtype is BFloat16, ldc_m=1,
                        ldc_n=M)
        return Tensor(out, 0, layout)

    def backward(self, gradient: Any) -> tuple[Any, ...]:
        raise RuntimeError("MX tensors are not differentiable; use mx_linear for a differentiable contraction")


def _quantize_view(ptr: int, rows: int, K: int, ldr: int, ldc: int, code: int, device: int):
    """Quantise a strided Float32 matrix into fresh planes (tensor-core placement)."""
    from .carrier import CUDA

    kblocks = K // 32
    payload = CUDA(rows * K, dtype=DType.E4M3 if code == N.SW_MX_E4M3 else DType.E2M1, empty=True, device=device)
    scales = CUDA(kernels.scale_bytes_tc128(rows, kblocks), dtype=DType.E8M0, empty=True, device=device)
    kernels.mx_quantize(code, ptr, rows, K, ldr, ldc, payload.data_ptr, kernels.mx_row_bytes(code, K),
                        scales.data_ptr)
    return payload, scales


def linear_forward(x: Tensor, w: Tensor, fmt: str) -> Tensor:
    """y = x . w^T with x [B, in], w [out, in] Float32 on CUDA, both quantised
    along `in`; y [B, out] in the canonical column-major layout."""
    from .carrier import CUDA
    from .layout_plan import canonical_layout

    code = FORMATS[fmt][2]
    xp, B, IN, xr, xc = _f32_operand(x, "x")
    wp, OUT, IN2, wr, wc = _f32_operand(w, "weight")
    if IN != IN2:
        raise ValueError("Matmul inner dimensions must match")
    # each extent is the contracted (blocked) one of some contraction of the
    # forward or the backward: whole 32-element MX blocks
    for name, n in (("batch", B), ("out", OUT), ("in", IN)):
        if n % 32 != 0:
            raise NotImplementedError(f"mx_linear needs {name} extent {n} to be a multiple of 32")
    dev = x.carrier.device
    qx = _quantize_view(xp, B, IN, xr, xc, code, dev)
    qw = _quantize_view(wp, OUT, IN, wr, wc, code, dev)
    layout = canonical_layout(x.layout.shape.top_level[0], w.layout.shape.top_level[0])
    out = CUDA(B * OUT, dtype=DType.Float32, empty=True, device=dev)
    rb = kernels.mx_row_bytes(code, IN)
    kernels.mx_gemm(code, qx[0].data_ptr, rb, qx[1].data_ptr, qw[0].data_ptr, rb, qw[1].data_ptr, out.data_ptr,
                    B, OUT, IN, ldc_m=1, ldc_n=B)
    return Tensor(out, 0, layout)


def linear_backward(x: Tensor, w: Tensor, gradient: Tensor, fmt: str, *, need_dx: bool = True
                    ) -> tuple[Tensor | None, Tensor]:
    """(dx, dw) of y = x . w^T: dx = g . w (K = out), dw = g^T . x (K = batch),
    each operand re-quantised along its contraction's K; gradients in the
    injective canonical layouts of x and w."""
    from .carrier import CUDA
    from .layout_plan import injective_layout_for

    code = FORMATS[fmt][2]
    gp, B, OUT, gr_, gc = _f32_operand(gradient, "gradient")
    xp, _, IN, xr, xc = _f32_operand(x, "x")
    wp, _, _, wr, wc = _f32_operand(w, "weight")
    dev = x.carrier.device
    dx = None
    if need_dx:
        # dx[b, i] = sum_o g[b, o] w[o, i]: operands g [B, OUT] and w^T [IN, OUT]
        qg = _quantize_view(gp, B, OUT, gr_, gc, code, dev)
        qwt = _quantize_view(wp, IN, OUT, wc, wr, code, dev)
        dx_layout = injective_layout_for(x.layout)
        dxc = CUDA(dx_layout.cosize, dtype=DType.Float32, empty=True, device=dev)
        (_, s0), (_, s1) = single_stride(mode_leaves(dx_layout, 0)), single_stride(mode_leaves(dx_layout, 1))
        rb = kernels.mx_row_bytes(code, OUT)
        kernels.mx_gemm(code, qg[0].data_ptr, rb, qg[1].data_ptr, qwt[0].data_ptr, rb, qwt[1].data_ptr, dxc.data_ptr,
                        B, IN, OUT, ldc_m=s0, ldc_n=s1)
        dx = Tensor(dxc, 0, dx_layout)
    # dw[o, i] = sum_b g[b, o] x[b, i]: operands g^T [OUT, B] and x^T [IN, B]
    qgt = _quantize_view(gp, OUT, B, gc, gr_, code, dev)
    qxt = _quantize_view(xp, IN, B, xc, xr, code, dev)
    dw_layout = injective_layout_for(w.layout)
    dwc = CUDA(dw_layout.cosize, dtype=DType.Float32, empty=True, device=dev)
    (_, s0), (_, s1) = single_stride(mode_leaves(dw_layout, 0)), single_stride(mode_leaves(dw_layout, 1))
    rb = kernels.mx_row_bytes(code, B)
    kernels.mx_gemm(code, qgt[0].data_ptr, rb, qgt[1].data_ptr, qxt[0].data_ptr, rb, qxt[1].data_ptr, dwc.data_ptr,
                    OUT, IN, B, ldc_m=s0, ldc_n=s1)
    return dx, Tensor(dwc, 0, dw_layout)


class MxLinear(Operation):
    """Differentiable MX contraction y[b, o] = sum_i x[b, i] w[o, i] (the
    ``nn.Linear`` contraction, src/strideweave/nn/modules.py:40-127, with
    weight [out, in]).  Float32 in and out; see linear_forward and
    linear_backward for the quantisation of each contraction.
    """

    fmt = "MXFP8_E4M3"

    def _forward(self, x: Any, w: Any) -> Tensor:
        out = linear_forward(x, w, self.fmt)
        self.ctx["output_layout"] = out.layout
        return out

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        x, w = self.inputs()
        dx, dw = linear_backward(x, w, gradient, self.fmt)
        return (dx, dw)


class MxLinearFP4(MxLinear):
    fmt = "MXFP4"


MX_OPERATIONS = {"mx_matmul": MxMatmul, "mx_linear": MxLinear, "mx_linear_fp4": MxLinearFP4}


def matmul(a: Tensor, b: Tensor, *, out_dtype: Any = None) -> Tensor:
    """C = A . B^T over two MX tensors, dispatched through A's carrier."""
    return a.carrier.dispatch_op("mx_matmul").forward(a, b, out_dtype=out_dtype)


def linear(x: Tensor, w: Tensor, *, fmt: str = "MXFP8_E4M3") -> Tensor:
    """Differentiable MX contraction x . w^T (autograd through the reference's
    Operation machinery)."""
    name = "mx_linear" if fmt == "MXFP8_E4M3" else "mx_linear_fp4"
    return x.carrier.dispatch_op(name).forward(x, w)
