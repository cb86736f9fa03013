"""Host wrappers of the C ABI kernels, on raw device addresses.

These are the calls the CUDA carrier's operations make; they validate what
Python can see cheaply, build the POD plan structs and raise the exception the
library's status maps to.  Addresses are plain integers (``sw_alloc``
results, or any CUDA device address); ``stream`` is a ``cudaStream_t`` value
(0 = the legacy default stream).
"""

from __future__ import annotations

from ctypes import byref, c_void_p
from typing import Sequence

from . import _native as N

Leaf = tuple[int, int]  # (extent, stride)
SwizzleStage = tuple[int, int, int]  # (bits, base, shift)

REDUCE_KINDS = {"reduce_sum": N.SW_REDUCE_SUM, "reduce_max": N.SW_REDUCE_MAX, "argmax": N.SW_REDUCE_ARGMAX,
                "reduce_sum_f64": N.SW_REDUCE_SUM_F64}


def make_reduce_plan(kind: str, offset: int, kept: Sequence[Leaf], reduced: Sequence[Leaf],
                     swizzle: Sequence[SwizzleStage] = ()) -> N.ReducePlan:
    """Build an ``sw_reduce_plan`` from (extent, stride) leaves, first leaf fastest."""
    if kind not in REDUCE_KINDS:
        raise ValueError(f"unknown reduction {kind!r}")
    if len(kept) > N.SW_MAX_LEAVES or len(reduced) > N.SW_MAX_LEAVES:
        raise NotImplementedError(f"more than {N.SW_MAX_LEAVES} leaves in one mode")
    if len(swizzle) > N.SW_MAX_SWIZZLE:
        raise NotImplementedError(f"more than {N.SW_MAX_SWIZZLE} swizzle stages")
    plan = N.ReducePlan()
    plan.kind = REDUCE_KINDS[kind]
    plan.kept_rank = len(kept)
    plan.reduced_rank = len(reduced)
    plan.swizzle_rank = len(swizzle)
    plan.offset = int(offset)
    for i, (extent, stride) in enumerate(kept):
        plan.kept_shape[i] = int(extent)
        plan.kept_stride[i] = int(stride)
    for i, (extent, stride) in enumerate(reduced):
        plan.reduced_shape[i] = int(extent)
        plan.reduced_stride[i] = int(stride)
    for i, (bits, base, shift) in enumerate(swizzle):
        plan.swizzle_bits[i] = int(bits)
        plan.swizzle_base[i] = int(base)
        plan.swizzle_shift[i] = int(shift)
    return plan


def reduce_f32(kind: str, x_ptr: int, x_size: int, offset: int, kept: Sequence[Leaf], reduced: Sequence[Leaf],
               out_ptr: int, *, swizzle: Sequence[SwizzleStage] = (), stream: int = 0) -> None:
    """out[i] = reduction over the reduced leaves of kept ordinal i (see sw_reduce_f32)."""
    plan = make_reduce_plan(kind, offset, kept, reduced, swizzle)
    N.check(N.lib.sw_reduce_f32(byref(plan), c_void_p(x_ptr), int(x_size), c_void_p(out_ptr), c_void_p(stream)))


def reduce_backward_f32(kind: str, x_ptr: int, x_size: int, x_offset: int, kept: Sequence[Leaf],
                        reduced: Sequence[Leaf], swizzle: Sequence[SwizzleStage], grad_out_ptr: int, grad_in_ptr: int,
                        grad_kept: Sequence[Leaf], grad_reduced: Sequence[Leaf], grad_size: int,
                        grad_offset: int = 0, *, stream: int = 0) -> None:
    """grad_in = VJP of a reduce_sum / reduce_max (see sw_reduce_backward_f32)."""
    plan = make_reduce_plan(kind, x_offset, kept, reduced, swizzle)
    gplan = make_reduce_plan(kind, grad_offset, grad_kept, grad_reduced)
    N.check(N.lib.sw_reduce_backward_f32(byref(plan), c_void_p(x_ptr or None), int(x_size), c_void_p(grad_out_ptr),
                                         c_void_p(grad_in_ptr), byref(gplan), int(grad_size), c_void_p(stream)))


def copy_view_f32(src_ptr: int, src_size: int, src_offset: int, src_kept: Sequence[Leaf],
                  src_reduced: Sequence[Leaf], dst_ptr: int, dst_size: int, dst_offset: int,
                  dst_kept: Sequence[Leaf], dst_reduced: Sequence[Leaf], *, swizzle: Sequence[SwizzleStage] = (),
                  dst_swizzle: Sequence[SwizzleStage] = (), stream: int = 0) -> None:
    """Copy a two-mode 32-bit view into another placement, the source's flat
    indices through ``swizzle`` and the destination's through ``dst_swizzle``
    (see sw_copy_view_f32)."""
    sp = make_reduce_plan("reduce_sum", src_offset, src_kept, src_reduced, swizzle)
    dp = make_reduce_plan("reduce_sum", dst_offset, dst_kept, dst_reduced, dst_swizzle)
    N.check(N.lib.sw_copy_view_f32(byref(sp), c_void_p(src_ptr), int(src_size), byref(dp), c_void_p(dst_ptr),
                                   int(dst_size), c_void_p(stream)))


def mx_format(name: str) -> int:
    formats = {"E4M3": N.SW_MX_E4M3, "MXFP8_E4M3": N.SW_MX_E4M3, "E2M1": N.SW_MX_E2M1, "MXFP4": N.SW_MX_E2M1}
    try:
        return formats[name]
    except KeyError:
        raise NotImplementedError(f"MX format {name!r} has no kernel") from None


def mx_row_bytes(fmt: int, cols: int) -> int:
    return cols if fmt == N.SW_MX_E4M3 else (cols + 1) // 2


def scale_bytes_tc128(rows: int, kblocks: int) -> int:
    return int(N.lib.sw_mx_scale_bytes_tc128(int(rows), int(kblocks)))


def scale_index_tc128(r: int, kb: int, kblocks: int) -> int:
    return int(N.lib.sw_mx_scale_index(int(r), int(kb), int(kblocks)))


def mx_quantize(fmt: int, x_ptr: int, rows: int, cols: int, ld_row: int, ld_col: int, payload_ptr: int,
                ld_payload: int, scales_ptr: int, *, scale_layout: int = N.SW_SCALES_TC128, ld_scales: int = 0,
                stream: int = 0) -> None:
    N.check(N.lib.sw_mx_quantize(fmt, c_void_p(x_ptr), rows, cols, ld_row, ld_col, c_void_p(payload_ptr),
                                 ld_payload, c_void_p(scales_ptr), scale_layout, ld_scales, c_void_p(stream)))


def mx_quantize_view(fmt: int, x_ptr: int, x_size: int, offset: int, rows: Sequence[Leaf], cols: Sequence[Leaf],
                     payload_ptr: int, ld_payload: int, scales_ptr: int, *, swizzle: Sequence[SwizzleStage] = (),
                     scale_layout: int = N.SW_SCALES_TC128, ld_scales: int = 0, stream: int = 0) -> None:
    """Quantise the view whose row mode has leaves ``rows`` and whose quantised
    mode has leaves ``cols`` (first leaf fastest, flat indices through
    ``swizzle``) into MX planes (see sw_mx_quantize_view)."""
    plan = make_reduce_plan("reduce_sum", offset, rows, cols, swizzle)
    N.check(N.lib.sw_mx_quantize_view(fmt, byref(plan), c_void_p(x_ptr), int(x_size), c_void_p(payload_ptr),
                                      int(ld_payload), c_void_p(scales_ptr), scale_layout, int(ld_scales),
                                      c_void_p(stream)))


def mx_scales_to_tc128(src_ptr: int, ld_src: int, rows: int, kblocks: int, dst_ptr: int, *, stream: int = 0) -> None:
    """Row-major scales -> the tensor-core atom placement (see sw_mx_scales_to_tc128)."""
    N.check(N.lib.sw_mx_scales_to_tc128(c_void_p(src_ptr), int(ld_src), int(rows), int(kblocks), c_void_p(dst_ptr),
                                        c_void_p(stream)))


def mx_quantize_dual(fmt: int, transform: int, x_ptr: int, h_ptr: int, rows: int, cols: int, ld: int,
                     row_planes: tuple[int, int] | None, col_planes: tuple[int, int] | None, *,
                     scale_layout: int = N.SW_SCALES_TC128, stream: int = 0) -> None:
    """S[rows, cols] (x, gelu(x) or x * gelu'(h); unit stride along cols) quantised
    along cols into ``row_planes`` (payload, scales) and along rows into
    ``col_planes``, payload rows packed (see sw_mx_quantize_dual)."""
    pr, sr = row_planes if row_planes else (0, 0)
    pc, sc = col_planes if col_planes else (0, 0)
    N.check(N.lib.sw_mx_quantize_dual(fmt, transform, c_void_p(x_ptr), c_void_p(h_ptr or None), rows, cols, ld,
                                      c_void_p(pr or None), mx_row_bytes(fmt, cols), c_void_p(sr or None),
                                      scale_layout, cols // 32, c_void_p(pc or None), mx_row_bytes(fmt, rows),
                                      c_void_p(sc or None), scale_layout, rows // 32, c_void_p(stream)))


def mx_dequantize(fmt: int, payload_ptr: int, ld_payload: int, scales_ptr: int, rows: int, cols: int, out_ptr: int,
                  ld_out: int, *, scale_layout: int = N.SW_SCALES_TC128, ld_scales: int = 0,
                  stream: int = 0) -> None:
    N.check(N.lib.sw_mx_dequantize(fmt, c_void_p(payload_ptr), ld_payload, c_void_p(scales_ptr), scale_layout,
                                   ld_scales, rows, cols, c_void_p(out_ptr), ld_out, c_void_p(stream)))


def mx_gemm(fmt: int, a_ptr: int, lda: int, sfa_ptr: int, b_ptr: int, ldb: int, sfb_ptr: int, c_ptr: int,
            M: int, N_: int, K: int, *, out_bf16: bool = False, ldc_m: int | None = None, ldc_n: int = 1,
            beta_one: bool = False, max_ctas: int = 0, stream: int = 0) -> None:
    """C[m, n] = sum_k A[m, k] B[n, k] over MX operands (see sw_mx_gemm); at
    most ``max_ctas`` SMs when it is positive (sw_mx_gemm_ex)."""
    if ldc_m is None:
        ldc_m = N_
    N.check(N.lib.sw_mx_gemm_ex(fmt, fmt, c_void_p(a_ptr), lda, c_void_p(sfa_ptr), c_void_p(b_ptr), ldb,
                                c_void_p(sfb_ptr), c_void_p(c_ptr), N.SW_OUT_BF16 if out_bf16 else N.SW_OUT_F32,
                                ldc_m, ldc_n, M, N_, K, int(beta_one), int(max_ctas), c_void_p(stream)))


def mx_gemm_routed(fmt: int, a_ptr: int, lda: int, sfa_ptr: int, b_ptr: int, ldb: int, sfb_ptr: int,
                   dests: Sequence[int], rows_per_dest: int, ldc: int, M: int, N_: int, K: int, *, first: int = 0,
                   max_ctas: int = 0, stream: int = 0) -> None:
    """Float32 C[m, n] = sum_k A[m, k] B[n, k] with row block q written at
    dests[q] (row-major, pitch ldc), any of them a peer's memory; the tile
    walk starts with row block `first` (see sw_mx_gemm_routed)."""
    arr = (c_void_p * len(dests))(*[int(d) for d in dests])
    N.check(N.lib.sw_mx_gemm_routed(fmt, c_void_p(a_ptr), lda, c_void_p(sfa_ptr), c_void_p(b_ptr), ldb,
                                    c_void_p(sfb_ptr), arr, len(dests), rows_per_dest, ldc, int(first), M, N_, K,
                                    int(max_ctas), c_void_p(stream)))


def mx_gemm_batched(fmt: int, a_ptr: int, lda: int, sfa_ptr: int, b_ptr: int, ldb: int, sfb_ptr: int, c_ptr: int,
                    batch: int, M: int, N_: int, K: int, *, out_bf16: bool = False, ldc_m: int | None = None,
                    ldc_n: int = 1, batch_stride_c: int | None = None, beta_one: bool = False,
                    stream: int = 0) -> None:
    """C_p = A_p B_p^T for p < batch over stacked MX operands (A: [batch M, K],
    B: [batch N, K], TC128 scales of each stack) in one launch (see
    sw_mx_gemm_batched).  C_p defaults to the p-th [M, N] row-major block."""
    if ldc_m is None:
        ldc_m = N_
    if batch_stride_c is None:
        batch_stride_c = M * ldc_m if ldc_n == 1 else N_ * ldc_n
    N.check(N.lib.sw_mx_gemm_batched(fmt, fmt, c_void_p(a_ptr), lda, c_void_p(sfa_ptr), c_void_p(b_ptr), ldb,
                                     c_void_p(sfb_ptr), c_void_p(c_ptr),
                                     N.SW_OUT_BF16 if out_bf16 else N.SW_OUT_F32, ldc_m, ldc_n, batch_stride_c,
                                     batch, M, N_, K, int(beta_one), c_void_p(stream)))


def matmul_f32(a_ptr: int, sam: int, sak: int, b_ptr: int, sbn: int, sbk: int, c_ptr: int, scm: int, scn: int,
               M: int, N_: int, K: int, *, acc64: bool = False, stream: int = 0) -> None:
    """C[m, n] = sum_k A[m, k] B[n, k] with binary32 products, summed in binary32
    (or in binary64 and rounded once when ``acc64``)."""
    N.check(N.lib.sw_matmul_f32_batched_ex(c_void_p(a_ptr), 0, sam, sak, c_void_p(b_ptr), 0, sbn, sbk,
                                           c_void_p(c_ptr), 0, scm, scn, 1, M, N_, K,
                                           N.SW_ACC_F64 if acc64 else N.SW_ACC_F32, c_void_p(stream)))
