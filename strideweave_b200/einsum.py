"""Batched einsum on the device without the union product.

The reference lowers a two-input einsum with batch symbols by aligning both
inputs over the union index space, multiplying elementwise and reducing the
contracted symbols (src/strideweave/einops/__init__.py:459-475).  That
materialises a tensor of |batch| x |free| x |contracted| elements.  For the
common shape of a batched contraction - one batch symbol, one contracted
symbol, at most one free symbol per side, every mode a single stride - this
module computes the same result with one batched Float32 contraction
(``sw_matmul_f32_batched``), in the layout the reference returns (canonical
column-major over the output modes), with gradients.  Anything else goes to
the reference's own ``einsum``, which also runs on the CUDA carrier (through
its ``elementwise_mul`` and ``reduce_sum``).
"""

from __future__ import annotations

import re
from typing import Any

from . import _native as N
from ._host import DType, Layout, Operation, Shape, Stride, Tensor, require_capability, resolve_operation_plan
from .layout_plan import injective_layout_for, mode_leaves


def _single_stride(t: Tensor, mode: int) -> int | None:
    leaves = [(e, s) for e, s in mode_leaves(t.layout, mode) if e != 1]
    if not leaves:
        return 0
    ext, st = leaves[0]
    for e, s in leaves[1:]:
        if s != st * ext:
            return None
        ext *= e
    return st


def _mode_extent(t: Tensor, mode: int) -> int:
    n = 1
    for e, _ in mode_leaves(t.layout, mode):
        n *= e
    return n


def _plan(lhs: Tensor, rhs: Tensor, description: str) -> dict | None:
    """Symbol roles and strides when the fast path applies, else None."""
    m = re.fullmatch(r"\s*([\w ]+?)\s*,\s*([\w ]+?)\s*->\s*([\w ]*?)\s*", description)
    if not m:
        return None
    ls, rs, os_ = (part.split() for part in m.groups())
    if len(set(ls)) != len(ls) or len(set(rs)) != len(rs) or len(set(os_)) != len(os_):
        return None
    if any(not re.fullmatch(r"[A-Za-z_]\w*", sym) for sym in ls + rs + os_):
        return None
    if len(ls) != len(lhs.layout) or len(rs) != len(rhs.layout):
        return None
    shared = set(ls) & set(rs)
    batch = [s for s in os_ if s in shared]
    contracted = [s for s in ls if s in shared and s not in os_]
    lfree = [s for s in ls if s not in shared]
    rfree = [s for s in rs if s not in shared]
    if len(batch) != 1 or len(contracted) != 1 or len(lfree) > 1 or len(rfree) > 1:
        return None
    if set(os_) != set(batch + lfree + rfree):
        return None
    sizes: dict[str, int] = {}
    lstride: dict[str, int] = {}
    rstride: dict[str, int] = {}
    for t, syms, strides in ((lhs, ls, lstride), (rhs, rs, rstride)):
        for mode, sym in enumerate(syms):
            st = _single_stride(t, mode)
            if st is None:
                return None
            n = _mode_extent(t, mode)
            if sizes.setdefault(sym, n) != n:
                raise ValueError(f"symbol {sym!r} has sizes {sizes[sym]} and {n}")
            strides[sym] = st
    b, k = batch[0], contracted[0]
    i = lfree[0] if lfree else None
    j = rfree[0] if rfree else None
    out_sizes = [sizes[s] for s in os_]
    out_strides, acc = [], 1
    for n in out_sizes:  # canonical column-major, first output mode fastest
        out_strides.append(acc)
        acc *= n
    ostride = dict(zip(os_, out_strides))
    return {
        "batch": sizes[b], "M": sizes[i] if i else 1, "N": sizes[j] if j else 1, "K": sizes[k],
        "sab": lstride[b], "sam": lstride[i] if i else 0, "sak": lstride[k],
        "sbb": rstride[b], "sbn": rstride[j] if j else 0, "sbk": rstride[k],
        "scb": ostride[b], "scm": ostride[i] if i else 0, "scn": ostride[j] if j else 0,
        "layout": Layout(Shape(out_sizes), Stride(out_strides)) if out_sizes else Layout(Shape(1), Stride(1)),
    }


def _bmm(a: int, sab: int, sam: int, sak: int, b: int, sbb: int, sbn: int, sbk: int, c: int, scb: int, scm: int,
         scn: int, batch: int, M: int, Nn: int, K: int) -> None:
    N.check(N.lib.sw_matmul_f32_batched(N.c_void_p(a), sab, sam, sak, N.c_void_p(b), sbb, sbn, sbk, N.c_void_p(c),
                                        scb, scm, scn, batch, M, Nn, K, None))


class CudaBatchedContraction(Operation):
    """out[b, i, j] = sum_k lhs[b, i, k] rhs[b, j, k] (strides from the plan in
    ``ctx``), the reference's batched einsum result computed as one batched
    contraction; gradients in each input's injective canonical layout."""

    def _forward(self, lhs: Any, rhs: Any) -> Tensor:
        from .carrier import CUDA

        p = self.ctx["plan"]
        plan = resolve_operation_plan("matmul", lhs.carrier.dtype(), rhs.carrier.dtype())
        require_capability(CUDA, plan)
        out = Tensor(CUDA(p["layout"].cosize, empty=True, device=lhs.carrier.device), 0, p["layout"])
        a = lhs.carrier.data_ptr + 4 * lhs.offset
        b = rhs.carrier.data_ptr + 4 * rhs.offset
        _bmm(a, p["sab"], p["sam"], p["sak"], b, p["sbb"], p["sbn"], p["sbk"], out.carrier.data_ptr, p["scb"],
             p["scm"], p["scn"], p["batch"], p["M"], p["N"], p["K"])
        return out

    def backward(self, gradient: Any) -> tuple[Any, Any]:
        from .carrier import CUDA

        lhs, rhs = self.inputs()
        p = self.ctx["plan"]
        if gradient.layout.shape != p["layout"].shape:
            raise ValueError("Tensor shapes must match")
        if not isinstance(gradient.carrier, CUDA) or gradient.carrier.swizzle is not None:
            raise TypeError("gradient must be an unswizzled CUDA tensor")
        g_plan = _plan_like_output(gradient, p)
        g = gradient.carrier.data_ptr + 4 * gradient.offset
        a = lhs.carrier.data_ptr + 4 * lhs.offset
        b = rhs.carrier.data_ptr + 4 * rhs.offset
        outs = []
        for t, role in ((lhs, "lhs"), (rhs, "rhs")):
            lay = injective_layout_for(t.layout)
            outs.append(Tensor(CUDA(lay.cosize, empty=False, device=t.carrier.device), 0, lay))
        dl, dr = outs
        dlp = _strides_in(dl, self.ctx["lhs_syms"], p, "lhs")
        drp = _strides_in(dr, self.ctx["rhs_syms"], p, "rhs")
        # dlhs[b, i, k] = sum_j g[b, i, j] rhs[b, j, k]
        _bmm(g, g_plan["b"], g_plan["i"], g_plan["j"], b, p["sbb"], p["sbk"], p["sbn"], dl.carrier.data_ptr,
             dlp["b"], dlp["i"], dlp["k"], p["batch"], p["M"], p["K"], p["N"])
        # drhs[b, j, k] = sum_i g[b, i, j] lhs[b, i, k]
        _bmm(g, g_plan["b"], g_plan["j"], g_plan["i"], a, p["sab"], p["sak"], p["sam"], dr.carrier.data_ptr,
             drp["b"], drp["j"], drp["k"], p["batch"], p["N"], p["K"], p["M"])
        return (dl, dr)


def _mx_planes(fmt: int, ptr: int, sb: int, sr: int, sk: int, batch: int, rows: int, K: int, device: int):
    """Stacked MX planes of batch x [rows, K] Float32 views (element strides
    sb, sr, sk), quantised along K: one [batch rows, K] operand with its TC128
    scales, as sw_mx_gemm_batched reads them."""
    from . import kernels
    from .carrier import CUDA

    rb = kernels.mx_row_bytes(fmt, K)
    katoms = (K // 32 + 3) // 4
    payload = CUDA(batch * rows * K, dtype=DType.E4M3 if fmt == N.SW_MX_E4M3 else DType.E2M1, empty=True,
                   device=device)
    scales = CUDA(kernels.scale_bytes_tc128(batch * rows, K // 32), dtype=DType.E8M0, empty=True, device=device)
    if batch == 1 or sb == rows * sr:  # the problems' rows stack into one view
        kernels.mx_quantize(fmt, ptr, batch * rows, K, sr, sk, payload.data_ptr, rb, scales.data_ptr)
    else:
        for q in range(batch):
            kernels.mx_quantize(fmt, ptr + 4 * q * sb, rows, K, sr, sk, payload.data_ptr + q * rows * rb, rb,
                                scales.data_ptr + q * (rows // 128) * katoms * 512)
    return payload, scales, rb


class CudaMxBatchedContraction(CudaBatchedContraction):
    """The batched contraction with both inputs quantised to an MX format
    along the contracted symbol (``ctx["fmt"]``) and contracted by one
    batched block-scaled launch (``sw_mx_gemm_batched``) into the Float32
    result layout of the plain path.  Gradients are the Float32 contractions
    of the unquantised inputs (straight through the quantisation), as the
    plain path computes them."""

    def _forward(self, lhs: Any, rhs: Any) -> Tensor:
        from . import kernels
        from .carrier import CUDA

        p = self.ctx["plan"]
        fmt = self.ctx["fmt"]
        plan = resolve_operation_plan("matmul", lhs.carrier.dtype(), rhs.carrier.dtype())
        require_capability(CUDA, plan)
        dev = lhs.carrier.device
        out = Tensor(CUDA(p["layout"].cosize, empty=True, device=dev), 0, p["layout"])
        a = lhs.carrier.data_ptr + 4 * lhs.offset
        b = rhs.carrier.data_ptr + 4 * rhs.offset
        pa, sa, rb = _mx_planes(fmt, a, p["sab"], p["sam"], p["sak"], p["batch"], p["M"], p["K"], dev)
        pb, sb, _ = _mx_planes(fmt, b, p["sbb"], p["sbn"], p["sbk"], p["batch"], p["N"], p["K"], dev)
        kernels.mx_gemm_batched(fmt, pa.data_ptr, rb, sa.data_ptr, pb.data_ptr, rb, sb.data_ptr,
                                out.carrier.data_ptr, p["batch"], p["M"], p["N"], p["K"], ldc_m=p["scm"],
                                ldc_n=p["scn"], batch_stride_c=p["scb"])
        return out


def _plan_like_output(gradient: Tensor, p: dict) -> dict:
    syms = p["out_syms"]
    st = {}
    for mode, sym in enumerate(syms):
        s = _single_stride(gradient, mode)
        if s is None:
            raise NotImplementedError("a gradient mode that is not one stride")
        st[sym] = s
    return {"b": st[p["b"]], "i": st.get(p["i"], 0) if p["i"] else 0, "j": st.get(p["j"], 0) if p["j"] else 0}


def _strides_in(t: Tensor, syms: list[str], p: dict, side: str) -> dict:
    st = {sym: _single_stride(t, mode) for mode, sym in enumerate(syms)}
    free = p["i"] if side == "lhs" else p["j"]
    out = {"b": st[p["b"]], "k": st[p["k"]]}
    out["i" if side == "lhs" else "j"] = st[free] if free else 0
    return out


def einsum(lhs: Any, rhs: Any, description: str, *, fmt: str | None = None) -> Tensor:
    """``sw.einsum(lhs, rhs, description)`` for CUDA-carrier tensors, with the
    batched fast path described in the module docstring.

    ``fmt`` ("MXFP8_E4M3" or "MXFP4") computes that fast path on the
    block-scaled tensor cores instead: both inputs quantised along the
    contracted symbol, one batched MX contraction, Float32 result.  It needs
    the fast path's shape with a free symbol on each side, both free extents
    multiples of 128 and the contracted one of 128 (E4M3) or 256 (E2M1); other
    einsums with ``fmt`` raise NotImplementedError."""
    from strideweave.einops import einsum as reference_einsum

    from . import kernels
    from .carrier import CUDA

    code = kernels.mx_format(fmt) if fmt is not None else None

    if (isinstance(lhs, Tensor) and isinstance(rhs, Tensor) and isinstance(lhs.carrier, CUDA)
            and isinstance(rhs.carrier, CUDA) and lhs.carrier.dtype() is DType.Float32
            and rhs.carrier.dtype() is DType.Float32 and lhs.carrier.swizzle is None
            and rhs.carrier.swizzle is None):
        lhs._require_single_subtensor("einsum")
        rhs._require_single_subtensor("einsum")
        p = _plan(lhs, rhs, description)
        if p is not None:
            m = re.fullmatch(r"\s*([\w ]+?)\s*,\s*([\w ]+?)\s*->\s*([\w ]*?)\s*", description)
            ls, rs, os_ = (part.split() for part in m.groups())
            shared = set(ls) & set(rs)
            p["b"] = next(s for s in os_ if s in shared)
            p["k"] = next(s for s in ls if s in shared and s not in os_)
            p["i"] = next((s for s in ls if s not in shared), None)
            p["j"] = next((s for s in rs if s not in shared), None)
            p["out_syms"] = os_
            if code is not None:
                if not (p["i"] and p["j"] and p["M"] % 128 == 0 and p["N"] % 128 == 0 and p["K"] % 32 == 0):
                    raise NotImplementedError(
                        f"einsum with fmt={fmt!r} needs a free symbol on each side, free extents that are "
                        f"multiples of 128 and a contracted extent that is a multiple of 32")
                op = CudaMxBatchedContraction()
                op.ctx["fmt"] = code
            else:
                op = CudaBatchedContraction()
            op.ctx["plan"] = p
            op.ctx["lhs_syms"] = ls
            op.ctx["rhs_syms"] = rs
            return op.forward(lhs, rhs)
    if code is not None:
        raise NotImplementedError(f"einsum with fmt={fmt!r} needs two unswizzled Float32 CUDA tensors in the shape "
                                  "of a batched contraction (one batch and one contracted symbol)")
    return reference_einsum(lhs, rhs, description)


__all__ = ["CudaBatchedContraction", "CudaMxBatchedContraction", "einsum"]
