"""Generate the golden fixtures of the hot path from the reference itself.

Run in a container where the reference StrideWeave is importable (an installed
copy such as ``baseline/_ref`` on ``PYTHONPATH``)::

    PYTHONPATH=baseline/_ref python tests/golden/make_golden.py

It runs the reference CPU carrier (``sw.reduce_sum``, ``sw.reduce_max``,
``sw.argmax``, ``sw.matmul``) and ``Swizzle`` on small seeded inputs and
writes inputs and outputs to ``tests/golden/*.npz``.  The tests compare the
CPU oracle (and, on a GPU, the CUDA path) against these files; nothing reads
the reference at test time.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import strideweave as sw
from strideweave import CPU, Layout, Shape, Stride, Swizzle, SwizzleStage, Tensor

HERE = Path(__file__).resolve().parent


def adversarial_rows(rng: np.random.Generator, n: int, m: int) -> np.ndarray:
    """U(-1,1) rows with the special values the reference pins for extrema."""
    x = rng.uniform(-1.0, 1.0, size=(n, m)).astype(np.float32)
    nan_a = np.array([0x7FC00001], dtype=np.uint32).view(np.float32)[0]
    nan_b = np.array([0xFFC00123], dtype=np.uint32).view(np.float32)[0]
    x[1, 5] = nan_a
    x[1, 9] = nan_b  # first NaN (payload 0x7FC00001) must win
    x[2, :] = -0.0
    x[3, :] = -1.0
    x[3, 7] = -0.0  # a single zero keeps its sign
    x[4, :] = -1.0
    x[4, 7] = -0.0
    x[4, 11] = 0.0  # two zeros give +0
    x[5, :] = 0.25
    x[5, 3] = 0.75
    x[5, 40] = 0.75  # argmax tie: first ordinal
    x[6, :] = -np.inf
    x[7, 2] = np.inf
    x[7, 6] = np.inf
    x[8, 0] = nan_b
    x[9, m - 1] = np.float32(2.0)
    x[10, :] = np.float32(-3.0)
    return x


def reference_reduce(flat: np.ndarray, layout: Layout, kept: int) -> dict[str, np.ndarray]:
    carrier = CPU(flat.size, pointer=flat.ctypes.data)
    tensor = Tensor(carrier, 0, layout)
    out = {}
    with sw.no_grad():
        for name, fn in (("sum", sw.reduce_sum), ("max", sw.reduce_max), ("argmax", sw.argmax)):
            r = fn(tensor, "a b -> a")
            dtype = np.int32 if name == "argmax" else np.float32
            out[name] = np.array([r[i] for i in range(kept)], dtype=dtype)
    return out


def main() -> None:
    rng = np.random.default_rng(20261201)
    n, m = 64, 96
    x = adversarial_rows(rng, n, m)

    # (a) row-major view of the n x m values
    rowmajor = np.ascontiguousarray(x).ravel()
    res_a = reference_reduce(rowmajor, Layout(Shape([n, m]), Stride([m, 1])), n)
    # (b) transposed stride view: the same logical values stored column-major
    colmajor = np.ascontiguousarray(x.T).ravel()
    res_b = reference_reduce(colmajor, Layout(Shape([n, m]), Stride([1, n])), n)
    # (c) hierarchical tiled layout: 16x32 tiles, rows (16, n/16), cols (32, m/32);
    # tile (tr, tc) stored contiguously row-major, tiles ordered tc-fastest
    tr, tc = 16, 32
    tiled_shape = Shape([[tr, n // tr], [tc, m // tc]])
    tiled_stride = Stride([[tc, tr * tc * (m // tc)], [1, tr * tc]])
    tiled_layout = Layout(tiled_shape, tiled_stride)
    tiled = np.empty(n * m, dtype=np.float32)
    for i in range(n):
        for j in range(m):
            off = (i % tr) * tc + (i // tr) * tr * tc * (m // tc) + (j % tc) + (j // tc) * tr * tc
            tiled[off] = x[i, j]
    res_c = reference_reduce(tiled, tiled_layout, n)

    # swizzle: the carrier stores flat index f at swizzle(f); the reference
    # cannot place a tensor through a Swizzle, so the logical (unswizzled)
    # data is reduced by the reference and the swizzle map itself is pinned.
    size = n * m  # 6144 is not a power of two: pin the map on a 8192 domain
    swz = Swizzle(Shape(8192), SwizzleStage(bits=3, base=2, shift=3))
    swz_in = np.arange(8192, dtype=np.int64)
    swz_out = np.array([swz(int(i)) for i in swz_in], dtype=np.int64)

    # matmul: lhs[M,K] . rhs[N,K] -> out[M,N] (canonical column-major result)
    M, N, K = 24, 40, 72
    lhs = rng.standard_normal((M, K)).astype(np.float32)
    rhs = rng.standard_normal((N, K)).astype(np.float32)
    tl = Tensor(CPU(lhs.size, pointer=lhs.ctypes.data), 0, Layout(Shape([M, K]), Stride([K, 1])))
    tr_ = Tensor(CPU(rhs.size, pointer=rhs.ctypes.data), 0, Layout(Shape([N, K]), Stride([K, 1])))
    with sw.no_grad():
        r = sw.matmul(tl, tr_)
        mm = np.array([[r[i, j] for j in range(N)] for i in range(M)], dtype=np.float32)
        r64 = sw.matmul(tl, tr_, accumulator_dtype=sw.DType.Float64)
        mm64 = np.array([[r64[i, j] for j in range(N)] for i in range(M)], dtype=np.float32)
    out_layout = str(r.layout)

    np.savez_compressed(
        HERE / "reductions.npz",
        x=x, rowmajor=rowmajor, colmajor=colmajor, tiled=tiled,
        **{f"a_{k}": v for k, v in res_a.items()},
        **{f"b_{k}": v for k, v in res_b.items()},
        **{f"c_{k}": v for k, v in res_c.items()},
        swz_in=swz_in, swz_out=swz_out,
    )
    np.savez_compressed(HERE / "matmul.npz", lhs=lhs, rhs=rhs, out=mm, out_acc64=mm64,
                        out_layout=np.array(out_layout))
    print("wrote", HERE / "reductions.npz", HERE / "matmul.npz", "result layout", out_layout, "size", size)


if __name__ == "__main__":
    main()
