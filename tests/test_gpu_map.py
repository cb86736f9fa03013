"""sw_map_f32, the strided elementwise map behind the carrier's add / sub /
mul / pow / neg and the einsum lowering's union product, against numpy over
the same strided views.

The map is elementwise over one shared index space, so the library may walk
the leaves in any order: it drops unit leaves, orders the rest by output
stride, merges leaves that continue contiguously in every operand, and walks
rows (16-byte vectors where the row is dense).  Each case below takes a
different one of those paths; every result must equal numpy's binary32
arithmetic bit for bit (pow: the device powf, within one unit in the last
place) and leave every element outside the output view untouched.
"""

from __future__ import annotations

import ctypes
import zlib

import numpy as np
import pytest

from strideweave_b200 import _native as N
from tests.gpu_util import to_device, to_host

pytestmark = pytest.mark.gpu


def view(flat: np.ndarray, offset: int, shape, strides) -> np.ndarray:
    """numpy view of flat[offset + sum(i_d * stride_d)] over leaves (first fastest)."""
    idx = np.full((), offset, dtype=np.int64)
    for n, s in zip(shape, strides):
        idx = idx[..., None] + np.arange(n, dtype=np.int64) * s
    return flat[idx]


def run_map(op, shape, a, oa, sa, b, ob, sb, out_size, oo, so, scalar=0.0):
    rank = len(shape)
    arr = ctypes.c_int64 * max(rank, 1)
    da, db = to_device(a), to_device(b)
    guard = np.full(out_size, -7.25, np.float32)
    dout = to_device(guard)
    N.check(N.lib.sw_map_f32(op, rank, arr(*shape), N.c_void_p(da.ptr), oa, arr(*sa), a.size,
                             N.c_void_p(db.ptr), ob, arr(*sb), b.size, N.c_void_p(dout.ptr), oo, arr(*so), out_size,
                             float(scalar), None))
    N.raise_device_status()
    return to_host(dout, out_size, np.float32), guard


R, C = 512, 1024
CASES = {
    # the bench's X[R, C] * g[r]: leaf 0 is the strided one until the leaves are ordered
    "broadcast_rows": ((R, C), 0, (C, 1), 0, (1, 0), R * C, 0, (C, 1), R * C, R),
    # a row-major, out column-major: rows follow the output's unit stride, a strided reads
    "transposing": ((R, C), 0, (C, 1), 0, (C, 1), R * C, 0, (1, R), R * C, R * C),
    # three leaves that merge into one dense run, unaligned offsets (scalar row walk)
    "merged_unaligned": ((16, 8, 64), 1, (1, 16, 128), 3, (1, 16, 128), 8200, 2, (1, 16, 128), 8200, 8200),
    # hierarchical tiles of 32 x 32 with a broadcast column vector b
    "tiled": ((32, 16, 32, 8), 0, (1, 1024, 32, 32768), 0, (0, 0, 1, 32), R * 512, 0,
              (1, 1024, 32, 32768), R * 512, 256),
    # a short fastest leaf (3): the generic per-element walk
    "short_leaf": ((3, 700), 0, (700, 1), 0, (700, 1), 2100, 0, (1, 3), 2100, 2100),
    # rank 0: a single element
    "scalar": ((), 5, (), 2, (), 8, 3, (), 8, 8),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("op", ["add", "sub", "mul", "scale", "pow2", "pow", "pow_grad"])
def test_map_equals_numpy_on_strided_views(case, op):
    shape, oa, sa, ob, sb, out_size, oo, so, a_size, b_size = CASES[case]
    rng = np.random.default_rng(zlib.crc32(f"{case}/{op}".encode()))
    a = rng.uniform(0.25, 2.0, size=a_size).astype(np.float32)
    b = rng.uniform(-2.0, 2.0, size=b_size).astype(np.float32)
    codes = {"add": N.SW_MAP_ADD, "sub": N.SW_MAP_SUB, "mul": N.SW_MAP_MUL, "scale": N.SW_MAP_SCALE,
             "pow2": N.SW_MAP_POW, "pow": N.SW_MAP_POW, "pow_grad": N.SW_MAP_POW_GRAD}
    scalar = {"scale": -1.5, "pow2": 2.0, "pow": 1.7, "pow_grad": 1.7}.get(op, 0.0)
    if op == "pow_grad":  # g * p * x^(p - 1) with x = b's view: keep x positive
        b = np.abs(b) + np.float32(0.25)
    got, guard = run_map(codes[op], shape, a, oa, sa, b, ob, sb, out_size, oo, so, scalar)
    va, vb = view(a, oa, shape, sa), view(b, ob, shape, sb)
    s = np.float32(scalar)
    with np.errstate(all="ignore"):
        want = {"add": lambda: va + vb, "sub": lambda: va - vb, "mul": lambda: va * vb,
                "scale": lambda: va * s, "pow2": lambda: va * va,
                "pow": lambda: np.power(va, s), "pow_grad": lambda: (va * s) * np.power(vb, s - np.float32(1))}[op]()
    want = np.asarray(want, dtype=np.float32)
    written = np.zeros(out_size, bool)
    written[view(np.arange(out_size), oo, shape, so)] = True
    np.testing.assert_array_equal(got[~written], guard[~written])  # nothing outside the view
    vgot = view(got, oo, shape, so)
    if op in ("pow", "pow_grad"):
        np.testing.assert_allclose(vgot, want, rtol=3e-7, atol=0)
    else:
        np.testing.assert_array_equal(vgot.view(np.uint32), want.view(np.uint32))
