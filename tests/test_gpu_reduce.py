"""Layout-aware reductions on the GPU against the reference (golden fixtures)
and the CPU oracle, through the C ABI.

max and argmax are bit-exact; sum is within the path's 2e-3 relative
Frobenius tolerance of the reference's Float32 sequential sum.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.gpu_util import bits, empty, rel_frobenius, to_device, to_host

pytestmark = pytest.mark.gpu

SUM_TOL = 2e-3
GOLDEN = Path(__file__).resolve().parent / "golden"
N_, M_ = 64, 96
GOLDEN_LAYOUTS = {
    "a": ("rowmajor", [(N_, M_)], [(M_, 1)]),
    "b": ("colmajor", [(N_, 1)], [(M_, N_)]),
    "c": ("tiled", [(16, 32), (N_ // 16, 16 * 32 * (M_ // 32))], [(32, 1), (M_ // 32, 16 * 32)]),
}
KINDS = {"sum": "reduce_sum", "max": "reduce_max", "argmax": "argmax"}


def gpu_reduce(kind, storage, offset, kept, reduced, swizzle=()):
    from strideweave_b200 import kernels

    n = int(np.prod([s for s, _ in kept])) if kept else 1
    x = to_device(storage.astype(np.float32))
    out = empty(4 * n)
    kernels.reduce_f32(KINDS[kind], x.ptr, storage.size, offset, kept, reduced, out.ptr, swizzle=swizzle)
    return to_host(out, n, np.int32 if kind == "argmax" else np.float32)


def check(kind, got, want):
    if kind == "sum":
        finite = np.isfinite(want)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert rel_frobenius(got[finite], want[finite]) <= SUM_TOL
    else:
        np.testing.assert_array_equal(bits(got), bits(want))


@pytest.fixture(scope="module")
def red():
    return np.load(GOLDEN / "reductions.npz")


@pytest.mark.parametrize("case", ["a", "b", "c"])
@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
def test_golden_layouts(red, case, kind):
    storage_key, kept, reduced = GOLDEN_LAYOUTS[case]
    check(kind, gpu_reduce(kind, red[storage_key], 0, kept, reduced), red[f"{case}_{kind}"])


@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
def test_golden_through_carrier_swizzle(red, kind):
    stages = [(3, 2, 3)]
    logical = np.zeros(8192, dtype=np.float32)
    logical[: N_ * M_] = red["rowmajor"]
    physical = np.empty_like(logical)
    physical[np.array([O.swizzle_index(f, stages) for f in range(8192)])] = logical
    check(kind, gpu_reduce(kind, physical, 0, [(N_, M_)], [(M_, 1)], swizzle=stages), red[f"a_{kind}"])


def config2_layouts():
    """The three layouts of the reduction config over X[8192 x 4096]."""
    R, C = 8192, 4096
    return {
        "rowmajor": ([(R, C)], [(C, 1)], []),
        "transposed": ([(R, 1)], [(C, R)], []),
        # 128 x 32 tiles (16 KiB), tile rows of 128 bytes, column tiles
        # contiguous; the carrier stores its flat space through a 3-bit
        # swizzle of the 16-byte chunks of each 128-byte row.
        "tiled_swizzled": ([(128, 32), (64, 128 * 32 * 128)], [(32, 1), (128, 128 * 32)], [(3, 2, 3)]),
    }


@pytest.mark.parametrize("layout", ["rowmajor", "transposed", "tiled_swizzled"])
@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
def test_full_size_against_oracle(layout, kind):
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, size=8192 * 4096).astype(np.float32)
    x[123] = np.nan  # a NaN somewhere in the storage
    kept, reduced, swz = config2_layouts()[layout]
    got = gpu_reduce(kind, x, 0, kept, reduced, swz)
    want = O.reduce("sum64" if kind == "sum" else kind, x, 0, kept, reduced, swizzle=swz)
    check(kind, got, want)


@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
@pytest.mark.parametrize(
    "shape",
    [
        (1, 1),      # one kept element, one reduced element
        (1, 4099),   # single long ragged fibre
        (4099, 3),   # many short fibres
        (37, 4099),  # ragged extents: generic gather path
        (128, 4096),
    ],
)
def test_edge_shapes_row_and_column(kind, shape):
    rng = np.random.default_rng(11)
    n, m = shape
    x = rng.standard_normal(n * m + 5).astype(np.float32)
    for kept, reduced, off in (([(n, m)], [(m, 1)], 0), ([(n, 1)], [(m, n)], 0), ([(n, m)], [(m, 1)], 5)):
        got = gpu_reduce(kind, x, off, kept, reduced)
        want = O.reduce(kind, x, off, kept, reduced)
        check(kind, got, want)


@pytest.mark.parametrize("kind", ["max", "argmax"])
def test_extrema_specials_in_every_lane_position(kind):
    # NaN payloads, +-0, ties and infinities placed at many positions so that
    # every lane / split boundary of the parallel trees sees them.
    rng = np.random.default_rng(3)
    n, m = 256, 1024
    x = rng.uniform(-1, 1, size=(n, m)).astype(np.float32)
    nan1 = np.array([0x7FC0BEEF], dtype=np.uint32).view(np.float32)[0]
    nan2 = np.array([0xFF800001], dtype=np.uint32).view(np.float32)[0]
    for i in range(n):
        kind_i = i % 6
        j = (i * 37) % m
        if kind_i == 0:
            x[i, j] = nan1
            x[i, (j + 500) % m] = nan2
        elif kind_i == 1:
            x[i, :] = -1.0
            x[i, j] = -0.0
        elif kind_i == 2:
            x[i, :] = -1.0
            x[i, j] = -0.0
            x[i, (j + 1) % m] = 0.0
        elif kind_i == 3:
            x[i, j] = 5.0
            x[i, (j * 7 + 3) % m] = 5.0
        elif kind_i == 4:
            x[i, :] = -np.inf
        else:
            x[i, j] = np.inf
    for storage, kept, reduced in ((x.ravel(), [(n, m)], [(m, 1)]), (x.T.ravel().copy(), [(n, 1)], [(m, n)])):
        check(kind, gpu_reduce(kind, storage, 0, kept, reduced), O.reduce(kind, storage, 0, kept, reduced))


@pytest.mark.parametrize("kind", ["sum", "max", "argmax"])
@pytest.mark.parametrize("n_kept,n_red", [(2372, 517), (4740, 33), (8196, 130)])
def test_narrow_column_walk_with_ragged_blocks_and_specials(kind, n_kept, n_red):
    # transposed fibres with kept extents that take the narrow walk (a CTA of
    # 16 or 32 kept columns over the whole fibre) and end in a partial CTA;
    # NaN payloads, signed zeros, ties and infinities in several row streams
    rng = np.random.default_rng(n_kept + n_red)
    x = rng.uniform(-1, 1, size=(n_kept, n_red)).astype(np.float32)
    nan1 = np.array([0x7FC0BEEF], dtype=np.uint32).view(np.float32)[0]
    nan2 = np.array([0xFF800001], dtype=np.uint32).view(np.float32)[0]
    for i in range(0, n_kept, 7):
        j = (i * 31) % n_red
        k = i % 5
        if k == 0:
            x[i, j], x[i, (j + n_red // 2) % n_red] = nan1, nan2
        elif k == 1:
            x[i, :] = -1.0
            x[i, j], x[i, (j + 3) % n_red] = -0.0, 0.0
        elif k == 2:
            x[i, j] = x[i, (j * 7 + 1) % n_red] = 4.0
        elif k == 3:
            x[i, :] = -np.inf
        else:
            x[i, j] = np.inf
    storage = x.T.ravel().copy()
    kept, reduced = [(n_kept, 1)], [(n_red, n_kept)]
    check(kind, gpu_reduce(kind, storage, 0, kept, reduced), O.reduce(kind, storage, 0, kept, reduced))


def test_hierarchical_modes_with_permuted_leaves():
    # reduced mode ((8, 16):(64, 1)) - its unit-stride leaf is not the first
    rng = np.random.default_rng(5)
    x = rng.standard_normal(64 * 8 * 16).astype(np.float32)
    kept = [(64, 128)]
    reduced = [(8, 16), (16, 1)]
    for kind in ("sum", "max", "argmax"):
        check(kind, gpu_reduce(kind, x, 0, kept, reduced), O.reduce(kind, x, 0, kept, reduced))


def test_empty_kept_mode_is_a_no_op():
    from strideweave_b200 import kernels

    x = to_device(np.zeros(16, dtype=np.float32))
    out = empty(16)
    kernels.reduce_f32("reduce_sum", x.ptr, 16, 0, [(0, 1)], [(4, 4)], out.ptr)


@pytest.mark.parametrize("n_kept,n_red", [(1000, 4099), (8192, 517), (64, 100000)])
def test_split_column_walk_repeats_and_regrows_its_scratch(n_kept, n_red):
    # transposed storage: the fibre is split into slices whose partials meet in
    # scratch memory; each launch must leave its counters at zero for the next
    # one, and a kind with wider partials regrows the buffer
    rng = np.random.default_rng(n_kept + n_red)
    x = rng.uniform(-1, 1, size=(n_kept, n_red)).astype(np.float32)
    x[::7, (np.arange(0, n_kept, 7) * 13) % n_red] = 2.0      # ties across slices
    x[::7, (np.arange(0, n_kept, 7) * 29 + 1) % n_red] = 2.0
    storage = x.T.ravel().copy()
    kept, reduced = [(n_kept, 1)], [(n_red, n_kept)]
    for kind in ("sum", "max", "argmax", "sum", "argmax", "max"):
        check(kind, gpu_reduce(kind, storage, 0, kept, reduced), O.reduce(kind, storage, 0, kept, reduced))
