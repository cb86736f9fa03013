"""sw_reduce_f32_noalloc against sw_reduce_f32, through the C ABI.

The no-allocation entry point is for callers that cannot let a library
allocate device memory: an engine that has already divided the whole device
among its own pools, or a process whose device-memory budget is fixed and
audited allocation by allocation.  It must give what sw_reduce_f32 gives
(max and argmax bit for bit, sum within the path's 2e-3 relative Frobenius
tolerance), and keep doing so on a second call, which finds the shared
scratch array as the first call left it.

This file is collected last, so a run that stops at its first failure has
already run every other test; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from strideweave_b200 import _native as N
from tests.gpu_util import bits, empty, rel_frobenius, to_device, to_host

pytestmark = pytest.mark.gpu

SUM_TOL = 2e-3
KINDS = ("reduce_sum", "reduce_max", "argmax")


def run(entry, kind, x, n_elems, kept, reduced):
    from strideweave_b200 import kernels

    n = int(np.prod([s for s, _ in kept]))
    plan = kernels.make_reduce_plan(kind, 0, kept, reduced)
    out = empty(4 * n)
    N.check(entry(ctypes.byref(plan), N.c_void_p(x.ptr), n_elems, N.c_void_p(out.ptr), None))
    N.raise_device_status()
    return to_host(out, n, np.int32 if kind == "argmax" else np.float32)


def agree(kind, got, want):
    if kind == "reduce_sum":
        assert rel_frobenius(got, want) <= SUM_TOL
    else:
        np.testing.assert_array_equal(bits(got), bits(want))


@pytest.mark.parametrize(
    "n_kept,n_red,transposed",
    [
        (1000, 4099, True),   # split column walk: 74 slices meet in the static scratch
        (8192, 4096, True),   # the transposed reduction of the benchmark
        (512, 3000, False),   # row walk: no scratch at all
    ],
)
def test_noalloc_entry_matches_the_allocating_entry_twice(n_kept, n_red, transposed):
    rng = np.random.default_rng(n_kept * 7 + n_red)
    a = rng.uniform(-1, 1, size=(n_kept, n_red)).astype(np.float32)
    a[::5, (np.arange(0, n_kept, 5) * 31) % n_red] = 3.0       # ties in different slices
    a[::5, (np.arange(0, n_kept, 5) * 17 + 2) % n_red] = 3.0
    if transposed:
        storage = a.T.ravel().copy()
        kept, reduced = [(n_kept, 1)], [(n_red, n_kept)]
    else:
        storage = a.ravel()
        kept, reduced = [(n_kept, n_red)], [(n_red, 1)]
    x = to_device(storage)
    for kind in KINDS:
        want = run(N.lib.sw_reduce_f32, kind, x, storage.size, kept, reduced)
        first = run(N.lib.sw_reduce_f32_noalloc, kind, x, storage.size, kept, reduced)
        second = run(N.lib.sw_reduce_f32_noalloc, kind, x, storage.size, kept, reduced)
        agree(kind, first, want)
        agree(kind, second, want)
