"""sw_reduce_f32_noalloc against sw_reduce_f32 and the CPU oracle, through the C ABI.

The no-allocation entry point is for callers that cannot let a library
allocate device memory: an engine that has already divided the whole device
among its own pools, or a process whose device-memory budget is fixed and
audited allocation by allocation.  It must give what sw_reduce_f32 gives
(max and argmax bit for bit, sum within the path's 2e-3 relative Frobenius
tolerance) and what the oracle's sequential folds give, keep doing so on a
second call, which finds the shared scratch array as the first call left it,
and leave the device's memory pool exactly as it found it.

This file is collected last, so a run that stops at its first failure has
already run every other test; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from strideweave_b200 import _native as N
from tests.gpu_util import bits, empty, rel_frobenius, to_device, to_host

pytestmark = pytest.mark.gpu

SUM_TOL = 2e-3
KINDS = ("reduce_sum", "reduce_max", "argmax")


ORACLE_KIND = {"reduce_sum": "sum", "reduce_max": "max", "argmax": "argmax"}


def run(entry, kind, x, n_elems, kept, reduced, stream=None, out=None):
    from strideweave_b200 import kernels

    n = int(np.prod([s for s, _ in kept]))
    plan = kernels.make_reduce_plan(kind, 0, kept, reduced)
    out = empty(4 * n) if out is None else out
    N.check(entry(ctypes.byref(plan), N.c_void_p(x.ptr), n_elems, N.c_void_p(out.ptr), N.c_void_p(stream)))
    N.raise_device_status()
    return to_host(out, n, np.int32 if kind == "argmax" else np.float32)


def pool_used_bytes() -> int:
    """Bytes in use in the current device's default memory pool, the pool
    that sw_alloc and the allocating reductions draw from."""
    from cuda.bindings import driver as drv

    (err,) = drv.cuInit(0)
    assert err == drv.CUresult.CUDA_SUCCESS
    err, dev = drv.cuDeviceGet(N.current_device())
    assert err == drv.CUresult.CUDA_SUCCESS
    err, pool = drv.cuDeviceGetDefaultMemPool(dev)
    assert err == drv.CUresult.CUDA_SUCCESS
    err, used = drv.cuMemPoolGetAttribute(pool, drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_CURRENT)
    assert err == drv.CUresult.CUDA_SUCCESS
    return int(used)


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
        oracle = O.reduce(ORACLE_KIND[kind], storage, 0, kept, reduced)
        first = run(N.lib.sw_reduce_f32_noalloc, kind, x, storage.size, kept, reduced)
        second = run(N.lib.sw_reduce_f32_noalloc, kind, x, storage.size, kept, reduced)
        agree(kind, want, oracle)
        agree(kind, first, oracle)
        agree(kind, second, oracle)
        agree(kind, first, want)
        agree(kind, second, want)


def test_noalloc_entry_leaves_the_memory_pool_untouched():
    """On a stream no reduction has used yet, two split column walks through
    the no-allocation entry leave the pool's bytes in use unchanged; the
    allocating entry on the same stream then reserves its scratch, which shows
    the measurement would see an allocation."""
    n_kept, n_red = 1000, 4099
    rng = np.random.default_rng(11)
    storage = rng.uniform(-1, 1, size=n_kept * n_red).astype(np.float32)
    kept, reduced = [(n_kept, 1)], [(n_red, n_kept)]
    x = to_device(storage)
    outs = [empty(4 * n_kept) for _ in range(3)]
    stream = N.c_void_p()
    N.check(N.lib.sw_stream_create(ctypes.byref(stream)))
    try:
        N.synchronize()
        before = pool_used_bytes()
        got = [run(N.lib.sw_reduce_f32_noalloc, "argmax", x, storage.size, kept, reduced, stream.value, outs[i])
               for i in range(2)]
        N.check(N.lib.sw_stream_synchronize(stream))
        assert pool_used_bytes() == before
        want = O.reduce("argmax", storage, 0, kept, reduced)
        for g in got:
            np.testing.assert_array_equal(g, want)
        run(N.lib.sw_reduce_f32, "argmax", x, storage.size, kept, reduced, stream.value, outs[2])
        N.check(N.lib.sw_stream_synchronize(stream))
        assert pool_used_bytes() > before
    finally:
        N.synchronize()
        N.check(N.lib.sw_stream_destroy(stream))
