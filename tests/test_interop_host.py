"""Host-side interop checks that need no GPU: the CPU <-> CUDA pair is in the
reference's move registry once the carrier is imported, and the DLPack dtype
table agrees with what torch's exporter writes into a capsule."""

from __future__ import annotations

import ctypes

import pytest

sw = pytest.importorskip("strideweave")


def test_move_registry_dispatches_the_cuda_pair():
    from strideweave import CPU
    from strideweave.carriers.move import dispatch_move

    from strideweave_b200.carrier import CUDA
    from strideweave_b200.move import CpuToCudaMoveOperation, CudaToCpuMoveOperation, register

    register()  # idempotent
    assert dispatch_move(CPU, CUDA) is CpuToCudaMoveOperation
    assert dispatch_move(CUDA, CPU) is CudaToCpuMoveOperation


def test_dlpack_dtype_table_matches_torch_capsules():
    torch = pytest.importorskip("torch")
    from strideweave import DType

    from strideweave_b200 import BFloat16
    from strideweave_b200.dlpack import _CODES, DLManagedTensor, _api

    expected = {
        torch.float32: DType.Float32,
        torch.int32: DType.Int32,
        torch.bool: DType.Bool,
        torch.bfloat16: BFloat16,
        torch.float8_e4m3fn: DType.E4M3,
        torch.float8_e8m0fnu: DType.E8M0,
    }
    samples = {dt: torch.zeros(4, dtype=dt) for dt in expected}
    samples[torch.float4_e2m1fn_x2] = torch.zeros(4, dtype=torch.uint8).view(torch.float4_e2m1fn_x2)
    expected[torch.float4_e2m1fn_x2] = DType.E2M1
    for dt, t in samples.items():
        cap = t.__dlpack__()
        dl = DLManagedTensor.from_address(_api.PyCapsule_GetPointer(cap, b"dltensor")).dl_tensor
        assert _CODES[(dl.dtype.code, dl.dtype.bits, dl.dtype.lanes)] is expected[dt], dt
        del dl, cap
    assert ctypes.sizeof(DLManagedTensor) >= 48


def test_exported_capsule_life_cycle_needs_no_device():
    # an export capsule dropped unconsumed, and one consumed (renamed, its
    # deleter called by the consumer), both release what they keep alive;
    # the capsule destructor must not touch the dying capsule object
    import gc

    from strideweave_b200 import dlpack as D

    for consume in (False, True):
        m = D.DLManagedTensor()
        m.deleter = D._release_export
        D._LIVE[ctypes.addressof(m)] = (m,)
        cap = D._api.PyCapsule_New(ctypes.addressof(m), b"dltensor", D._capsule_destructor)
        if consume:
            D._api.PyCapsule_SetName(cap, b"used_dltensor")
            m.deleter(ctypes.pointer(m))
        del cap
        gc.collect()
        assert ctypes.addressof(m) not in D._LIVE


@pytest.mark.parametrize("stages", [[(3, 2, 3)], [(2, 4, -3)], [(3, 2, 3), (2, 7, -4)]])
def test_vectorised_swizzle_map_equals_the_reference_swizzle(stages):
    """The numpy swizzle map the carrier's host paths (moves, uploads, reads)
    use equals the reference's Swizzle evaluated index by index."""
    import numpy as np
    from strideweave import Shape, Swizzle, SwizzleStage

    from strideweave_b200.layout_plan import swizzle_map

    size = 1 << 13
    swz = Swizzle(Shape(size), *[SwizzleStage(bits=b, base=a, shift=s) for b, a, s in stages])
    np.testing.assert_array_equal(swizzle_map(stages, size), [swz(i) for i in range(size)])
