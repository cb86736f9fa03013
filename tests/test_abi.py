"""The C ABI library loads and exports every symbol the header declares.

No GPU is needed: only host-side entry points run here (argument validation
that rejects before any CUDA call, and the scale-placement arithmetic).
"""

from __future__ import annotations

import re
from ctypes import c_void_p
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "strideweave_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(sw_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def native():
    from strideweave_b200 import build

    build.build()
    from strideweave_b200 import _native

    return _native


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("sw_reduce_f32", "sw_mx_quantize", "sw_mx_dequantize", "sw_mx_gemm", "sw_alloc",
                     "sw_last_error", "sw_matmul_f32"):
        assert required in names


def test_library_exports_every_declared_symbol(native):
    names = declared_functions()
    assert set(names) == set(native.SIGNATURES), "ctypes table and header disagree"
    for name in names:
        assert getattr(native.lib, name) is not None


def test_abi_version(native):
    assert native.lib.sw_abi_version() == 1


def test_scale_placement_matches_the_oracle(native):
    from oracle import oracle as O
    from strideweave_b200 import kernels

    for rows, kblocks in ((128, 4), (256, 8), (384, 32), (130, 5)):
        assert kernels.scale_bytes_tc128(rows, kblocks) == O.scale_bytes_tc128(rows, kblocks)
        for r in range(0, rows, 7):
            for kb in range(kblocks):
                assert kernels.scale_index_tc128(r, kb, kblocks) == O.scale_index_tc128(r, kb, kblocks)


def test_invalid_arguments_are_rejected_before_any_device_work(native):
    from strideweave_b200 import kernels

    with pytest.raises(NotImplementedError, match="K to be a positive multiple of 32"):
        kernels.mx_gemm(1, 16, 1024, 16, 16, 1024, 16, 16, 100, 128, 1000)
    with pytest.raises(NotImplementedError, match="needs M % 128 == 0 and N % 128 == 0"):
        kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 2, 100, 128, 1024)
    with pytest.raises(NotImplementedError, match="mixed operand formats"):
        native.check(native.lib.sw_mx_gemm(1, 2, c_void_p(16), 1024, c_void_p(16), c_void_p(16), 1024,
                                           c_void_p(16), c_void_p(16), 0, 128, 1, 128, 128, 1024, 0, None))
    with pytest.raises(ValueError, match="16-byte aligned"):
        kernels.mx_gemm(1, 17, 1024, 16, 16, 1024, 16, 16, 128, 128, 1024)
    with pytest.raises(ValueError, match="bad batch count"):
        kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, -1, 128, 256, 1024)
    with pytest.raises(ValueError, match="bad batch count"):
        kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 2, 128, 256, 1024, batch_stride_c=-1)
    with pytest.raises(NotImplementedError, match="stacked extent too large"):
        kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 1 << 24, 1024, 256, 1024)
    kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 0, 128, 256, 1024)  # no problems: no work
    # stacked results that overlap are refused (a row-major problem spans 127 * 256 + 255 + 1 elements;
    # the interleaved placement, batch stride 1 under pitches 2 and 256, is disjoint and runs on a GPU)
    for stride in (0, 1, 128 * 256 - 1):
        with pytest.raises(ValueError, match="results of the stacked problems may overlap"):
            kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 2, 128, 256, 1024, batch_stride_c=stride)
    with pytest.raises(ValueError, match="may overlap"):  # column-major problems 100 elements apart
        kernels.mx_gemm_batched(1, 16, 1024, 16, 16, 1024, 16, 16, 2, 128, 256, 1024, ldc_m=1, ldc_n=128,
                                batch_stride_c=100)
    # the NCCL wrappers check their arguments before they load NCCL
    from ctypes import byref

    from strideweave_b200.sharding import NcclCommunicator

    with pytest.raises(ValueError, match="128 bytes"):
        NcclCommunicator(2, 0, b"too short")
    ident = (native.ctypes.c_uint8 * native.SW_NCCL_ID_BYTES)()
    comm = native.c_void_p()
    with pytest.raises(ValueError, match="bad rank"):
        native.check(native.lib.sw_nccl_comm_init(byref(comm), 2, 2, ident))
    with pytest.raises(ValueError, match="null"):
        native.check(native.lib.sw_nccl_get_unique_id(None))
    with pytest.raises(ValueError, match="bad argument"):
        native.check(native.lib.sw_nccl_reduce_scatter_f32(c_void_p(16), c_void_p(16), -1, c_void_p(16), None))
    native.check(native.lib.sw_nccl_all_gather_f32(c_void_p(16), c_void_p(16), 0, c_void_p(16), None))  # empty
    native.check(native.lib.sw_nccl_comm_destroy(None))  # no communicator: nothing to do
    # the peer-memory K-split's pieces check their arguments before any CUDA call
    with pytest.raises(ValueError, match="1 to 8 destinations"):
        kernels.mx_gemm_routed(1, 16, 1024, 16, 16, 1024, 16, [16] * 9, 128, 256, 9 * 128, 256, 1024)
    with pytest.raises(ValueError, match="whole 128-row tiles"):
        kernels.mx_gemm_routed(1, 16, 1024, 16, 16, 1024, 16, [16, 32], 100, 256, 200, 256, 1024)
    with pytest.raises(ValueError, match="N must be a multiple of 4"):
        kernels.mx_gemm_routed(1, 16, 1024, 16, 16, 1024, 16, [16], 128, 260, 128, 258, 1024)
    with pytest.raises(ValueError, match="first destination must be one of the 2"):
        kernels.mx_gemm_routed(1, 16, 1024, 16, 16, 1024, 16, [16, 32], 128, 256, 256, 256, 1024, first=2)
    with pytest.raises(ValueError, match="destination 1 is null or not 16-byte aligned"):
        kernels.mx_gemm_routed(1, 16, 1024, 16, 16, 1024, 16, [16, 20], 128, 256, 256, 256, 1024)
    with pytest.raises(ValueError, match="bad flag count"):
        native.check(native.lib.sw_peer_wait(c_void_p(16), -1, 1, 1000, None))
    with pytest.raises(ValueError, match="limit must lie"):
        native.check(native.lib.sw_peer_wait(c_void_p(16), 2, 1, 0, None))
    native.check(native.lib.sw_peer_wait(None, 0, 1, 1000, None))  # no flags: nothing to wait for
    with pytest.raises(ValueError, match="at most 8 flags"):
        native.check(native.lib.sw_peer_signal(None, 9, 1, None))
    with pytest.raises(ValueError, match="null flag 1"):
        native.check(native.lib.sw_peer_signal((c_void_p * 2)(16, None), 2, 1, None))
    with pytest.raises(ValueError, match="bad extent"):
        native.check(native.lib.sw_sum_slots_f32(c_void_p(16), 16, 0, c_void_p(16), None))
    with pytest.raises(ValueError, match="whole 16-byte vectors"):
        native.check(native.lib.sw_sum_slots_f32(c_void_p(16), 6, 2, c_void_p(16), None))
    with pytest.raises(ValueError, match="bad argument"):
        native.check(native.lib.sw_ipc_alloc(byref(comm), 0, ident))
    with pytest.raises(ValueError, match="null argument"):
        native.check(native.lib.sw_ipc_open(None, byref(comm)))
    native.check(native.lib.sw_ipc_close(None))  # nothing mapped: nothing to do
    native.check(native.lib.sw_ipc_free(None))
    with pytest.raises(ValueError, match="unknown format"):
        kernels.mx_quantize(7, 16, 4, 32, 32, 1, 16, 32, 16)
    with pytest.raises(ValueError, match="payload pitch"):
        kernels.mx_quantize(1, 16, 4, 64, 64, 1, 16, 32, 16)
    with pytest.raises(ValueError, match="unknown reduction kind"):
        plan = kernels.make_reduce_plan("reduce_sum", 0, [(4, 1)], [(4, 4)])
        plan.kind = 9
        from ctypes import byref

        native.check(native.lib.sw_reduce_f32(byref(plan), c_void_p(16), 16, c_void_p(16), None))
    with pytest.raises(ValueError, match="outside carrier"):
        kernels.reduce_f32("reduce_max", 16, 15, 0, [(4, 1)], [(4, 4)], 16)
    with pytest.raises(ValueError, match="fibers must be non-empty"):
        kernels.reduce_f32("argmax", 16, 16, 0, [(4, 1)], [(0, 4)], 16)
    assert native.last_error() != ""
