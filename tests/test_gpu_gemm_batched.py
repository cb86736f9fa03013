"""The batched block-scaled contraction (sw_mx_gemm_batched) on the device.

Problem p of a stacked launch must equal the single contraction of its own
operands bit for bit, whichever epilogue writes it:
  * staged row-major fp32 and bf16;
  * staged column-major fp32;
  * direct stores for results with gaps between them, and for accumulation;
  * the narrow-tile path.
Each problem also stays within the path's 2e-3 relative Frobenius tolerance
of the oracle (the reference contraction of the dequantised operands).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from strideweave_b200 import _native as N
from tests.gpu_util import empty, rel_frobenius, to_host
from tests.test_gpu_gemm import operands

pytestmark = pytest.mark.gpu

TOL = 2e-3
BATCH, M, K = 3, 256, 512


def layout(kind: str, n: int) -> dict:
    """Output pitches and problem stride of each case, in elements."""
    if kind == "cols":
        return dict(ldc_m=1, ldc_n=M, batch_stride_c=n * M)
    if kind == "gapped":
        return dict(ldc_m=n, ldc_n=1, batch_stride_c=M * n + 64)
    return dict(ldc_m=n, ldc_n=1, batch_stride_c=M * n)


def as_matrix(raw: np.ndarray, kind: str, n: int, bf16: bool) -> np.ndarray:
    block = raw[: M * n]
    if bf16:
        block = (block.astype(np.uint32) << 16).view(np.float32)
    return block.reshape(n, M).T if kind == "cols" else block.reshape(M, n)


@pytest.mark.parametrize("fmt", [O.E4M3, O.E2M1])
@pytest.mark.parametrize("kind", ["rows", "cols", "bf16", "gapped", "narrow", "accumulate"])
def test_each_problem_equals_its_own_contraction(fmt, kind):
    from strideweave_b200 import kernels

    n = 128 if kind == "narrow" else 512
    bf16 = kind == "bf16"
    esize = 2 if bf16 else 4
    hdt = np.uint16 if bf16 else np.float32
    (pa, sa, ra), (pb, sb, rb), da, db = operands(fmt, BATCH * M, BATCH * n, K, seed=31, b_sigma=0.05)
    lay = layout(kind, n)
    total = (BATCH - 1) * lay["batch_stride_c"] + M * n
    c = empty(total * esize, fill=0)
    init = np.ones(total, np.float32) if kind == "accumulate" else None
    if init is not None:
        c.upload(init)
    kernels.mx_gemm_batched(fmt, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, BATCH, M, n, K, out_bf16=bf16,
                            beta_one=init is not None, **lay)
    N.raise_device_status()
    got = to_host(c, total, hdt)
    katoms = (K // 32 + 3) // 4
    for p in range(BATCH):
        one = empty(M * n * esize, fill=0)
        if init is not None:
            one.upload(np.ones(M * n, np.float32))
        kernels.mx_gemm(fmt, pa.ptr + p * M * ra, ra, sa.ptr + p * (M // 128) * katoms * 512,
                        pb.ptr + p * n * rb, rb, sb.ptr + p * (n // 128) * katoms * 512, one.ptr, M, n, K,
                        out_bf16=bf16, ldc_m=lay["ldc_m"], ldc_n=lay["ldc_n"], beta_one=init is not None)
        N.raise_device_status()
        block = got[p * lay["batch_stride_c"]: p * lay["batch_stride_c"] + M * n]
        np.testing.assert_array_equal(block, to_host(one, M * n, hdt), err_msg=f"problem {p}")
        want = da[p * M:(p + 1) * M].astype(np.float64) @ db[p * n:(p + 1) * n].astype(np.float64).T
        if init is not None:
            want += 1.0
        err = rel_frobenius(as_matrix(block, kind, n, bf16), want)
        assert err <= (4e-3 if bf16 else TOL), (p, err)
    if kind == "gapped":  # the gaps between the results stay untouched
        for p in range(BATCH - 1):
            gap = got[p * lay["batch_stride_c"] + M * n:(p + 1) * lay["batch_stride_c"]]
            assert not gap.any()


def test_batch_arguments_are_checked():
    from strideweave_b200 import kernels

    (pa, sa, ra), (pb, sb, rb), _, _ = operands(O.E4M3, M, 256, K, seed=32)
    c = empty(4 * M * 256, fill=0)
    kernels.mx_gemm_batched(O.E4M3, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, 0, M, 256, K)  # no-op
    with pytest.raises(ValueError):
        kernels.mx_gemm_batched(O.E4M3, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, -1, M, 256, K)
    with pytest.raises(ValueError):
        kernels.mx_gemm_batched(O.E4M3, pa.ptr, ra, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, 2, M, 256, K,
                                batch_stride_c=-5)
    assert not to_host(c, M * 256, np.float32).any()
