"""The sharded MX contraction on the device (MXShardedContraction), against
one contraction of the whole problem.

* One rank: the M-split and the chunked K-split reproduce the single
  contraction bit for bit (each output tile is the same tile with the same
  K order).
* Two ranks, where the box has two GPUs: the M-split rows match bit for bit;
  the K-split sums two K halves in another order, so it is held to the
  path's 2e-3 relative Frobenius bound.  The collective runs through
  torch.distributed, then through the C-ABI NCCL communicator, with the same
  result.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

M, NN, K = 512, 1024, 2048


def operand(seed: int, rows: int, cols: int, sigma: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((rows, cols)) * sigma).astype(np.float32)


def planes(fmt: int, x: np.ndarray):
    """Device (payload, scales) of x quantised along its rows' K (TC128 scales)."""
    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels

    rows, k = x.shape
    rb = kernels.mx_row_bytes(fmt, k)
    src = N.DeviceBuffer(x.nbytes)
    src.upload(np.ascontiguousarray(x))
    pay = N.DeviceBuffer(rows * rb)
    sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, k // 32))
    kernels.mx_quantize(fmt, src.ptr, rows, k, k, 1, pay.ptr, rb, sc.ptr)
    N.synchronize()
    return pay, sc


def full_contraction(fmt: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    import torch

    from strideweave_b200 import kernels

    pa, sa = planes(fmt, a)
    pb, sb = planes(fmt, b)
    rb = kernels.mx_row_bytes(fmt, a.shape[1])
    c = torch.empty(a.shape[0] * b.shape[0], dtype=torch.float32, device="cuda")
    kernels.mx_gemm(fmt, pa.ptr, rb, sa.ptr, pb.ptr, rb, sb.ptr, c.data_ptr(), a.shape[0], b.shape[0], a.shape[1])
    torch.cuda.synchronize()
    return c.cpu().numpy().reshape(a.shape[0], b.shape[0])


def ksplit_rows(plan, outs) -> np.ndarray:
    """The rank's C rows [M/g, N] from the chunk-major outputs."""
    return np.concatenate([o.cpu().numpy().reshape(plan.rows_local, plan.chunk_cols) for o in outs], axis=1)


@pytest.mark.parametrize("fmt_name", ["E4M3", "E2M1"])
def test_one_rank_splits_equal_one_contraction(fmt_name):
    import torch

    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import MXShardedContraction, ShardPlan

    fmt = N.SW_MX_E4M3 if fmt_name == "E4M3" else N.SW_MX_E2M1
    q = 128 if fmt == N.SW_MX_E4M3 else 256
    a, b = operand(1, M, K), operand(2, NN, K, 0.02)
    want = full_contraction(fmt, a, b)
    pa, pb = planes(fmt, a), planes(fmt, b)
    m_op = MXShardedContraction(ShardPlan("m", 1, 0, M, NN, K, k_quantum=q), fmt, pa, pb)
    got_m = m_op.run()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got_m.cpu().numpy().reshape(M, NN), want)
    plan = ShardPlan("k", 1, 0, M, NN, K, k_quantum=q, chunks=4)
    got_k = ksplit_rows(plan, MXShardedContraction(plan, fmt, pa, pb).run())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got_k, want)


def _rank(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import MXShardedContraction, NcclCommunicator, ShardPlan

    try:
        torch.cuda.set_device(rank)
        N.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        fmt = N.SW_MX_E4M3
        a, b = operand(1, M, K), operand(2, NN, K, 0.02)
        mp = ShardPlan("m", world, rank, M, NN, K)
        rows = slice(mp.row0, mp.row0 + mp.rows_local)
        got_m = MXShardedContraction(mp, fmt, planes(fmt, a[rows]), planes(fmt, b)).run()
        kp = ShardPlan("k", world, rank, M, NN, K, chunks=2)
        ks = slice(kp.k0, kp.k0 + kp.k_local)
        pa, pb = planes(fmt, np.ascontiguousarray(a[:, ks])), planes(fmt, np.ascontiguousarray(b[:, ks]))
        got_k = ksplit_rows(kp, MXShardedContraction(kp, fmt, pa, pb).run())
        # the same K-split with the collective through the C-ABI communicator
        ids = [NcclCommunicator.new_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        comm = NcclCommunicator(world, rank, ids[0])
        got_c = ksplit_rows(kp, MXShardedContraction(kp, fmt, pa, pb, comm=comm).run())
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        results.put((rank, mp.row0, got_m.cpu().numpy().reshape(mp.rows_local, NN), got_k, got_c))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, repr(exc), None, None, None))


def test_two_rank_splits_match_one_contraction():
    import torch
    import torch.multiprocessing as mp

    from strideweave_b200 import _native as N

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            item = results.get(timeout=240)
            got[item[0]] = item[1:]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    a, b = operand(1, M, K), operand(2, NN, K, 0.02)
    want = full_contraction(N.SW_MX_E4M3, a, b)
    for rank in range(world):
        row0, m_rows, k_rows, c_rows = got[rank]
        assert m_rows is not None, row0  # the rank's exception
        block = want[row0:row0 + M // world]
        np.testing.assert_array_equal(m_rows, block)
        err = np.linalg.norm(k_rows - block) / np.linalg.norm(block)
        assert err <= 2e-3, err
        np.testing.assert_array_equal(c_rows, k_rows)
