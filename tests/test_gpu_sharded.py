"""The sharded MX contraction on the device (MXShardedContraction), against
one contraction of the whole problem.

* One rank: the M-split and the chunked K-split reproduce the single
  contraction bit for bit (each output tile is the same tile with the same
  K order), and the result is a CUDA-carrier tensor with the documented
  row-major / chunk-major layout.
* Two ranks, where the box has two GPUs: the M-split rows match bit for bit;
  the K-split sums two K halves in another order, so it is held to the
  path's 2e-3 relative Frobenius bound.  The reduce-scatter runs through the
  C-ABI NCCL communicator; nothing on the data path uses torch.  The
  host-streamed M-split, each rank copying half of B's rows and the
  quantised halves all-gathered, gives the same rows bit for bit.
"""

from __future__ import annotations

import multiprocessing
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

M, NN, K = 512, 1024, 2048
TOL = 2e-3


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
    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels

    pa, sa = planes(fmt, a)
    pb, sb = planes(fmt, b)
    rb = kernels.mx_row_bytes(fmt, a.shape[1])
    c = N.DeviceBuffer(4 * a.shape[0] * b.shape[0])
    kernels.mx_gemm(fmt, pa.ptr, rb, sa.ptr, pb.ptr, rb, sb.ptr, c.ptr, a.shape[0], b.shape[0], a.shape[1])
    out = np.empty((a.shape[0], b.shape[0]), np.float32)
    N.synchronize()
    c.download(out)
    return out


def ksplit_rows(plan, result) -> np.ndarray:
    """The rank's C rows [M/g, N] from the chunk-major result tensor."""
    flat = result.carrier.to_numpy()
    blocks = flat.reshape(plan.chunks, plan.rows_local, plan.chunk_cols)
    return np.concatenate(list(blocks), axis=1)


@pytest.mark.parametrize("fmt_name", ["E4M3", "E2M1"])
def test_one_rank_splits_equal_one_contraction(fmt_name):
    from strideweave import Layout, Shape, Stride

    from strideweave_b200 import CUDA
    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import MXShardedContraction, ShardPlan

    fmt = N.SW_MX_E4M3 if fmt_name == "E4M3" else N.SW_MX_E2M1
    a, b = operand(1, M, K), operand(2, NN, K, 0.02)
    want = full_contraction(fmt, a, b)
    pa, pb = planes(fmt, a), planes(fmt, b)
    m_op = MXShardedContraction(ShardPlan("m", 1, 0, M, NN, K), fmt, pa, pb)
    got_m = m_op.run()
    assert isinstance(got_m.carrier, CUDA)
    assert got_m.layout == Layout(Shape([M, NN]), Stride([NN, 1]))
    np.testing.assert_array_equal(got_m.carrier.to_numpy().reshape(M, NN), want)
    plan = ShardPlan("k", 1, 0, M, NN, K, chunks=4)
    op = MXShardedContraction(plan, fmt, pa, pb)
    got = op.run()
    nc = NN // 4
    assert got.layout == Layout(Shape([M, [nc, 4]]), Stride([nc, [1, M * nc]]))
    np.testing.assert_array_equal(ksplit_rows(plan, got), want)
    # a second step on the same buffers gives the same result
    np.testing.assert_array_equal(ksplit_rows(plan, op.run()), want)
    op.close()
    # the peer-memory transport at one rank: the routed contraction lands in
    # the rank's own slot and the slot sum is a copy
    pp = ShardPlan("k", 1, 0, M, NN, K)
    peer = MXShardedContraction(pp, fmt, pa, pb, transport="peer")
    for _ in range(2):
        got = peer.run()
        assert got.layout == Layout(Shape([M, NN]), Stride([NN, 1]))
        np.testing.assert_array_equal(got.carrier.to_numpy().reshape(M, NN), want)
    N.raise_device_status()
    peer.close()


@pytest.mark.parametrize("fmt_name", ["E4M3", "E2M1"])
def test_host_streamed_msplit_equals_one_contraction(fmt_name):
    """run_from_host: Float32 A and B in pinned host memory, copied, quantised
    and contracted block by block, C copied back while later blocks arrive;
    the host C equals the single contraction of the same operands bit for
    bit, on two steps in a row (new data in the second), and the block size
    is checked before anything is enqueued."""
    import torch

    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels
    from strideweave_b200.sharding import MXShardedContraction, ShardPlan

    fmt = N.SW_MX_E4M3 if fmt_name == "E4M3" else N.SW_MX_E2M1
    rows, k = 1024, K
    rb = kernels.mx_row_bytes(fmt, k)
    pa = (N.DeviceBuffer(rows * rb), N.DeviceBuffer(kernels.scale_bytes_tc128(rows, k // 32)))
    pb = (N.DeviceBuffer(NN * rb), N.DeviceBuffer(kernels.scale_bytes_tc128(NN, k // 32)))
    op = MXShardedContraction(ShardPlan("m", 1, 0, rows, NN, k), fmt, pa, pb)
    for chunk in (100, 384, 0):
        with pytest.raises(ValueError):
            op.run_from_host(1, 1, 1, chunk_rows=chunk)
    host_c = torch.empty((rows, NN), dtype=torch.float32).pin_memory()
    for seed in (11, 12):
        a, b = operand(seed, rows, k), operand(seed + 100, NN, k, 0.02)
        host_a = torch.from_numpy(a).pin_memory()
        host_b = torch.from_numpy(b).pin_memory()
        op.run_from_host(host_a.data_ptr(), host_b.data_ptr(), host_c.data_ptr(), chunk_rows=256)
        N.synchronize()
        N.raise_device_status()
        np.testing.assert_array_equal(host_c.numpy(), full_contraction(fmt, a, b))
        # the device result carrier holds the same rows
        np.testing.assert_array_equal(op.result.carrier.to_numpy().reshape(rows, NN), host_c.numpy())
    op.close()


def test_multi_rank_ksplit_needs_a_communicator():
    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import MXShardedContraction, ShardPlan

    with pytest.raises(ValueError, match="NcclCommunicator"):
        MXShardedContraction(ShardPlan("k", 2, 0, M, NN, K, chunks=2), N.SW_MX_E4M3, (16, 16), (16, 16))


def _rank(rank: int, world: int, ids, results) -> None:
    # torch (the pinned host buffers of the streamed step) loads its own NCCL;
    # it is imported before the C-ABI communicator opens NCCL, as in bench.py
    import torch

    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import MXShardedContraction, NcclCommunicator, ShardPlan

    try:
        N.set_device(rank)
        if rank == 0:
            nccl_id = NcclCommunicator.new_id()
            for _ in range(world - 1):
                ids.put(nccl_id)
        else:
            nccl_id = ids.get(timeout=60)
        comm = NcclCommunicator(world, rank, nccl_id)
        fmt = N.SW_MX_E4M3
        a, b = operand(1, M, K), operand(2, NN, K, 0.02)
        mp = ShardPlan("m", world, rank, M, NN, K)
        rows = slice(mp.row0, mp.row0 + mp.rows_local)
        got_m = MXShardedContraction(mp, fmt, planes(fmt, a[rows]), planes(fmt, b)).run()
        kp = ShardPlan("k", world, rank, M, NN, K, chunks=2)
        ks = slice(kp.k0, kp.k0 + kp.k_local)
        pa, pb = planes(fmt, np.ascontiguousarray(a[:, ks])), planes(fmt, np.ascontiguousarray(b[:, ks]))
        op = MXShardedContraction(kp, fmt, pa, pb, comm=comm)
        got_k = ksplit_rows(kp, op.run())
        again = ksplit_rows(kp, op.run())
        N.synchronize()
        op.close()
        # the peer-memory transport: row blocks written into the owners'
        # slots over NVLink, slots summed in rank order (three steps, so the
        # step flags cycle through the slot reuse)
        pp = ShardPlan("k", world, rank, M, NN, K)
        peer = MXShardedContraction(pp, fmt, pa, pb, comm=comm, transport="peer")
        peers = [peer.run().carrier.to_numpy().reshape(pp.rows_local, NN) for _ in range(3)]
        N.raise_device_status()
        peer.close()
        # the host-streamed M-split: this rank copies its A rows and its half
        # of B's rows from host memory; the quantised B halves are all-gathered
        from strideweave_b200 import kernels

        rb = kernels.mx_row_bytes(fmt, K)
        hp_a = (N.DeviceBuffer(mp.rows_local * rb), N.DeviceBuffer(kernels.scale_bytes_tc128(mp.rows_local, K // 32)))
        hp_b = (N.DeviceBuffer(NN * rb), N.DeviceBuffer(kernels.scale_bytes_tc128(NN, K // 32)))
        hop = MXShardedContraction(mp, fmt, hp_a, hp_b, comm=comm)
        host_a = torch.from_numpy(np.ascontiguousarray(a[rows])).pin_memory()
        host_b = torch.from_numpy(b).pin_memory()
        host_c = torch.empty((mp.rows_local, NN), dtype=torch.float32).pin_memory()
        streamed = []
        for _ in range(2):
            hop.run_from_host(host_a.data_ptr(), host_b.data_ptr(), host_c.data_ptr(), chunk_rows=128)
            N.synchronize()
            streamed.append(host_c.numpy().copy())
        N.raise_device_status()
        hop.close()
        comm.close()
        results.put((rank, mp.row0, got_m.carrier.to_numpy().reshape(mp.rows_local, NN), got_k, again, peers,
                     streamed))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, repr(exc), None, None, None, None, None))


def test_two_rank_splits_match_one_contraction():
    from strideweave_b200 import _native as N

    if N.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = multiprocessing.get_context("spawn")
    ids, results = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, ids, results)) for r in range(world)]
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
        row0, m_rows, k_rows, again, peers, streamed = got[rank]
        assert m_rows is not None, row0  # the rank's exception
        block = want[row0:row0 + M // world]
        np.testing.assert_array_equal(m_rows, block)
        for c in streamed:  # B sliced over the ranks and all-gathered: the same rows, bit for bit
            np.testing.assert_array_equal(c, block)
        err = np.linalg.norm(k_rows - block) / np.linalg.norm(block)
        assert err <= TOL, err
        np.testing.assert_array_equal(again, k_rows)  # the same step again, bit for bit
        # two partials sum to the same binary32 in either order: the peer
        # transport equals NCCL's reduce-scatter bit for bit, every step
        for p in peers:
            np.testing.assert_array_equal(p, k_rows)
