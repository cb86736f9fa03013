"""NCCL through the C ABI (sw_nccl_*): a one-rank communicator on any GPU,
and, where the box has two GPUs, a reduce-scatter and an all-gather between
two processes whose communicators come from one id that rank 0 created."""

from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_one_rank_collectives_are_copies():
    import torch

    from strideweave_b200.sharding import NcclCommunicator

    comm = NcclCommunicator(1, 0, NcclCommunicator.new_id())
    x = torch.arange(1000, dtype=torch.float32, device="cuda")
    out = torch.empty_like(x)
    comm.reduce_scatter_f32(out.data_ptr(), x.data_ptr(), x.numel())
    torch.cuda.synchronize()
    assert torch.equal(out, x)
    gathered = torch.empty_like(x)
    comm.all_gather_f32(gathered.data_ptr(), x.data_ptr(), x.numel())
    torch.cuda.synchronize()
    assert torch.equal(gathered, x)
    comm.close()


def _rank(rank: int, world: int, n: int, ids, results) -> None:
    import torch

    from strideweave_b200 import _native as N
    from strideweave_b200.sharding import NcclCommunicator

    try:
        torch.cuda.set_device(rank)
        N.set_device(rank)
        if rank == 0:
            nccl_id = NcclCommunicator.new_id()
            for _ in range(world - 1):
                ids.put(nccl_id)
        else:
            nccl_id = ids.get(timeout=60)
        comm = NcclCommunicator(world, rank, nccl_id)
        send = torch.arange(world * n, dtype=torch.float32, device="cuda") + 10.0 * rank
        recv = torch.empty(n, dtype=torch.float32, device="cuda")
        comm.reduce_scatter_f32(recv.data_ptr(), send.data_ptr(), n)
        gathered = torch.empty(world * n, dtype=torch.float32, device="cuda")
        comm.all_gather_f32(gathered.data_ptr(), recv.data_ptr(), n)
        torch.cuda.synchronize()
        comm.close()
        results.put((rank, recv.cpu().numpy(), gathered.cpu().numpy()))
    except Exception as exc:  # reported to the parent, which fails the test
        results.put((rank, repr(exc), None))


def test_two_rank_reduce_scatter_and_all_gather():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, n = 2, 4096
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    ids, results = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, n, ids, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, recv, gathered = results.get(timeout=180)
            got[rank] = (recv, gathered)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    base = np.arange(world * n, dtype=np.float64)
    want_gathered = np.concatenate([sum(base[r * n:(r + 1) * n] + 10.0 * q for q in range(world))
                                    for r in range(world)])
    for rank in range(world):
        recv, gathered = got[rank]
        assert gathered is not None, recv  # the rank's exception
        np.testing.assert_array_equal(recv, want_gathered[rank * n:(rank + 1) * n].astype(np.float32))
        np.testing.assert_array_equal(gathered, want_gathered.astype(np.float32))
