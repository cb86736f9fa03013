"""Host logic of the sharded contraction on CPU ranks (gloo, world size 2).

The same schedule that drives the tcgen05 GEMM and NCCL on GPUs runs here
with a numpy chunk contraction and a gloo collective, and every rank's
C rows are checked against A . B^T.  A rank that fails before a collective
must make its peer fail within the process-group timeout, not hang.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from strideweave_b200.sharding import ShardPlan, run_ksplit, run_msplit  # noqa: E402


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def operands(M, N, K, seed=0):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K)), rng.standard_normal((N, K))


def _worker(rank, world, port, mode, M, N, K, chunks, fail_rank, results):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        plan = ShardPlan(mode, world, rank, M, N, K, k_quantum=32, chunks=chunks)
        A, B = operands(M, N, K)
        if mode == "m":
            a_loc = A[plan.row0:plan.row0 + plan.rows_local]
            out = np.empty((plan.rows_local, N))

            def contract(chunk, o, ldc):
                o[:] = a_loc @ B.T

            run_msplit(plan, contract, out)
            results[rank] = ("ok", out.ravel().tolist(), None)
        else:
            a_loc = A[:, plan.k0:plan.k0 + plan.k_local]
            b_loc = B[:, plan.k0:plan.k0 + plan.k_local]
            nc = plan.chunk_cols
            partials = [torch.zeros(M * nc, dtype=torch.float64) for _ in range(2)]
            outs = [torch.zeros(plan.rows_local * nc, dtype=torch.float64) for _ in range(chunks)]

            def contract(c, part, ldc):
                if rank == fail_rank and c == 1:
                    raise RuntimeError("injected failure before chunk 1")
                part.copy_(torch.from_numpy((a_loc @ b_loc[c * nc:(c + 1) * nc].T).ravel()))

            def reduce_scatter(out, part, c):
                # gloo: all-reduce, then keep this rank's row block
                buf = part.clone()
                dist.all_reduce(buf)
                out.copy_(buf.view(M, nc)[plan.row0:plan.row0 + plan.rows_local].reshape(-1))

            run_ksplit(plan, contract, reduce_scatter, partials, outs)
            # assemble the chunk-major storage the result layout describes
            flat = torch.cat(outs).numpy()
            results[rank] = ("ok", flat.tolist(), plan.result_layout_tree())
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, which asserts on it
        results[rank] = ("error", repr(exc), traceback.format_exc())


def run_world(mode, M, N, K, chunks, fail_rank=-1, world=2):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, M, N, K, chunks, fail_rank, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank did not finish within 120 s")
    return dict(results)


def test_plan_partitions_and_validation():
    p = ShardPlan("k", 8, 3, 65536, 16384, 16384, chunks=4)
    assert (p.rows_local, p.row0, p.k_local, p.k0, p.chunk_cols) == (8192, 24576, 2048, 6144, 4096)
    assert p.result_layout_tree() == ([8192, [4096, 4]], [4096, [1, 8192 * 4096]])
    m = ShardPlan("m", 8, 7, 65536, 16384, 16384)
    assert (m.rows_local, m.row0, m.k_local) == (8192, 57344, 16384)
    assert m.local_flops * 8 == pytest.approx(2.0 * 65536 * 16384 * 16384)
    with pytest.raises(ValueError):
        ShardPlan("k", 8, 0, 65536, 16384, 16384 + 128)
    with pytest.raises(ValueError):
        ShardPlan("m", 3, 0, 1024, 256, 256)
    with pytest.raises(ValueError):
        ShardPlan("x", 2, 0, 256, 256, 256)


def test_msplit_two_ranks_cover_c():
    M, N, K = 512, 256, 192
    res = run_world("m", M, N, K, chunks=1)
    A, B = operands(M, N, K)
    want = A @ B.T
    for r in range(2):
        status, flat, _ = res[r]
        assert status == "ok", flat
        np.testing.assert_allclose(np.array(flat).reshape(256, N), want[r * 256:(r + 1) * 256], rtol=1e-12)


def test_ksplit_two_ranks_reduce_scatter_chunked():
    sw = pytest.importorskip("strideweave")
    M, N, K, chunks = 512, 512, 256, 4
    res = run_world("k", M, N, K, chunks)
    A, B = operands(M, N, K)
    want = A @ B.T
    for r in range(2):
        status, flat, tree = res[r]
        assert status == "ok", flat
        layout = sw.Layout(sw.Shape(tree[0]), sw.Stride(tree[1]))
        flat = np.array(flat)
        got = np.array([[flat[layout.index((i, j))] for j in range(N)] for i in range(256)])
        np.testing.assert_allclose(got, want[r * 256:(r + 1) * 256], rtol=1e-12, atol=1e-12)


def test_a_failing_rank_makes_its_peer_fail_not_hang():
    res = run_world("k", 512, 512, 256, chunks=4, fail_rank=1)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # rank 0 waits in the chunk-1 collective for a peer that never joins: the
    # 5 s process-group timeout (or the peer's exit) ends it with an error
    assert res[0][0] == "error"
