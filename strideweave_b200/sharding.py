"""Sharded MX contraction across the GPUs of one node (one process per GPU).

Two partitions of C[M, N] = A[M, K] . B[N, K]^T:

* **M-split.** Rank r owns the A rows [r*M/g, (r+1)*M/g) and a replica of B.
  It computes its own C row block. There is no collective on the data path.
* **K-split.** Rank r owns A[:, Kr] and B[:, Kr] for its K slice and computes
  a full Float32 partial C. The partials are summed with a reduce-scatter
  over NVLink, so rank r ends with the C rows [r*M/g, (r+1)*M/g).
  - N is cut into `chunks` column blocks. Block c's reduce-scatter runs on a
    communication stream while block c+1 is contracted, so communication
    overlaps the tensor cores. The persistent contraction would otherwise
    hold every SM (one CTA with ~220 KB of shared memory each), and the
    collective's kernels could not start beside it. So a K-split's
    contractions run on all but `comm_sms` SMs (32 measured best on two
    GPUs: 3.17 against 2.61 PFLOP/s with none left).
  - Each chunk partial is a row-major [M, Nc] buffer, so its row blocks are
    contiguous and can be scattered to the ranks as they are.
  - The local result is stored chunk-major. Element (m, n) sits at
    (n // Nc) * (M/g * Nc) + m * Nc + n % Nc, which is the StrideWeave layout
    (M/g, (Nc, chunks)) : (Nc, (1, M/g * Nc)). The carrier tiles its flat
    index space without a gather.

The schedule is written once, against three callables: a chunk contraction,
a reduce-scatter and an allocator. On GPUs these are the tcgen05 MX GEMM and
NCCL (through `torch.distributed`). The CPU tests run the same schedule with
numpy and `gloo`.

The reference has no distributed code: it runs every operation on one host
carrier.  This module shards large contractions across the GPUs of a node by
M-split, or by K-split with an NCCL reduce-scatter.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

ROW_TILE = 128  # the contraction's M / N tile


@dataclass(frozen=True)
class ShardPlan:
    """Partition of one contraction across `world` ranks (see module doc)."""

    mode: str  # "m" or "k"
    world: int
    rank: int
    M: int
    N: int
    K: int
    k_quantum: int = 128  # K granularity of the MX kernel (128 E4M3, 256 E2M1)
    chunks: int = 1
    comm_sms: int = 32  # SMs a K-split's contractions leave to the overlapping reduce-scatter

    def __post_init__(self) -> None:
        if self.mode not in ("m", "k"):
            raise ValueError("mode must be 'm' (M-split) or 'k' (K-split)")
        if not 0 <= self.rank < self.world:
            raise ValueError("rank out of range")
        if self.M % (self.world * ROW_TILE) != 0:
            raise ValueError(f"M={self.M} must split into {self.world} blocks of whole {ROW_TILE}-row tiles")
        if self.mode == "k" and self.K % (self.world * self.k_quantum) != 0:
            raise ValueError(f"K={self.K} must split into {self.world} slices of whole {self.k_quantum}-blocks")
        if self.chunks < 1 or self.N % (self.chunks * ROW_TILE) != 0:
            raise ValueError(f"N={self.N} must split into {self.chunks} chunks of whole {ROW_TILE}-column tiles")

    @property
    def rows_local(self) -> int:
        return self.M // self.world

    @property
    def row0(self) -> int:
        return self.rank * self.rows_local

    @property
    def k_local(self) -> int:
        return self.K if self.mode == "m" else self.K // self.world

    @property
    def k0(self) -> int:
        return 0 if self.mode == "m" else self.rank * self.k_local

    @property
    def chunk_cols(self) -> int:
        return self.N // self.chunks

    @property
    def local_flops(self) -> float:
        rows = self.rows_local if self.mode == "m" else self.M
        return 2.0 * rows * self.N * self.k_local

    def result_layout_tree(self) -> tuple[list[Any], list[Any]]:
        """(shape, stride) trees of the local result C rows (chunk-major)."""
        mg, nc = self.rows_local, self.chunk_cols
        if self.mode == "m" or self.chunks == 1:
            return [mg, self.N], [self.N, 1]
        return [mg, [nc, self.chunks]], [nc, [1, mg * nc]]


# contract(chunk, out_handle, ldc): C[rows, chunk cols] into out (row-major, ldc)
ChunkContract = Callable[[int, Any, int], None]
# reduce_scatter(out_handle, in_handle, chunk): sum over ranks, rank r gets rows block r
ReduceScatter = Callable[[Any, Any, int], None]


def run_msplit(plan: ShardPlan, contract: ChunkContract, out: Any) -> Any:
    """M-split: one local contraction into `out` ([rows_local, N] row-major)."""
    if plan.mode != "m":
        raise ValueError("run_msplit needs an M-split plan")
    contract(-1, out, plan.N)
    return out


def run_ksplit(plan: ShardPlan, contract: ChunkContract, reduce_scatter: ReduceScatter,
               partials: list[Any], outs: list[Any], *, before_comm: Callable[[int], None] | None = None,
               after_all: Callable[[], None] | None = None) -> list[Any]:
    """K-split schedule: contract chunk c into partials[c] ([M, Nc] row-major),
    then reduce-scatter it into outs[c] ([M/g, Nc]); `before_comm(c)` orders
    the collective after chunk c's contraction (a stream event on GPUs)."""
    if plan.mode != "k":
        raise ValueError("run_ksplit needs a K-split plan")
    if len(partials) < 1 or len(outs) != plan.chunks:
        raise ValueError("one output per chunk and at least one partial buffer")
    for c in range(plan.chunks):
        part = partials[c % len(partials)]
        contract(c, part, plan.chunk_cols)
        if before_comm is not None:
            before_comm(c)
        reduce_scatter(outs[c], part, c)
    if after_all is not None:
        after_all()
    return outs


# ---- NCCL through the C ABI ---------------------------------------------------------


class NcclCommunicator:
    """One rank's NCCL communicator created through the C ABI (``sw_nccl_*``),
    for a sharded contraction driven without torch.distributed.  Rank 0
    creates the id with ``new_id()``; the host hands the same bytes to every
    rank (any channel the ranks share), and each rank builds its communicator
    with its device current."""

    def __init__(self, world: int, rank: int, nccl_id: bytes) -> None:
        from . import _native as N

        if len(nccl_id) != N.SW_NCCL_ID_BYTES:
            raise ValueError(f"an NCCL id is {N.SW_NCCL_ID_BYTES} bytes")
        self._N = N
        self.world, self.rank = world, rank
        buf = (N.ctypes.c_uint8 * N.SW_NCCL_ID_BYTES).from_buffer_copy(nccl_id)
        comm = N.c_void_p()
        N.check(N.lib.sw_nccl_comm_init(N.ctypes.byref(comm), world, rank, buf))
        self._comm = comm.value

    @staticmethod
    def new_id() -> bytes:
        from . import _native as N

        buf = (N.ctypes.c_uint8 * N.SW_NCCL_ID_BYTES)()
        N.check(N.lib.sw_nccl_get_unique_id(buf))
        return bytes(buf)

    def reduce_scatter_f32(self, out_ptr: int, in_ptr: int, recv_count: int, stream: int = 0) -> None:
        """out[i] = sum over ranks of in[rank * recv_count + i]."""
        N = self._N
        N.check(N.lib.sw_nccl_reduce_scatter_f32(N.c_void_p(in_ptr), N.c_void_p(out_ptr), int(recv_count),
                                                 N.c_void_p(self._comm), N.c_void_p(stream or None)))

    def all_gather_f32(self, out_ptr: int, in_ptr: int, send_count: int, stream: int = 0) -> None:
        """out[r * send_count + i] = in of rank r, element i."""
        N = self._N
        N.check(N.lib.sw_nccl_all_gather_f32(N.c_void_p(in_ptr), N.c_void_p(out_ptr), int(send_count),
                                             N.c_void_p(self._comm), N.c_void_p(stream or None)))

    def close(self) -> None:
        if self._comm is not None:
            self._N.check(self._N.lib.sw_nccl_comm_destroy(self._N.c_void_p(self._comm)))
            self._comm = None


# ---- the GPU implementation ---------------------------------------------------------


class MXShardedContraction:
    """Sharded MX contraction on this rank's GPU: tcgen05 MX GEMM for the local
    products, NCCL (torch.distributed, backend "nccl") for the reduce-scatter.

    `a_planes` / `b_planes` are this rank's operand shards as (payload, scales)
    device buffers in the tensor-core placement: A rows [rows, k_local]
    (M-split: rows = M/g; K-split: rows = M) and B [N, k_local].
    """

    def __init__(self, plan: ShardPlan, fmt: int, a_planes: tuple[Any, Any], b_planes: tuple[Any, Any],
                 group: Any = None, comm: NcclCommunicator | None = None) -> None:
        import torch

        from . import _native as N
        from . import kernels

        self.plan = plan
        self.fmt = fmt
        self.N = N
        self.kernels = kernels
        self.torch = torch
        self.group = group
        self.comm = comm  # reduce-scatter through the C ABI instead of torch.distributed
        self.a_pay, self.a_sc = a_planes
        self.b_pay, self.b_sc = b_planes
        self.row_bytes = kernels.mx_row_bytes(fmt, plan.k_local)
        self.katoms = (plan.k_local // 32 + 3) // 4
        dev = torch.device("cuda", torch.cuda.current_device())
        rows = plan.rows_local if plan.mode == "m" else plan.M
        if plan.mode == "m":
            self.out = torch.empty(plan.rows_local * plan.N, dtype=torch.float32, device=dev)
        else:
            nbuf = min(2, plan.chunks)  # double-buffered partials
            self.partials = [torch.empty(rows * plan.chunk_cols, dtype=torch.float32, device=dev)
                             for _ in range(nbuf)]
            self.outs = [torch.empty(plan.rows_local * plan.chunk_cols, dtype=torch.float32, device=dev)
                         for _ in range(plan.chunks)]
            self.comm_stream = torch.cuda.Stream(device=dev)
            self.done = [torch.cuda.Event() for _ in range(plan.chunks)]
            self.freed = [torch.cuda.Event() for _ in range(plan.chunks)]

    def _contract(self, chunk: int, out: Any, ldc: int) -> None:
        plan = self.plan
        s = self.torch.cuda.current_stream().cuda_stream
        rows = plan.rows_local if plan.mode == "m" else plan.M
        if chunk < 0:
            n0, ncols = 0, plan.N
        else:
            n0, ncols = chunk * plan.chunk_cols, plan.chunk_cols
        b_ptr = self.b_pay.ptr + n0 * self.row_bytes
        b_sc = self.b_sc.ptr + (n0 // 128) * self.katoms * 512
        # a K-split's reduce-scatter of the previous chunk runs beside this
        # contraction: leave it some SMs (the persistent GEMM fills every SM)
        max_ctas = 0
        if plan.mode == "k" and plan.world > 1 and plan.chunks > 1 and plan.comm_sms > 0:
            sms = self.torch.cuda.get_device_properties(self.torch.cuda.current_device()).multi_processor_count
            max_ctas = max(1, sms - plan.comm_sms)
        self.kernels.mx_gemm(self.fmt, self.a_pay.ptr, self.row_bytes, self.a_sc.ptr, b_ptr, self.row_bytes, b_sc,
                             out.data_ptr(), rows, ncols, plan.k_local, ldc_m=ldc, ldc_n=1, max_ctas=max_ctas,
                             stream=s)

    def run(self) -> Any:
        plan = self.plan
        torch = self.torch
        if plan.mode == "m":
            return run_msplit(plan, self._contract, self.out)
        import torch.distributed as dist

        compute = torch.cuda.current_stream()

        def before_comm(c: int) -> None:
            self.done[c].record(compute)
            self.comm_stream.wait_event(self.done[c])

        def reduce_scatter(out: Any, part: Any, c: int) -> None:
            with torch.cuda.stream(self.comm_stream):
                if self.comm is not None:
                    self.comm.reduce_scatter_f32(out.data_ptr(), part.data_ptr(), out.numel(),
                                                 self.comm_stream.cuda_stream)
                elif plan.world == 1:
                    out.copy_(part)
                else:
                    dist.reduce_scatter_tensor(out, part, op=dist.ReduceOp.SUM, group=self.group)
                self.freed[c].record(self.comm_stream)

        def contract(c: int, part: Any, ldc: int) -> None:
            if c >= len(self.partials):  # the buffer is reused: wait until its scatter finished
                compute.wait_event(self.freed[c - len(self.partials)])
            self._contract(c, part, ldc)

        def after_all() -> None:
            compute.wait_stream(self.comm_stream)

        return run_ksplit(plan, contract, reduce_scatter, self.partials, self.outs, before_comm=before_comm,
                          after_all=after_all)
