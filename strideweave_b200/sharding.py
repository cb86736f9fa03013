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
NCCL, both through the C ABI (no torch on the data path: carrier storage,
streams and events are the library's own). The CPU tests run the same
schedule with numpy and `gloo`.

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


def _address(buf: Any) -> int:
    """Device address of a buffer handle: a CUDA carrier, a DeviceBuffer or an int."""
    if isinstance(buf, int):
        return buf
    if hasattr(buf, "data_ptr"):
        ptr = buf.data_ptr
        return ptr() if callable(ptr) else int(ptr)
    return int(buf.ptr)


class MXShardedContraction:
    """Sharded MX contraction on this rank's GPU, driven entirely through the
    C ABI: the tcgen05 MX GEMM for the local products and, for a K-split over
    several ranks, the C-ABI NCCL communicator for the reduce-scatter.

    `a_planes` / `b_planes` are this rank's operand shards as (payload, scales)
    device buffers (CUDA carriers, DeviceBuffers or addresses) in the
    tensor-core placement: A rows [rows, k_local] (M-split: rows = M/g;
    K-split: rows = M) and B [N, k_local].

    The result lives on a CUDA carrier of this device: the rank's C rows
    [M/g, N] in Float32, row-major for an M-split and chunk-major
    (M/g, (Nc, chunks)) : (Nc, (1, M/g * Nc)) for a K-split, so each chunk's
    reduce-scatter writes one contiguous block.  `run()` enqueues a step on
    `stream` (default: the legacy default stream, where every carrier
    operation is ordered) and returns that Tensor; the buffers are reused by
    every step.
    """

    def __init__(self, plan: ShardPlan, fmt: int, a_planes: tuple[Any, Any], b_planes: tuple[Any, Any],
                 comm: NcclCommunicator | None = None, stream: int = 0, transport: str = "nccl") -> None:
        from . import _native as N
        from . import kernels
        from ._host import DType, Layout, Shape, Stride, Tensor
        from .carrier import CUDA

        if transport not in ("nccl", "peer"):
            raise ValueError("transport must be 'nccl' (chunked reduce-scatter) or 'peer' (NVLink peer stores)")
        if plan.mode == "k" and plan.world > 1 and comm is None:
            raise ValueError("a K-split over several ranks needs an NcclCommunicator for its reduce-scatter")
        if comm is not None and (comm.world != plan.world or comm.rank != plan.rank):
            raise ValueError("the communicator's world and rank must match the plan's")
        if transport == "peer" and plan.mode == "k" and plan.chunks != 1:
            raise ValueError("the peer K-split writes whole rows: plan one chunk")
        self.transport = transport if plan.mode == "k" else "nccl"
        self.plan, self.fmt, self.comm, self.stream = plan, fmt, comm, int(stream or 0)
        self.N, self.kernels = N, kernels
        self.a_pay, self.a_sc = (_address(x) for x in a_planes)
        self.b_pay, self.b_sc = (_address(x) for x in b_planes)
        self.row_bytes = kernels.mx_row_bytes(fmt, plan.k_local)
        self.katoms = (plan.k_local // 32 + 3) // 4
        dev = N.current_device()
        mg = plan.rows_local
        self.out = CUDA(mg * plan.N, dtype=DType.Float32, empty=True, device=dev)
        shape, stride = plan.result_layout_tree()
        self.result = Tensor(self.out, 0, Layout(Shape(shape), Stride(stride)))
        # a K-split's reduce-scatter of one chunk runs beside the next chunk's
        # contraction: the persistent GEMM then leaves comm_sms SMs free
        self.max_ctas = 0
        if plan.mode == "k" and plan.world > 1 and plan.chunks > 1 and plan.comm_sms > 0:
            self.max_ctas = max(1, N.sm_count() - plan.comm_sms)
        if self.transport == "peer":
            self.landing = PeerLanding(plan.world, plan.rank, plan.rows_local * plan.N, comm)
            self.step = 0
        elif plan.mode == "k":
            nbuf = min(2, plan.chunks)  # double-buffered partials [M, Nc]
            self.partials = [CUDA(plan.M * plan.chunk_cols, dtype=DType.Float32, empty=True, device=dev)
                             for _ in range(nbuf)]
            self.comm_stream = N.Stream()
            self.done = [N.Event() for _ in range(plan.chunks)]
            self.freed = [N.Event() for _ in range(plan.chunks)]
            self.all_done = N.Event()
        # the carriers come from the pool in the legacy default stream's order;
        # the other streams may use them only once that point has passed
        N.synchronize()

    def _contract(self, chunk: int, out_ptr: int, ldc: int) -> None:
        plan = self.plan
        rows = plan.rows_local if plan.mode == "m" else plan.M
        n0, ncols = (0, plan.N) if chunk < 0 else (chunk * plan.chunk_cols, plan.chunk_cols)
        b_ptr = self.b_pay + n0 * self.row_bytes
        b_sc = self.b_sc + (n0 // 128) * self.katoms * 512
        self.kernels.mx_gemm(self.fmt, self.a_pay, self.row_bytes, self.a_sc, b_ptr, self.row_bytes, b_sc, out_ptr,
                             rows, ncols, plan.k_local, ldc_m=ldc, ldc_n=1, max_ctas=self.max_ctas,
                             stream=self.stream)

    def _chunk_out(self, c: int) -> int:
        plan = self.plan
        return self.out.data_ptr + 4 * c * plan.rows_local * plan.chunk_cols

    def run(self) -> Any:
        plan, N = self.plan, self.N
        if plan.mode == "m":
            run_msplit(plan, self._contract, self.out.data_ptr)
            return self.result
        if self.transport == "peer":
            self._run_peer()
            return self.result
        comm_stream = self.comm_stream.handle
        nbuf = len(self.partials)

        def contract(c: int, part: Any, ldc: int) -> None:
            if c >= nbuf:  # the buffer is reused: its previous chunk's collective must have read it
                self.freed[c - nbuf].wait(self.stream)
            self._contract(c, part.data_ptr, ldc)

        def before_comm(c: int) -> None:
            self.done[c].record(self.stream)
            self.done[c].wait(comm_stream)

        def reduce_scatter(out_ptr: int, part: Any, c: int) -> None:
            count = plan.rows_local * plan.chunk_cols
            if self.comm is not None:
                self.comm.reduce_scatter_f32(out_ptr, part.data_ptr, count, comm_stream)
            else:  # one rank: its partial is the sum
                N.check(N.lib.sw_memcpy_d2d(N.c_void_p(out_ptr), N.c_void_p(part.data_ptr), 4 * count,
                                            N.c_void_p(comm_stream)))
            self.freed[c].record(comm_stream)

        def after_all() -> None:
            self.all_done.record(comm_stream)
            self.all_done.wait(self.stream)

        outs = [self._chunk_out(c) for c in range(plan.chunks)]
        run_ksplit(plan, contract, reduce_scatter, self.partials, outs, before_comm=before_comm, after_all=after_all)
        return self.result

    def run_from_host(self, a_host: int, b_host: int, c_host: int, *, chunk_rows: int = 2048) -> Any:
        """One M-split step whose operands and result live in host memory.

        `a_host` holds this rank's Float32 A rows [M/g, K] and `b_host` the
        Float32 B [N, K], both row-major; the rank's Float32 C rows [M/g, N]
        land row-major at `c_host`.  Pinned (page-locked) host memory lets the
        copies run asynchronously; pageable memory works but serialises them.

        The step is a three-stream pipeline over blocks of `chunk_rows` rows:
        a copy stream brings B and then block after block of A to the device,
        the step's stream quantises B once and then, block by block, quantises
        A into this contraction's A planes and contracts the block into the
        result carrier, and a second copy stream returns each finished block of
        C while later blocks are still arriving.  Host-to-device and
        device-to-host copies use the two directions of the link at once, so
        the step costs about the host-to-device time of A and B plus one
        block's contraction and return.  Every block's result equals the one
        `run()` gives from the same planes, bit for bit (each output tile runs
        the same K loop).  Returns the result Tensor, as `run()` does; the
        call only enqueues, so synchronise `stream` before reading `c_host`.

        With several ranks and a communicator, B crosses each rank's host link
        once in all: rank r copies and quantises only B rows
        [r N/g, (r + 1) N/g) and an NCCL all-gather over NVLink assembles the
        quantised B planes on every rank (in place, on the step's stream),
        instead of every rank copying all of B from host memory.
        """
        plan, N, kernels = self.plan, self.N, self.kernels
        if plan.mode != "m":
            raise ValueError("run_from_host streams an M-split; a K-split's operands are per-rank K slices")
        rows, k, n = plan.rows_local, plan.k_local, plan.N
        if chunk_rows <= 0 or chunk_rows % ROW_TILE != 0 or rows % chunk_rows != 0:
            raise ValueError(f"chunk_rows={chunk_rows} must be a whole number of {ROW_TILE}-row tiles dividing the "
                             f"rank's {rows} rows")
        if not (a_host and b_host and c_host):
            raise ValueError("run_from_host needs host addresses for A, B and C")
        st = self._staging(chunk_rows)
        s, h2d, d2h = self.stream, st["h2d"].handle, st["d2h"].handle
        cvp = N.c_void_p
        # B rows this rank brings from host memory: all of them, or its slice
        b_rows, b_row0 = st["b_rows"], st["b_row0"]
        # the copy streams start after everything already enqueued on the step's stream
        st["start"].record(s)
        st["start"].wait(h2d)
        st["start"].wait(d2h)
        N.check(N.lib.sw_memcpy_h2d(cvp(st["b32"].ptr), cvp(b_host + 4 * b_row0 * k), st["b32"].nbytes, cvp(h2d)))
        st["b_ready"].record(h2d)
        block_a = 4 * chunk_rows * k
        for i in range(rows // chunk_rows):
            N.check(N.lib.sw_memcpy_h2d(cvp(st["a32"].ptr + i * block_a), cvp(a_host + i * block_a), block_a,
                                        cvp(h2d)))
            st["a_ready"][i].record(h2d)
        st["b_ready"].wait(s)
        sc_group = self.katoms * 512  # scale bytes of one 128-row group
        kernels.mx_quantize(self.fmt, st["b32"].ptr, b_rows, k, k, 1, self.b_pay + b_row0 * self.row_bytes,
                            self.row_bytes, self.b_sc + (b_row0 // ROW_TILE) * sc_group, stream=s)
        if b_rows != n:
            # in-place all-gathers of the quantised slices (counts in 4-byte words)
            pay_bytes, sc_bytes = b_rows * self.row_bytes, (b_rows // ROW_TILE) * sc_group
            self.comm.all_gather_f32(self.b_pay, self.b_pay + plan.rank * pay_bytes, pay_bytes // 4, s)
            self.comm.all_gather_f32(self.b_sc, self.b_sc + plan.rank * sc_bytes, sc_bytes // 4, s)
        block_c = 4 * chunk_rows * n
        for i in range(rows // chunk_rows):
            r0 = i * chunk_rows
            a_pay = self.a_pay + r0 * self.row_bytes
            a_sc = self.a_sc + (r0 // ROW_TILE) * self.katoms * 512
            st["a_ready"][i].wait(s)
            kernels.mx_quantize(self.fmt, st["a32"].ptr + i * block_a, chunk_rows, k, k, 1, a_pay, self.row_bytes,
                                a_sc, stream=s)
            kernels.mx_gemm(self.fmt, a_pay, self.row_bytes, a_sc, self.b_pay, self.row_bytes, self.b_sc,
                            self.out.data_ptr + i * block_c, chunk_rows, n, k, ldc_m=n, ldc_n=1, stream=s)
            st["c_ready"][i].record(s)
            st["c_ready"][i].wait(d2h)
            # enqueued without a host wait, so the next blocks' work is
            # enqueued while this block's copy runs
            N.check(N.lib.sw_memcpy_d2h_async(cvp(c_host + i * block_c), cvp(self.out.data_ptr + i * block_c),
                                              block_c, cvp(d2h)))
        st["done"].record(d2h)
        st["done"].wait(s)
        return self.result

    def _staging(self, chunk_rows: int) -> dict:
        """Device staging of run_from_host (Float32 A and B), its copy streams
        and events; made on first use for a block size and kept."""
        st = getattr(self, "_host_staging", None)
        if st is not None and st["chunk_rows"] == chunk_rows:
            return st
        N, plan = self.N, self.plan
        blocks = plan.rows_local // chunk_rows
        if st is None:
            # with a communicator each rank brings N/g rows of B (whole 128-row
            # scale groups) and the ranks all-gather the quantised rest
            sliced = self.comm is not None and plan.world > 1 and plan.N % (plan.world * ROW_TILE) == 0
            b_rows = plan.N // plan.world if sliced else plan.N
            st = {"a32": N.DeviceBuffer(4 * plan.rows_local * plan.k_local),
                  "b32": N.DeviceBuffer(4 * b_rows * plan.k_local), "b_rows": b_rows,
                  "b_row0": plan.rank * b_rows if sliced else 0,
                  "h2d": N.Stream(), "d2h": N.Stream(), "start": N.Event(), "b_ready": N.Event(),
                  "done": N.Event()}
            N.synchronize()  # the buffers come from the legacy default stream's pool order
        st["chunk_rows"] = chunk_rows
        st["a_ready"] = [N.Event() for _ in range(blocks)]
        st["c_ready"] = [N.Event() for _ in range(blocks)]
        self._host_staging = st
        return st

    def _run_peer(self) -> None:
        """One K-split step over NVLink peer memory (see PeerLanding): wait
        until every owner has summed this rank's previous contribution,
        contract with each C row block routed into its owner's slot for this
        rank, signal the owners, wait for every writer's signal, sum this
        rank's slots in rank order into the result, free the writers' slots."""
        plan, L, s = self.plan, self.landing, self.stream
        self.step += 1
        e = self.step & 0xFFFFFFFF
        L.wait(L.consumed_flags, e - 1, s)
        # rank r writes owner r + 1's block first and its own last: at any
        # moment each GPU receives from one writer
        self.kernels.mx_gemm_routed(self.fmt, self.a_pay, self.row_bytes, self.a_sc, self.b_pay, self.row_bytes,
                                    self.b_sc, L.dests(), plan.rows_local, plan.N, plan.M, plan.N, plan.k_local,
                                    first=(plan.rank + 1) % plan.world, stream=s)
        L.signal(L.written_flag_of, e, s)
        L.wait(L.written_flags, e, s)
        L.sum_into(self.out.data_ptr, s)
        L.signal(L.consumed_flag_of, e, s)

    def close(self) -> None:
        """Release the streams, events and peer mappings now (the carriers
        free themselves).  Every rank of a peer K-split calls it: it meets the
        others first, so no rank frees memory another still writes."""
        st = getattr(self, "_host_staging", None)
        if st is not None:
            self.N.synchronize(self.stream)
            for e in (st["start"], st["b_ready"], st["done"], *st["a_ready"], *st["c_ready"]):
                e.close()
            st["h2d"].close()
            st["d2h"].close()
            st["a32"].free()
            st["b32"].free()
            self._host_staging = None
        if self.plan.mode != "k":
            return
        if self.transport == "peer":
            self.landing.close()
            return
        for e in (*self.done, *self.freed, self.all_done):
            e.close()
        self.comm_stream.close()


class PeerLanding:
    """This rank's landing buffer of a peer K-split and its view of the
    others' (CUDA IPC within one node).

    One device allocation holds `world` Float32 slots of `slot_elems`
    elements (slot p: rank p's partial of the rows this rank owns) and two
    arrays of `world` 32-bit step flags: written[p] (rank p finished writing
    its slot) and consumed[p] (rank p, an owner, finished summing this rank's
    contribution).  Other ranks write these flags over NVLink; flags only
    grow, so a step waits for "at least e".  The handles are exchanged with an
    all-gather on the NCCL communicator (the only collective the transport
    uses, once, at set-up)."""

    def __init__(self, world: int, rank: int, slot_elems: int, comm: NcclCommunicator | None,
                 wait_limit_ns: int = 5_000_000_000) -> None:
        from . import _native as N

        if world > 8:
            raise NotImplementedError("a peer K-split spans at most the 8 GPUs of one node")
        if slot_elems % 4:
            raise ValueError("slots must hold whole 16-byte vectors")
        self.N, self.world, self.rank = N, world, rank
        self.slot_elems = slot_elems
        self.wait_limit_ns = wait_limit_ns
        self.flags_off = 4 * world * slot_elems
        nbytes = self.flags_off + 8 * world + 256
        handle = (N.ctypes.c_uint8 * N.SW_IPC_HANDLE_BYTES)()
        ptr = N.c_void_p()
        N.check(N.lib.sw_ipc_alloc(N.ctypes.byref(ptr), nbytes, handle))
        self.base = ptr.value
        N.check(N.lib.sw_memset(N.c_void_p(self.base + self.flags_off), 0, 8 * world, None))
        self.peers = [0] * world
        self.peers[rank] = self.base
        self.comm = comm
        if world > 1:
            import numpy as np

            # exchange the 64-byte handles as 16 Float32 words each (an
            # all-gather copies the bits)
            words = N.SW_IPC_HANDLE_BYTES // 4
            mine, everyone = N.DeviceBuffer(4 * words), N.DeviceBuffer(4 * words * world)
            mine.upload(np.frombuffer(bytes(handle), dtype=np.uint8))
            comm.all_gather_f32(everyone.ptr, mine.ptr, words)
            N.synchronize()
            host = np.empty(N.SW_IPC_HANDLE_BYTES * world, dtype=np.uint8)
            everyone.download(host)
            for q in range(world):
                if q == rank:
                    continue
                h = (N.ctypes.c_uint8 * N.SW_IPC_HANDLE_BYTES).from_buffer_copy(
                    host[q * N.SW_IPC_HANDLE_BYTES:(q + 1) * N.SW_IPC_HANDLE_BYTES].tobytes())
                p = N.c_void_p()
                N.check(N.lib.sw_ipc_open(h, N.ctypes.byref(p)))
                self.peers[q] = p.value
            self._rendezvous()  # every rank's flags are zero before any writes them

    @property
    def written_flags(self) -> int:
        return self.base + self.flags_off

    @property
    def consumed_flags(self) -> int:
        return self.base + self.flags_off + 4 * self.world

    def written_flag_of(self, q: int) -> int:
        """Owner q's written[this rank]."""
        return self.peers[q] + self.flags_off + 4 * self.rank

    def consumed_flag_of(self, q: int) -> int:
        """Writer q's consumed[this rank]."""
        return self.peers[q] + self.flags_off + 4 * (self.world + self.rank)

    def dests(self) -> list[int]:
        """Where this rank's row block q goes: owner q's slot for this rank."""
        return [self.peers[q] + 4 * self.rank * self.slot_elems for q in range(self.world)]

    def wait(self, flags: int, target: int, stream: int) -> None:
        N = self.N
        N.check(N.lib.sw_peer_wait(N.c_void_p(flags), self.world, target & 0xFFFFFFFF, self.wait_limit_ns,
                                   N.c_void_p(stream)))

    def signal(self, flag_of: Callable[[int], int], value: int, stream: int) -> None:
        N = self.N
        arr = (N.c_void_p * self.world)(*[flag_of(q) for q in range(self.world)])
        N.check(N.lib.sw_peer_signal(arr, self.world, value & 0xFFFFFFFF, N.c_void_p(stream)))

    def sum_into(self, out_ptr: int, stream: int) -> None:
        N = self.N
        N.check(N.lib.sw_sum_slots_f32(N.c_void_p(self.base), self.slot_elems, self.world, N.c_void_p(out_ptr),
                                       N.c_void_p(stream)))

    def _rendezvous(self) -> None:
        N = self.N
        tick, ticks = N.DeviceBuffer(4), N.DeviceBuffer(4 * self.world)
        N.check(N.lib.sw_memset(N.c_void_p(tick.ptr), 0, 4, None))
        N.synchronize()
        self.comm.all_gather_f32(ticks.ptr, tick.ptr, 1)
        N.synchronize()

    def close(self) -> None:
        N = self.N
        if self.base is None:
            return
        N.synchronize()
        if self.world > 1:
            self._rendezvous()  # nobody writes into a buffer after this
            for q, p in enumerate(self.peers):
                if q != self.rank and p:
                    N.check(N.lib.sw_ipc_close(N.c_void_p(p)))
        N.check(N.lib.sw_ipc_free(N.c_void_p(self.base)))
        self.base = None
