"""Benchmark of the B200 StrideWeave carrier hot path.

Headline workload, at every world size: the sharded MXFP8 contraction
C[65536 x 16384] = A[65536 x 16384] . B[16384 x 16384]^T (inputs N(0, 1), E4M3
payloads with E8M0 scales per 32-block along K, fp32 accumulation, Float32 C),
M-split across the N GPUs: rank r contracts its 65536/N rows of A against a
replica of B, with no collective on the data path.  One step = one pass over
the whole C.  `value` is the whole-job TFLOP/s (2 M N K over the slowest
rank's device time), `scaling` "strong" (the problem is fixed as N grows).

The same line carries, under `k_split`, the K-split of the same contraction
(each rank a K/N slice, Float32 partials reduce-scattered over NVLink with
the C-ABI NCCL communicator, 8 N-chunks overlapping the next chunk's
contraction) with the reduce-scatter timed alone as its communication floor;
under `parity`, a sampled block of every rank's C checked against a float64
product of the device-dequantised operands (and, for the M-split, against a
single contraction of the same rows, bit for bit); and, at one GPU, the
layout-aware reductions, MX quantisation, the 8192^3 contractions and the MLP
training step of the other configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Operands (1.25 GiB per rank at N = 1, 0.38 GiB at N = 8) are larger than L2;
timing is by CUDA events on the launching stream; the multi-GPU time is the
max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# ---- the headline: the sharded MXFP8 contraction --------------------------------
M5, N5, K5 = 65536, 16384, 16384
FLOP5 = 2.0 * M5 * N5 * K5
K_CHUNKS = 8
PARITY_TOL = 2e-3  # relative Frobenius error of the contraction path
E2E_CHUNK_ROWS = 2048  # rows per block of the host-streamed step
# DRAM bytes (read + write) per launch of the M-split contraction at one GPU,
# from ncu on the per-rank shape of eight GPUs (8192 x 16384 x 16384, the
# committed capture) scaled by the 8x rows: A reads and C writes grow with the
# rows, and so do B's re-reads (one pass of B per raster group of row tiles).
NCU_TRAFFIC_GEMM_8192_ROWS = 2330.479e6 + 558.476e6

# ---- the layout-aware reductions (config 2) ---------------------------------------
R, C = 8192, 4096
X_BYTES = R * C * 4
RED_BYTES = X_BYTES + R * 4  # algorithmic bytes of one reduction launch
LAYOUTS = ("rowmajor", "transposed", "tiled_swizzled")
# DRAM bytes (read + write) per launch that ncu measured for each layout's
# three reductions (mean), against 134,250,496 algorithmic bytes: the
# committed `--profile-case reduce` capture of the kernels this file times.
NCU_TRAFFIC = {"rowmajor": 139.31e6, "transposed": 137.63e6, "tiled_swizzled": 139.46e6}
OPS = ("reduce_sum", "reduce_max", "argmax")
SWZ = [(3, 2, 3)]


def plan_of(layout: str):
    if layout == "rowmajor":
        return [(R, C)], [(C, 1)], []
    if layout == "transposed":
        return [(R, 1)], [(C, R)], []
    return [(128, 32), (64, 128 * 32 * 128)], [(32, 1), (128, 128 * 32)], SWZ


def storage_of(layout: str, x: np.ndarray) -> np.ndarray:
    """Physical storage holding logical X under `layout`."""
    if layout == "rowmajor":
        return np.ascontiguousarray(x).ravel()
    if layout == "transposed":
        return np.ascontiguousarray(x.T).ravel()
    # tile (tr, tc) of 128 x 32 at (tr * 128 + tc) * 4096, row-major inside
    t = x.reshape(64, 128, 128, 32).transpose(0, 2, 1, 3)  # [tr, tc, r, c]
    flat = np.ascontiguousarray(t).ravel()
    # carrier flat index f lives at swizzle(f): bits 2..4 ^= bits 5..7
    f = np.arange(flat.size, dtype=np.int64)
    phys = f ^ (((f >> 5) & 7) << 2)
    out = np.empty_like(flat)
    out[phys] = flat
    return out


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


METRIC = "sharded MXFP8 contraction TFLOP/s"


def headline_config(world: int) -> dict:
    """The `config` of the JSON line, the same in both arms."""
    return {"workload": "config5_sharded_mxfp8_65536x16384x16384", "M": M5, "N": N5, "K": K5,
            "split": "M (B replicated, no collective)", "parallelism": f"M-split x{world}",
            "formats": "E4M3 payload, E8M0 scale per 32 along K, fp32 accumulate, Float32 C",
            "l2": "operands larger than L2 (1.25 GiB at one GPU, 0.38 GiB per rank at eight)"}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------
# reference arm: the reference CPU carrier's matmul on the host cores


def reference_matmul_rate(rows_per_thread: int, cols: int, reps: int, warmup: int,
                          threads: int | None = None) -> tuple[float, int, str]:
    """Time the reference CPU carrier's Float32 matmul (``sw.matmul``, the
    contraction the MX contraction replaces, run on dequantised operands) on a
    bounded sample of the headline workload: ``rows_per_thread`` rows of A per
    host thread against ``cols`` rows of B, K = 16384, every thread a zero-copy
    row slice (the reference kernel is single-threaded and releases the GIL).
    Returns (TFLOP/s, threads, sample description)."""
    sys.path.append(str(ROOT / "baseline" / "_ref"))
    import strideweave as sw
    from strideweave import CPU, Layout, Shape, Stride, Tensor
    from concurrent.futures import ThreadPoolExecutor

    threads = threads or os.cpu_count() or 1
    rows = rows_per_thread * threads
    rng = np.random.default_rng(0)
    # N(0, 1) stand-ins for the dequantised operands (values do not change the
    # CPU kernel's speed)
    a = rng.standard_normal((rows, K5), dtype=np.float32)
    b = rng.standard_normal((cols, K5), dtype=np.float32)
    ta = Tensor(CPU(a.size, pointer=a.ctypes.data), 0, Layout(Shape([rows, K5]), Stride([K5, 1])))
    tb = Tensor(CPU(b.size, pointer=b.ctypes.data), 0, Layout(Shape([cols, K5]), Stride([K5, 1])))

    def job(t: int) -> None:
        with sw.no_grad():
            sw.matmul(ta[t * rows_per_thread:(t + 1) * rows_per_thread, :], tb)

    with ThreadPoolExecutor(threads) as pool:
        for _ in range(warmup):
            list(pool.map(job, range(threads)))
        t0 = time.perf_counter()
        for _ in range(reps):
            list(pool.map(job, range(threads)))
        dt = (time.perf_counter() - t0) / max(reps, 1)
    tflops = 2.0 * rows * cols * K5 / dt / 1e12
    sample = (f"{rows} rows of A x {cols} rows of B (K = {K5}) per step, {rows_per_thread} rows per host thread; "
              f"the reference CPU carrier's Float32 matmul on dequantised-operand stand-ins")
    return tflops, threads, sample


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    try:
        sys.path.append(str(ROOT / "baseline" / "_ref"))
        import strideweave  # noqa: F401
    except Exception as exc:  # pragma: no cover - reported, not raised
        print(json.dumps({"impl": "reference", "unavailable": f"reference not importable: {exc}"}))
        return
    tflops, threads, sample = reference_matmul_rate(rows_per_thread=2, cols=2048, reps=args.steps,
                                                    warmup=args.warmup)
    ms = FLOP5 / (tflops * 1e12) * 1e3
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(tflops, 8), "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": headline_config(args.gpus),
        "cpu_baseline": {"value": round(tflops, 8), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(tflops, 8), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ms_per_step extrapolates the sample's rate to the whole 65536 x 16384 x 16384 contraction",
    }))


def cpu_baseline_sample() -> dict:
    """The reference CPU carrier on a bounded sample (rank 0, N = 1 only)."""
    try:
        tflops, threads, sample = reference_matmul_rate(rows_per_thread=2, cols=2048, reps=2, warmup=1)
        kind = "reference"
    except ImportError:  # no installed reference: the oracle's restatement of its matmul
        from oracle import oracle as O

        rng = np.random.default_rng(0)
        a = rng.standard_normal((4, K5), dtype=np.float32)
        b = rng.standard_normal((512, K5), dtype=np.float32)
        t0 = time.perf_counter()
        O.matmul(a, b)
        tflops = 2.0 * 4 * 512 * K5 / (time.perf_counter() - t0) / 1e12
        threads, kind = 1, "port"
        sample = f"4 rows of A x 512 rows of B (K = {K5}), the oracle's restatement of the reference matmul"
    return {"value": round(tflops, 8), "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample}


# ---------------------------------------------------------------------------------
# the headline: config 5, the sharded MXFP8 contraction


def quantize_generated(torch, N, kernels, fmt, rows, cols, seed, sigma=1.0, block=8192):
    """Device planes of a seeded N(0, sigma^2) [rows, cols] operand, generated
    and quantised in row blocks (bounded Float32 staging)."""
    rb = kernels.mx_row_bytes(fmt, cols)
    katoms = (cols // 32 + 3) // 4
    pay = N.DeviceBuffer(rows * rb)
    sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, cols // 32))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    for r0 in range(0, rows, block):
        n = min(block, rows - r0)
        x = torch.randn((n, cols), generator=gen, device="cuda", dtype=torch.float32) * sigma
        kernels.mx_quantize(fmt, x.data_ptr(), n, cols, cols, 1, pay.ptr + r0 * rb, rb,
                            sc.ptr + (r0 // 128) * katoms * 512)
        N.synchronize()  # x is released by torch's allocator on its own stream
        del x
    return pay, sc


def max_over_ranks(torch, dist, world, value: float) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(N, fn, steps: int, warmup: int, torch, dist, world) -> float:
    """Mean device ms of `fn` over `steps` calls on the legacy default stream
    (events on that stream), max over ranks."""
    for _ in range(warmup):
        fn()
    N.synchronize()
    if world > 1:
        dist.barrier()
    N.synchronize()
    e0, e1 = N.Event(timing=True), N.Event(timing=True)
    e0.record(0)
    for _ in range(steps):
        fn()
    e1.record(0)
    ms = e0.elapsed_ms(e1) / steps
    N.synchronize()
    if world > 1:
        dist.barrier()
    return max_over_ranks(torch, dist, world, ms)


def dequantized_rows(N, kernels, fmt, planes, row0: int, rows: int, k: int) -> np.ndarray:
    """Float32 image of operand rows [row0, row0 + rows) (whole 128-row scale
    groups), by the device dequantiser."""
    rb = kernels.mx_row_bytes(fmt, k)
    katoms = (k // 32 + 3) // 4
    out = N.DeviceBuffer(4 * rows * k)
    kernels.mx_dequantize(fmt, planes[0].ptr + row0 * rb, rb, planes[1].ptr + (row0 // 128) * katoms * 512, rows, k,
                          out.ptr, k)
    host = np.empty((rows, k), np.float32)
    N.synchronize()
    out.download(host)
    return host


def result_block(N, op, row0: int, n0: int, rows: int = 128, cols: int = 256) -> np.ndarray:
    """C[row0 : row0 + rows, n0 : n0 + cols] of the rank's result (local rows)."""
    plan = op.plan
    if plan.mode == "m" or plan.chunks == 1:
        base, pitch, col = op.out.data_ptr, plan.N, n0
    else:
        c = n0 // plan.chunk_cols
        base, pitch, col = op.out.data_ptr + 4 * c * plan.rows_local * plan.chunk_cols, plan.chunk_cols, \
            n0 % plan.chunk_cols
    span = np.empty((rows, pitch), np.float32)
    N.synchronize()
    N.check(N.lib.sw_memcpy_d2h(N.c_void_p(span.ctypes.data), N.c_void_p(base + 4 * row0 * pitch), span.nbytes,
                                None))
    return span[:, col:col + cols].copy()


def sharded_parity(torch, dist, N, kernels, fmt, op, a, b, world, rank) -> dict:
    """A 128 x 256 block of this rank's C against the float64 product of the
    device-dequantised operands (the dequantiser is bit-exact with the CPU
    oracle in the tests), summed over every rank's K slice for a K-split; for
    an M-split also against a single contraction of the same rows, which must
    be bit-identical.  Returns the worst error over ranks."""
    plan = op.plan
    rng = np.random.default_rng(4242 + 31 * rank + (1 if plan.mode == "k" else 0))
    g_local = int(rng.integers(0, plan.rows_local // 128))
    row0 = g_local * 128                                   # in this rank's C rows
    n0 = int(rng.integers(0, plan.N // 256)) * 256         # whole 256-wide tile, inside one chunk
    got = result_block(N, op, row0, n0).astype(np.float64)
    out = {"sample": f"C rows [{plan.row0 + row0}, +128) x cols [{n0}, +256) on each rank"}
    if plan.mode == "m":
        da = dequantized_rows(N, kernels, fmt, a, row0, 128, plan.k_local).astype(np.float64)
        db = dequantized_rows(N, kernels, fmt, b, n0, 256, plan.k_local).astype(np.float64)
        want = da @ db.T
        # the same rows as one contraction on this GPU
        rb = kernels.mx_row_bytes(fmt, plan.k_local)
        katoms = (plan.k_local // 32 + 3) // 4
        single = N.DeviceBuffer(4 * 128 * 256)
        kernels.mx_gemm(fmt, a[0].ptr + row0 * rb, rb, a[1].ptr + g_local * katoms * 512, b[0].ptr + n0 * rb, rb,
                        b[1].ptr + (n0 // 128) * katoms * 512, single.ptr, 128, 256, plan.k_local)
        one = np.empty((128, 256), np.float32)
        N.synchronize()
        single.download(one)
        bit_exact = bool(np.array_equal(one.astype(np.float64), got))
    else:
        # every rank contributes its K slice to every rank's sample
        samples = [(plan.row0 + row0, n0)]
        if world > 1:
            gathered = [None] * world
            dist.all_gather_object(gathered, samples[0])
            samples = gathered
        mine = []
        for grow0, gn0 in samples:
            da = dequantized_rows(N, kernels, fmt, a, grow0, 128, plan.k_local).astype(np.float64)
            db = dequantized_rows(N, kernels, fmt, b, gn0, 256, plan.k_local).astype(np.float64)
            mine.append(da @ db.T)
        if world > 1:
            parts = [None] * world
            dist.all_gather_object(parts, mine)
            want = sum(p[rank] for p in parts)
        else:
            want = mine[0]
        bit_exact = None
    err = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))
    out["rel_frobenius"] = max_over_ranks(torch, dist, world, err)
    if bit_exact is not None:
        flag = max_over_ranks(torch, dist, world, 0.0 if bit_exact else 1.0)
        out["single_contraction_bit_exact"] = flag == 0.0
    out["tol"] = PARITY_TOL
    out["ok"] = out["rel_frobenius"] <= PARITY_TOL and out.get("single_contraction_bit_exact", True)
    return out


def bench_sharded(torch, dist, N, kernels, args, world, rank) -> dict:
    """Config 5 at this world size: the M-split (headline), its end-to-end
    pass from host memory, and the K-split with its communication floor."""
    from strideweave_b200.sharding import MXShardedContraction, NcclCommunicator, ShardPlan

    fmt = N.SW_MX_E4M3
    res: dict = {}
    # the C-ABI NCCL communicator: the end-to-end pass all-gathers the
    # quantised B slices with it, the K-split reduce-scatters with it
    comm = None
    if world > 1:
        ids = [NcclCommunicator.new_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        comm = NcclCommunicator(world, rank, ids[0])
    # ---- M-split ----
    mp = ShardPlan("m", world, rank, M5, N5, K5)
    a = quantize_generated(torch, N, kernels, fmt, mp.rows_local, K5, seed=7000 + rank)
    b = quantize_generated(torch, N, kernels, fmt, N5, K5, seed=9000)
    op = MXShardedContraction(mp, fmt, a, b, comm=comm)
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))).__enter__()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_seconds:  # clocks settle under load
        op.run()
        N.synchronize()
    ms = time_steps(N, op.run, args.steps, args.warmup, torch, dist, world)
    time.sleep(0.25)
    clocks.__exit__(None, None, None)
    res["m"] = {"ms": ms, "tflops": FLOP5 / (ms / 1e3) / 1e12, "launch_flop": mp.local_flops,
                "clocks": clocks.summary()}
    N.raise_device_status()
    res["m"]["parity"] = sharded_parity(torch, dist, N, kernels, fmt, op, a, b, world, rank)

    # ---- end to end: Float32 operands in pinned host memory -> quantise ->
    # contract -> C back to host, every step ----
    rows, k = mp.rows_local, K5
    pin_a = torch.empty((rows, k), dtype=torch.float32).pin_memory()
    pin_b = torch.empty((N5, k), dtype=torch.float32).pin_memory()
    pin_c = torch.empty((rows, N5), dtype=torch.float32).pin_memory()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5000 + rank)
    for host in (pin_a, pin_b):  # fill from device draws (host RNG over GiBs is slow)
        for r0 in range(0, host.shape[0], 8192):
            host[r0:r0 + 8192].copy_(torch.randn((min(8192, host.shape[0] - r0), k), generator=gen, device="cuda"))
    torch.cuda.synchronize()

    def e2e_step():
        # copies, quantisation, contraction and the return of C, pipelined
        # over blocks of rows on three streams (MXShardedContraction.run_from_host)
        op.run_from_host(pin_a.data_ptr(), pin_b.data_ptr(), pin_c.data_ptr(), chunk_rows=E2E_CHUNK_ROWS)

    e2e_ms = time_steps(N, e2e_step, max(2, min(args.steps, 3)), 1, torch, dist, world)
    b_rows = N5 // world if world > 1 else N5  # each rank's share of B from host memory
    res["e2e"] = {"value": FLOP5 / (e2e_ms / 1e3) / 1e12, "ms": e2e_ms,
                  "h2d": world * 4 * (rows + b_rows) * k, "d2h": world * pin_c.numel() * 4,
                  "chunk_rows": E2E_CHUNK_ROWS}
    N.raise_device_status()
    # the link bound: this rank's pinned host <-> device copy rates, each
    # direction alone (1 GiB, best of three)
    probe = N.DeviceBuffer(pin_b.numel() * 4)

    def copy_rate(h2d: bool) -> float:
        best = None
        for _ in range(3):
            e0, e1 = N.Event(timing=True), N.Event(timing=True)
            e0.record(0)
            if h2d:
                N.check(N.lib.sw_memcpy_h2d(N.c_void_p(probe.ptr), N.c_void_p(pin_b.data_ptr()), probe.nbytes, None))
            else:
                N.check(N.lib.sw_memcpy_d2h(N.c_void_p(pin_b.data_ptr()), N.c_void_p(probe.ptr), probe.nbytes, None))
            e1.record(0)
            N.synchronize()
            ms = e0.elapsed_ms(e1)
            best = ms if best is None else min(best, ms)
        return probe.nbytes / (best / 1e3) / 1e9

    h2d_gbs, d2h_gbs = copy_rate(True), copy_rate(False)
    # both directions at once (1 GiB each way on two streams): the rate the
    # streamed step actually shares between its inbound and outbound copies
    probe2 = N.DeviceBuffer(probe.nbytes)
    s_in, s_out = N.Stream(), N.Stream()
    both = None
    for _ in range(3):
        e0, e1, d_in, d_out = N.Event(timing=True), N.Event(timing=True), N.Event(), N.Event()
        e0.record(0)
        e0.wait(s_in.handle)
        e0.wait(s_out.handle)
        N.check(N.lib.sw_memcpy_h2d(N.c_void_p(probe.ptr), N.c_void_p(pin_b.data_ptr()), probe.nbytes,
                                    N.c_void_p(s_in.handle)))
        N.check(N.lib.sw_memcpy_d2h(N.c_void_p(pin_a.data_ptr()), N.c_void_p(probe2.ptr), probe.nbytes,
                                    N.c_void_p(s_out.handle)))
        d_in.record(s_in.handle)
        d_out.record(s_out.handle)
        d_in.wait(0)
        d_out.wait(0)
        e1.record(0)
        N.synchronize()
        ms = e0.elapsed_ms(e1)
        both = ms if both is None else min(both, ms)
    both_gbs = 2 * probe.nbytes / (both / 1e3) / 1e9
    s_in.close()
    s_out.close()
    probe.free()
    probe2.free()
    h2d_bytes, d2h_bytes = 4 * (rows + b_rows) * k, pin_c.numel() * 4
    link_ms = max(h2d_bytes / h2d_gbs, d2h_bytes / d2h_gbs, (h2d_bytes + d2h_bytes) / both_gbs) / 1e6
    res["e2e"]["link"] = {"h2d_gbs": round(h2d_gbs, 1), "d2h_gbs": round(d2h_gbs, 1),
                          "both_directions_gbs": round(both_gbs, 1), "bound_ms": round(link_ms, 2),
                          "frac_of_link_bound": round(link_ms / e2e_ms, 3)}
    # the streamed step's result equals the device step's on the same planes
    got = np.empty((2, N5), np.float32)
    N.check(N.lib.sw_memcpy_d2h(N.c_void_p(got.ctypes.data), N.c_void_p(op.out.data_ptr), got.nbytes, None))
    N.synchronize()
    res["e2e"]["host_rows_match_device"] = bool(np.array_equal(got, pin_c[:2].numpy()))
    op.close()
    del pin_a, pin_b, pin_c, op, a, b
    N.synchronize()
    torch.cuda.empty_cache()

    # ---- K-split ----
    kp = ShardPlan("k", world, rank, M5, N5, K5, chunks=K_CHUNKS)
    a = quantize_generated(torch, N, kernels, fmt, M5, kp.k_local, seed=8000 + rank)
    b = quantize_generated(torch, N, kernels, fmt, N5, kp.k_local, seed=9500 + rank)
    ksteps = max(3, args.steps // 4)
    # the peer-memory K-split (the contraction writes each row block into its
    # owner's slot over NVLink, owners sum their slots): the K-split of record
    pp = ShardPlan("k", world, rank, M5, N5, K5, chunks=1)
    op = MXShardedContraction(pp, fmt, a, b, comm=comm, transport="peer")
    kms = time_steps(N, op.run, ksteps, min(args.warmup, 2), torch, dist, world)
    res["k"] = {"ms": kms, "tflops": FLOP5 / (kms / 1e3) / 1e12, "transport": "NVLink peer stores + ordered slot sum"}
    N.raise_device_status()
    res["k"]["parity"] = sharded_parity(torch, dist, N, kernels, fmt, op, a, b, world, rank)
    op.close()
    del op
    # the same K-split with NCCL's reduce-scatter, chunked and overlapped
    op = MXShardedContraction(kp, fmt, a, b, comm=comm)
    nms = time_steps(N, op.run, ksteps, min(args.warmup, 2), torch, dist, world)
    res["k"]["nccl"] = {"ms": nms, "tflops": FLOP5 / (nms / 1e3) / 1e12, "chunks": K_CHUNKS,
                        "comm_sms": kp.comm_sms}
    N.raise_device_status()
    if comm is not None:
        # NCCL's reduce-scatter alone: all 8 chunks of Float32 partials (4 GiB
        # per rank), on the collective's stream, with every SM free
        count = kp.rows_local * kp.chunk_cols
        cs = op.comm_stream.handle

        def comm_only():
            for c in range(kp.chunks):
                comm.reduce_scatter_f32(op._chunk_out(c), op.partials[c % len(op.partials)].data_ptr, count, cs)
            ev = N.Event()
            ev.record(cs)
            ev.wait(0)

        cms = time_steps(N, comm_only, 3, 1, torch, dist, world)
        moved = (world - 1) / world * 4.0 * M5 * N5  # bytes each rank sends (and receives)
        compute_ms = res["m"]["ms"]  # the same FLOP per rank as the M-split's contraction
        bound = max(compute_ms, cms)
        res["k"]["comm_floor"] = {"ms": cms, "busbw_gbs": moved / (cms / 1e3) / 1e9,
                                  "bytes_per_rank": moved, "compute_ms": compute_ms, "bound_ms": bound,
                                  "frac_of_bound": bound / kms, "frac_of_bound_nccl": bound / nms}
        op.close()
        comm.close()
    else:
        op.close()
    del op, a, b
    N.synchronize()
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------------
# config 2: the layout-aware reductions (one GPU)


def bench_reductions(torch, N, kernels, args) -> dict:
    """Sum, max and argmax over mode 1 of X[8192 x 4096] ~ U(-1, 1) on a
    row-major, a transposed and a tiled + swizzled layout; one step = the 9
    reductions, consecutive launches reading different 128 MiB buffers."""
    rng = np.random.default_rng(1234)
    x = rng.uniform(-1, 1, size=(R, C)).astype(np.float32)
    host = {lay: storage_of(lay, x) for lay in LAYOUTS}
    dev = {lay: N.DeviceBuffer(X_BYTES) for lay in LAYOUTS}
    for lay in LAYOUTS:
        dev[lay].upload(host[lay])
    outs = {(op, lay): N.DeviceBuffer(R * 4) for op in OPS for lay in LAYOUTS}
    N.synchronize()
    order = [(op, lay) for op in OPS for lay in LAYOUTS]
    # plans are built once: the timed loop is one C call per launch
    plans = {}
    for op in OPS:
        for lay in LAYOUTS:
            kept, red, swz = plan_of(lay)
            plans[(op, lay)] = kernels.make_reduce_plan(op, 0, kept, red, swz)

    def launch_on(op, lay, ptr):
        N.check(N.lib.sw_reduce_f32(N.ctypes.byref(plans[(op, lay)]), N.c_void_p(ptr), R * C,
                                    N.c_void_p(outs[(op, lay)].ptr), None))

    def step():
        for op, lay in order:
            launch_on(op, lay, dev[lay].ptr)

    ms_per_step = time_steps(N, step, args.steps, args.warmup, torch, None, 1)
    # per-kernel durations: each kernel back to back over two copies of its
    # input (256 MiB > L2), one event pair per run of launches
    spare = {lay: N.DeviceBuffer(X_BYTES) for lay in LAYOUTS}
    for lay in LAYOUTS:
        N.check(N.lib.sw_memcpy_d2d(N.c_void_p(spare[lay].ptr), N.c_void_p(dev[lay].ptr), X_BYTES, None))
    per_kernel = {}
    # (20 launches a run, so the host's enqueue keeps ahead of the device;
    # the best of three runs)
    runs = 20
    for op in OPS:
        for lay in LAYOUTS:
            bufs = (dev[lay].ptr, spare[lay].ptr)
            launch_on(op, lay, bufs[0])
            best = None
            for _ in range(3):
                k0, k1 = N.Event(timing=True), N.Event(timing=True)
                k0.record(0)
                for r in range(runs):
                    launch_on(op, lay, bufs[(r + 1) % 2])
                k1.record(0)
                ms = k0.elapsed_ms(k1) / runs
                best = ms if best is None else min(best, ms)
            per_kernel[(op, lay)] = best
    # the timed reduce_max agrees with the sequential rule
    check = np.empty(R, dtype=np.float32)
    outs[("reduce_max", "rowmajor")].download(check)
    assert np.array_equal(check, x.max(axis=1)), "timed reduce_max disagrees with numpy"
    # end to end: pinned host input -> device -> 9 reductions -> host
    pinned = {lay: torch.from_numpy(host[lay]).pin_memory() for lay in LAYOUTS}
    res_host = torch.empty(R * 9, dtype=torch.float32).pin_memory()

    def e2e_step():
        for lay in LAYOUTS:
            N.check(N.lib.sw_memcpy_h2d(N.c_void_p(dev[lay].ptr), N.c_void_p(pinned[lay].data_ptr()), X_BYTES, None))
        step()
        for j, key in enumerate(order):
            N.check(N.lib.sw_memcpy_d2h(N.c_void_p(res_host.data_ptr() + 4 * R * j), N.c_void_p(outs[key].ptr),
                                        R * 4, None))

    e2e_ms = time_steps(N, e2e_step, max(3, args.steps // 4), 1, torch, None, 1)
    peaks = load_peaks()
    by_layout = {lay: sum(per_kernel[(op, lay)] for op in OPS) for lay in LAYOUTS}
    dominant = max(by_layout, key=by_layout.get)
    achieved = RED_BYTES / (by_layout[dominant] / 3 / 1e3) / 1e9
    N.raise_device_status()
    return {
        "gbs": round(9 * RED_BYTES / (ms_per_step / 1e3) / 1e9, 2), "ms_per_step": round(ms_per_step, 4),
        "config": "config 2: X[8192 x 4096] ~ U(-1,1); sum, max, argmax over mode 1 on row-major, transposed and "
                  "tiled ((128,64),(32,128)) + 3-bit swizzle layouts; inputs larger than L2, rotated",
        "roofline": {"bound": "hbm", "kernel": f"sw_reduce_f32[{dominant}]", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": NCU_TRAFFIC.get(dominant),
                     "per_kernel_gbs": {f"{op}/{lay}": round(RED_BYTES / (per_kernel[(op, lay)] / 1e3) / 1e9, 1)
                                        for op, lay in order}},
        "e2e": {"value": round(9 * RED_BYTES / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": 3 * X_BYTES, "d2h_bytes_per_step": 9 * R * 4},
    }


# ---------------------------------------------------------------------------------
# our arm


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true",
                    help="at one GPU, skip the secondary measurements (reductions, quantise, 8192^3, MLP)")
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="untimed busy time under the clock sampler before the timed region")
    ap.add_argument("--profile-case", choices=["reduce", "quantize", "dual", "mxfp8", "mxfp4", "mlp", "sharded",
                                               "misc"],
                    help="run a short, fixed sequence of launches for ncu and exit (no timing)")
    ap.add_argument("--reps", type=int, default=2, help="rounds of launches of --profile-case")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case, args.reps)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))

    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels

    N.set_device(local)
    sharded = bench_sharded(torch, dist, N, kernels, args, world, rank)
    extras = {}
    if world == 1 and not args.no_extras:
        extras["reductions"] = bench_reductions(torch, N, kernels, args)
        extras["quantize"] = bench_quantize(torch, N, kernels, 0, torch.cuda.current_stream())
        extras["contraction"] = bench_gemm(torch, N, kernels, 0, torch.cuda.current_stream())
        extras["mlp_step"] = bench_mlp(torch, N)

    if rank == 0:
        peaks = load_peaks()
        m = sharded["m"]
        # MXFP8 block-scaled MMA runs at twice the dense bf16 rate; the measured
        # cuBLAS bf16 figures stand for the clock and power of this pool.  The
        # headline contraction runs back to back for over a second under the
        # power cap, so its denominator is the sustained figure.
        peak = 2.0 * peaks["bf16_tflops_sustained"]
        kernel_tflops = m["launch_flop"] / (m["ms"] / 1e3) / 1e12
        traffic = None
        if NCU_TRAFFIC_GEMM_8192_ROWS is not None:
            traffic = NCU_TRAFFIC_GEMM_8192_ROWS * (M5 // world) / 8192
        k = sharded["k"]
        line = {
            "metric": METRIC,
            "value": round(m["tflops"], 1),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(m["ms"], 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "mxfp8 (e4m3 x e8m0), fp32 accumulate",
            "data": "synthetic N(0,1), seeded per rank",
            "config": headline_config(world),
            "roofline": {"bound": "tensor", "kernel": "mx_gemm_kernel<E4M3, 256, 3, fp32 rows>",
                         "achieved": round(kernel_tflops, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(kernel_tflops / peak, 4),
                         "peak_source": f"{peaks['source']}: 2 x bf16 dense sustained (MXFP8 is twice the bf16 "
                                        f"rate; the timed region runs under the power cap)",
                         "traffic": traffic, "frac_of_burst": round(kernel_tflops / (2.0 * peaks["bf16_tflops"]), 4),
                         "frac_of_spec_4500": round(kernel_tflops / 4500.0, 4)},
            "e2e": {"value": round(sharded["e2e"]["value"], 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": sharded["e2e"]["h2d"], "d2h_bytes_per_step": sharded["e2e"]["d2h"],
                    "ms_per_step": round(sharded["e2e"]["ms"], 3),
                    "path": f"MXShardedContraction.run_from_host: pinned Float32 A and B copied in blocks of "
                            f"{sharded['e2e']['chunk_rows']} rows, quantised and contracted per block while "
                            f"finished C blocks return (three streams)" +
                            (f"; each rank copies N/{world} rows of B and NCCL all-gathers the quantised B planes"
                             if world > 1 else ""),
                    "host_rows_match_device": sharded["e2e"]["host_rows_match_device"],
                    "link": sharded["e2e"]["link"]},
            "gpu_launches": world * args.steps,
            "clocks": m["clocks"],
            "parity": {"m_split": m["parity"], "k_split": k["parity"]},
            "k_split": {key: (round(v, 4) if isinstance(v, float) else v) for key, v in k.items()
                        if key not in ("parity",)},
        }
        if "comm_floor" in k:
            line["k_split"]["comm_floor"] = {key: round(v, 4) if isinstance(v, float) else v
                                             for key, v in k["comm_floor"].items()}
        for key, v in extras.items():
            line[key] = v
        if world == 1:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line))
    parity_ok = sharded["m"]["parity"]["ok"] and sharded["k"]["parity"]["ok"]
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not parity_ok:  # the line above says which check failed
        raise SystemExit("sharded contraction parity check failed")


# ---------------------------------------------------------------------------------
# secondary measurements (one GPU)


def bench_gemm(torch, N, kernels, s, stream) -> dict:
    """MXFP8 and MXFP4 contraction at M=N=K=8192 (device-resident operands)."""
    out = {}
    M = Nn = K = 8192
    rng = np.random.default_rng(0)
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    b = torch.from_numpy((rng.standard_normal((Nn, K)) * 0.02).astype(np.float32)).cuda()
    for name, fmt in (("mxfp8", N.SW_MX_E4M3), ("mxfp4", N.SW_MX_E2M1)):
        row_bytes = K if fmt == N.SW_MX_E4M3 else K // 2
        pa, pb = N.DeviceBuffer(M * row_bytes), N.DeviceBuffer(Nn * row_bytes)
        sa = N.DeviceBuffer(kernels.scale_bytes_tc128(M, K // 32))
        sb = N.DeviceBuffer(kernels.scale_bytes_tc128(Nn, K // 32))
        kernels.mx_quantize(fmt, a.data_ptr(), M, K, K, 1, pa.ptr, row_bytes, sa.ptr, stream=s)
        kernels.mx_quantize(fmt, b.data_ptr(), Nn, K, K, 1, pb.ptr, row_bytes, sb.ptr, stream=s)
        c = N.DeviceBuffer(M * Nn * 2)
        for _ in range(3):
            kernels.mx_gemm(fmt, pa.ptr, row_bytes, sa.ptr, pb.ptr, row_bytes, sb.ptr, c.ptr, M, Nn, K,
                            out_bf16=True, stream=s)
        torch.cuda.synchronize()
        reps = 10
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            kernels.mx_gemm(fmt, pa.ptr, row_bytes, sa.ptr, pb.ptr, row_bytes, sb.ptr, c.ptr, M, Nn, K,
                            out_bf16=True, stream=s)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        tflops = 2.0 * M * Nn * K / (ms / 1e3) / 1e12
        spec = 4500.0 if fmt == N.SW_MX_E4M3 else 9000.0
        peaks = load_peaks()
        clock_adj = peaks["bf16_tflops"] * (2 if fmt == N.SW_MX_E4M3 else 4)
        out[name] = {"tflops": round(tflops, 1), "ms": round(ms, 4), "frac_of_spec_dense": round(tflops / spec, 4),
                     "frac_of_clock_adjusted": round(tflops / clock_adj, 4),
                     "config": "M=N=K=8192, A~N(0,1), B~N(0,0.02), bf16 C"}
        del pa, pb, sa, sb, c
    N.raise_device_status()
    return out


def bench_quantize(torch, N, kernels, s, stream) -> dict:
    """MX quantisation of a Float32 [8192 x 8192] operand (256 MiB read),
    along rows (K-major source) and along strided columns (a K x N source
    quantised along K), back to back over two inputs (512 MiB > L2).
    Algorithmic bytes: the Float32 read plus the payload and TC128 scale
    writes."""
    rows = cols = 8192
    rng = np.random.default_rng(7)
    srcs = [torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float32)).cuda() for _ in range(2)]
    peaks = load_peaks()
    out = {}
    for name, fmt in (("mxfp8", N.SW_MX_E4M3), ("mxfp4", N.SW_MX_E2M1)):
        rb = kernels.mx_row_bytes(fmt, cols)
        pay = N.DeviceBuffer(rows * rb)
        sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, cols // 32))
        moved = rows * cols * 4 + rows * rb + kernels.scale_bytes_tc128(rows, cols // 32)
        for along, (ld_row, ld_col) in (("rows", (cols, 1)), ("strided_cols", (1, rows))):
            def q(i):
                kernels.mx_quantize(fmt, srcs[i % 2].data_ptr(), rows, cols, ld_row, ld_col, pay.ptr, rb, sc.ptr,
                                    stream=s)
            for i in range(4):
                q(i)
            torch.cuda.synchronize()
            reps = 20
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(reps):
                q(i)
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            gbs = moved / (us * 1e3)
            out[f"{name}_{along}"] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                      "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                                      "bytes": moved}
        del pay, sc
    # the MLP's two-way quantiser: S = x * gelu'(h) over a [4096 x 8192] hidden
    # gradient (two 128 MiB reads), both MXFP8 operands written
    r2, c2 = 4096, 8192
    xs = [srcs[i].view(-1)[: r2 * c2] for i in range(2)]
    hs = [srcs[1 - i].view(-1)[r2 * c2:] for i in range(2)]
    planes = [(N.DeviceBuffer(r2 * c2), N.DeviceBuffer(kernels.scale_bytes_tc128(r2, c2 // 32))),
              (N.DeviceBuffer(r2 * c2), N.DeviceBuffer(kernels.scale_bytes_tc128(c2, r2 // 32)))]
    moved = 2 * r2 * c2 * 4 + 2 * r2 * c2 + kernels.scale_bytes_tc128(r2, c2 // 32) + \
        kernels.scale_bytes_tc128(c2, r2 // 32)

    def qd(i):
        kernels.mx_quantize_dual(N.SW_MX_E4M3, N.SW_XF_GELU_GRAD, xs[i % 2].data_ptr(), hs[i % 2].data_ptr(), r2, c2,
                                 c2, (planes[0][0].ptr, planes[0][1].ptr), (planes[1][0].ptr, planes[1][1].ptr),
                                 stream=s)
    for i in range(4):
        qd(i)
    torch.cuda.synchronize()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        qd(i)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    gbs = moved / (us * 1e3)
    out["mxfp8_dual_gelu_grad_4096x8192"] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                             "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                                             "bytes": moved}
    # the view quantiser on config 2(c)'s placement: X[8192 x 4096] in
    # 128 x 32 tiles through the 3-bit swizzle, quantised along mode 1 where
    # it lies (two 128 MiB sources alternate)
    kept, red, swz = plan_of("tiled_swizzled")
    vpay = N.DeviceBuffer(R * C)
    vsc = N.DeviceBuffer(kernels.scale_bytes_tc128(R, C // 32))
    vsrc = [srcs[i].data_ptr() for i in range(2)]  # 256 MiB each: the first 128 MiB hold the tiled X

    def qv(i):
        kernels.mx_quantize_view(N.SW_MX_E4M3, vsrc[i % 2], R * C, 0, kept, red, vpay.ptr, C, vsc.ptr, swizzle=swz,
                                 stream=s)
    for i in range(4):
        qv(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        qv(i)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    moved = R * C * 4 + R * C + kernels.scale_bytes_tc128(R, C // 32)
    gbs = moved / (us * 1e3)
    out["mxfp8_view_tiled_swizzled_8192x4096"] = {"us": round(us, 2), "gbs": round(gbs, 1),
                                                  "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                                                  "bytes": moved}
    N.raise_device_status()
    return out


def bench_mlp(torch, N, steps=5, warmup=2) -> dict:
    """Config 4: one MXFP8 MLP training step - 1024 -> 4096 -> 4096 -> 1024 with
    GELU, batch 8192, fp32 master weights N(0, 0.02), inputs and targets N(0, 1),
    MSE loss; forward, reference-autograd backward (dgrad and wgrad with MX
    re-quantisation along each contraction's K), SGD update."""
    sys.path.append(str(ROOT / "baseline" / "_ref"))
    from strideweave import Layout, Shape, Stride, Tensor

    from strideweave_b200 import CUDA, nn

    B, dims = 8192, [1024, 4096, 4096, 1024]
    rng = np.random.default_rng(0)
    model = nn.MLP(dims, fmt="MXFP8_E4M3", seed=0, std=0.02)
    x = rng.standard_normal((B, dims[0])).astype(np.float32)
    t = rng.standard_normal((B, dims[-1])).astype(np.float32)
    xt = Tensor(CUDA.from_numpy(x.ravel()), 0, Layout(Shape([B, dims[0]]), Stride([dims[0], 1])))
    tt = Tensor(CUDA.from_numpy(t.T.ravel().copy()), 0, Layout(Shape([B, dims[-1]]), Stride([1, B])))
    losses = []

    def step():
        # the fused step: the same kernels as the autograd path, scheduled
        # explicitly (the reference's leaf-gradient copy is per element)
        return model.train_step(xt, tt, lr=1e-3)

    def timed(fn) -> float:
        for _ in range(warmup):
            losses.append(fn())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            losses.append(fn())
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    eager_ms = timed(step)
    # the same step captured once in a CUDA graph and replayed (one launch per step)
    graph = model.capture_step(xt, tt, lr=1e-3)
    ms = timed(graph.step)
    graph.close()
    per_gemm = [2.0 * B * dims[i] * dims[i + 1] for i in range(len(dims) - 1)]
    flops = 3 * sum(per_gemm) - per_gemm[0]  # forward + wgrad for all layers, dgrad for layers 2..3
    N.raise_device_status()
    first, last = float(losses[0][0]), float(losses[-1][0])
    return {"tflops": round(flops / (ms / 1e3) / 1e12, 1), "ms_per_step": round(ms, 3),
            "eager_ms_per_step": round(eager_ms, 3), "flop_per_step": flops, "loss_first": round(first, 5),
            "loss_last": round(last, 5),
            "config": "MXFP8 MLP 1024-4096-4096-1024, GELU, batch 8192, MSE, SGD lr 1e-3 (fwd + bwd + step, "
                      "no first-layer dgrad); ms_per_step replays the step captured in a CUDA graph, "
                      "eager_ms_per_step enqueues it from Python"}


def profile_case(case: str, reps: int) -> None:
    """A fixed, small sequence of launches for an ncu capture.

    reduce: the three layouts of X[8192 x 4096] x (sum, max, argmax), `reps`
    rounds (9 launches per round).  quantize: MXFP8 then MXFP4 of a Float32
    [8192 x 8192] along rows and along strided columns, `reps` rounds (4
    launches per round).  dual: the two-way MXFP8 quantiser over a
    [4096 x 8192] hidden activation, with GELU then with GELU', `reps` rounds
    (2 launches per round).  mxfp8 / mxfp4: quantise two 8192 x 8192
    operands, then `reps` contractions at M = N = K = 8192 (bf16 C).  sharded:
    the M-split contraction of one of eight ranks (8192 x 16384 x 16384,
    Float32 C), `reps` launches.  mlp: the MLP training step, `reps` steps
    after one warm-up step.  misc: one launch each, `reps` rounds, of the
    kernels the other cases do not reach - the batched contraction, the
    elementwise AXPY, the MSE loss and gradient, the Float32 contraction, the
    reduction gradients, the view copy, the view quantiser, the scale
    rewrite and the binary product.
    """
    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels

    N.set_device(0)
    if case == "mlp":
        import torch

        print(bench_mlp(torch, N, steps=reps, warmup=1))
        return
    if case == "quantize":
        rows = cols = 8192
        src = N.DeviceBuffer(rows * cols * 4)
        src.upload(np.random.default_rng(7).standard_normal((rows, cols)).astype(np.float32))
        for _ in range(reps):
            for fmt in (N.SW_MX_E4M3, N.SW_MX_E2M1):
                rb = kernels.mx_row_bytes(fmt, cols)
                pay = N.DeviceBuffer(rows * rb)
                sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, cols // 32))
                for ld_row, ld_col in ((cols, 1), (1, rows)):
                    kernels.mx_quantize(fmt, src.ptr, rows, cols, ld_row, ld_col, pay.ptr, rb, sc.ptr)
                N.synchronize()
        N.raise_device_status()
        print("profile case quantize: ok")
        return
    if case == "dual":
        rows, cols = 4096, 8192
        rng = np.random.default_rng(8)
        x, h = N.DeviceBuffer(rows * cols * 4), N.DeviceBuffer(rows * cols * 4)
        x.upload(rng.standard_normal((rows, cols)).astype(np.float32))
        h.upload((rng.standard_normal((rows, cols)) * 2).astype(np.float32))
        pr, pc = N.DeviceBuffer(rows * cols), N.DeviceBuffer(rows * cols)
        sr = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, cols // 32))
        sc = N.DeviceBuffer(kernels.scale_bytes_tc128(cols, rows // 32))
        for _ in range(reps):
            for xf in (N.SW_XF_GELU, N.SW_XF_GELU_GRAD):
                kernels.mx_quantize_dual(N.SW_MX_E4M3, xf, x.ptr, h.ptr, rows, cols, cols, (pr.ptr, sr.ptr),
                                         (pc.ptr, sc.ptr))
            N.synchronize()
        N.raise_device_status()
        print("profile case dual: ok")
        return
    if case == "reduce":
        x = np.random.default_rng(0).uniform(-1, 1, size=(R, C)).astype(np.float32)
        bufs = {}
        for lay in LAYOUTS:
            bufs[lay] = N.DeviceBuffer(X_BYTES)
            bufs[lay].upload(storage_of(lay, x))
        out = N.DeviceBuffer(R * 4)
        for _ in range(reps):
            for lay in LAYOUTS:
                for op in OPS:
                    kept, red, swz = plan_of(lay)
                    kernels.reduce_f32(op, bufs[lay].ptr, R * C, 0, kept, red, out.ptr, swizzle=swz)
    elif case == "sharded":
        import torch

        fmt, rows = N.SW_MX_E4M3, M5 // 8
        a = quantize_generated(torch, N, kernels, fmt, rows, K5, seed=7000)
        b = quantize_generated(torch, N, kernels, fmt, N5, K5, seed=9000)
        c = N.DeviceBuffer(4 * rows * N5)
        rb = kernels.mx_row_bytes(fmt, K5)
        for _ in range(reps):
            kernels.mx_gemm(fmt, a[0].ptr, rb, a[1].ptr, b[0].ptr, rb, b[1].ptr, c.ptr, rows, N5, K5)
    elif case == "misc":
        profile_misc(N, kernels, reps)
    else:
        fmt = N.SW_MX_E4M3 if case == "mxfp8" else N.SW_MX_E2M1
        M = Nn = K = 8192
        rb = K if fmt == N.SW_MX_E4M3 else K // 2
        rng = np.random.default_rng(0)
        planes = []
        for rows, sigma in ((M, 1.0), (Nn, 0.02)):
            src = N.DeviceBuffer(rows * K * 4)
            src.upload((rng.standard_normal((rows, K)) * sigma).astype(np.float32))
            pay = N.DeviceBuffer(rows * rb)
            sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, K // 32))
            kernels.mx_quantize(fmt, src.ptr, rows, K, K, 1, pay.ptr, rb, sc.ptr)
            N.synchronize()
            src.free()
            planes.append((pay, sc))
        c = N.DeviceBuffer(M * Nn * 2)
        for _ in range(reps):
            kernels.mx_gemm(fmt, planes[0][0].ptr, rb, planes[0][1].ptr, planes[1][0].ptr, rb, planes[1][1].ptr,
                            c.ptr, M, Nn, K, out_bf16=True)
    N.raise_device_status()
    print(f"profile case {case}: ok")


def profile_misc(N, kernels, reps: int) -> None:
    """One launch each of the secondary kernels, on inputs larger than L2
    where the kernel is bandwidth-bound (see profile_case)."""
    rng = np.random.default_rng(3)
    n = 64 << 20  # 64 Mi floats: 256 MiB per operand
    xa, xb = N.DeviceBuffer(4 * n), N.DeviceBuffer(4 * n)
    xa.upload(rng.standard_normal(n, dtype=np.float32))
    xb.upload(rng.standard_normal(n, dtype=np.float32))
    loss, grad = N.DeviceBuffer(4), N.DeviceBuffer(4 * n)
    # batched MX contraction: 4 problems of 2048 x 2048 x 4096, fp32 C stacked
    fmt, bm, bk, nb = N.SW_MX_E4M3, 2048, 4096, 4
    src = N.DeviceBuffer(4 * nb * bm * bk)
    src.upload(rng.standard_normal(nb * bm * bk, dtype=np.float32))
    pay = N.DeviceBuffer(nb * bm * bk)
    sc = N.DeviceBuffer(kernels.scale_bytes_tc128(nb * bm, bk // 32))
    kernels.mx_quantize(fmt, src.ptr, nb * bm, bk, bk, 1, pay.ptr, bk, sc.ptr)
    cb = N.DeviceBuffer(4 * nb * bm * bm)
    # Float32 contraction 1024^3 (the reference's own plan, SIMT)
    mf = 1024
    # reductions' gradients and the view copy over the transposed X[8192 x 4096]
    go = N.DeviceBuffer(4 * R)
    go.upload(rng.standard_normal(R, dtype=np.float32))
    # view quantiser over the tiled + swizzled config-2 layout
    vq_pay, vq_sc = N.DeviceBuffer(R * C), N.DeviceBuffer(kernels.scale_bytes_tc128(R, C // 32))
    rm_sc = N.DeviceBuffer(R * (C // 32))
    pair = N.ctypes.c_int64 * 2  # out[i, j] = x[i, j] * go[i]: leaves (R, C), go broadcast along j
    shape, dense, bcast = pair(R, C), pair(C, 1), pair(1, 0)
    for _ in range(reps):
        kernels.mx_gemm_batched(fmt, pay.ptr, bk, sc.ptr, pay.ptr, bk, sc.ptr, cb.ptr, nb, bm, bm, bk)
        N.check(N.lib.sw_elementwise_f32(N.SW_EW_AXPY, n, N.c_void_p(xa.ptr), N.c_void_p(xb.ptr), N.c_void_p(xa.ptr),
                                         -1e-3, None))
        N.check(N.lib.sw_mse_f32(n, N.c_void_p(xa.ptr), N.c_void_p(xb.ptr), N.c_void_p(loss.ptr), None,
                                 N.c_void_p(grad.ptr), None))
        kernels.matmul_f32(xa.ptr, mf, 1, xb.ptr, mf, 1, grad.ptr, 1, mf, mf, mf, mf)
        for kind in ("reduce_sum", "reduce_max"):
            kernels.reduce_backward_f32(kind, xa.ptr, R * C, 0, [(R, 1)], [(C, R)], [], go.ptr, grad.ptr,
                                        [(R, C)], [(C, 1)], R * C)
        kernels.copy_view_f32(xa.ptr, R * C, 0, [(R, 1)], [(C, R)], grad.ptr, R * C, 0, [(R, C)], [(C, 1)])
        kernels.mx_quantize_view(fmt, xa.ptr, R * C, 0, [(128, 32), (64, 128 * 32 * 128)],
                                 [(32, 1), (128, 128 * 32)], vq_pay.ptr, C, vq_sc.ptr, swizzle=SWZ)
        kernels.mx_quantize(fmt, xa.ptr, R, C, C, 1, vq_pay.ptr, C, rm_sc.ptr, scale_layout=N.SW_SCALES_ROWMAJOR,
                            ld_scales=C // 32)
        kernels.mx_scales_to_tc128(rm_sc.ptr, C // 32, R, C // 32, vq_sc.ptr)
        N.check(N.lib.sw_binary_f32(N.SW_BIN_MUL, 2, shape, N.c_void_p(xa.ptr), 0, dense, R * C, N.c_void_p(go.ptr),
                                    0, bcast, R, N.c_void_p(grad.ptr), 0, dense, R * C, None))
        # the other view-quantiser walks: a transposed source (runs of whole
        # blocks at a stride), tiles whose rows do not abut (row pitch 64),
        # and a strided source through sw_mx_quantize
        kernels.mx_quantize_view(fmt, xa.ptr, R * C, 0, [(R, 1)], [(C, R)], vq_pay.ptr, C, vq_sc.ptr)
        kernels.mx_quantize_view(fmt, xa.ptr, 2 * R * C, 0, [(128, 64), (32, 64 * 128 * 128)],
                                 [(32, 1), (128, 64 * 128)], vq_pay.ptr, C, vq_sc.ptr)
        kernels.mx_quantize(fmt, xa.ptr, R, C // 2, 2 * C, 2, vq_pay.ptr, C // 2, vq_sc.ptr)
        # dequantisation of the row-quantised plane, and the peer K-split's
        # ordered sum of two 32 Mi-float slots
        kernels.mx_dequantize(fmt, vq_pay.ptr, C, rm_sc.ptr, R, C, grad.ptr, C, scale_layout=N.SW_SCALES_ROWMAJOR,
                              ld_scales=C // 32)
        N.check(N.lib.sw_sum_slots_f32(N.c_void_p(xa.ptr), n // 2, 2, N.c_void_p(grad.ptr), None))
        N.synchronize()


if __name__ == "__main__":
    main()
