"""Benchmark of the B200 StrideWeave carrier hot path.

Default workload: layout-aware Float32 reductions - sum,
max and argmax over mode 1 of X[8192 x 4096] ~ U(-1, 1), on (a) a row-major
layout, (b) a transposed stride layout and (c) a hierarchical tiled layout
((128,64),(32,128)) stored through a 3-bit swizzle.  One step = the 9
reductions.  The line also carries the MX contractions of configs 1 and 3
(MXFP8 / MXFP4, M=N=K=8192) measured on the same device.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Inputs are larger than L2 (each layout's X is 128 MiB, and consecutive
launches read different buffers), timing is by CUDA events on the launching
stream, and the multi-GPU value is the max over ranks (weak scaling: each
rank reduces its own X, there is no collective on the data path).
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
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


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
# reference arm: the reference CPU carrier on the host cores


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.append(str(ROOT / "baseline" / "_ref"))
    try:
        import strideweave as sw
        from strideweave import CPU, Layout, Shape, Stride, Tensor
    except Exception as exc:  # pragma: no cover - reported, not raised
        print(json.dumps({"impl": "reference", "unavailable": f"reference not importable: {exc}"}))
        return
    from concurrent.futures import ThreadPoolExecutor

    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, size=(R, C)).astype(np.float32)
    # The reference cannot place a tensor through a Swizzle: layout (c) runs on
    # the tiled layout over un-swizzled storage (the logical data it reduces is
    # the same).
    stores = {
        "rowmajor": np.ascontiguousarray(x).ravel(),
        "transposed": np.ascontiguousarray(x.T).ravel(),
        "tiled_swizzled": np.ascontiguousarray(x.reshape(64, 128, 128, 32).transpose(0, 2, 1, 3)).ravel(),
    }
    layouts = {
        "rowmajor": Layout(Shape([R, C]), Stride([C, 1])),
        "transposed": Layout(Shape([R, C]), Stride([1, R])),
        "tiled_swizzled": Layout(Shape([[128, 64], [32, 128]]), Stride([[32, 128 * 32 * 128], [1, 128 * 32]])),
    }
    threads = os.cpu_count() or 1
    fns = {"reduce_sum": sw.reduce_sum, "reduce_max": sw.reduce_max, "argmax": sw.argmax}
    carriers = {k: CPU(v.size, pointer=v.ctypes.data) for k, v in stores.items()}

    def slice_job(layout, op, lo, hi):
        # rows lo..hi of the kept mode as a zero-copy view (the reference
        # kernels are single-threaded; slices run on separate host threads)
        base = Tensor(carriers[layout], 0, layouts[layout])
        view = base[lo:hi, :] if layout != "tiled_swizzled" else None
        if view is None:
            # tiled layout: slice whole 128-row tiles through the outer leaf
            tlo, thi = lo // 128, hi // 128
            view = Tensor(carriers[layout], tlo * 128 * 32 * 128,
                          Layout(Shape([[128, thi - tlo], [32, 128]]), Stride([[32, 128 * 32 * 128], [1, 128 * 32]])))
        with sw.no_grad():
            return fns[op](view, "a b -> a")

    bounds = [(i * R // threads // 128 * 128, (i + 1) * R // threads // 128 * 128) for i in range(threads)]
    bounds[-1] = (bounds[-1][0], R)

    def step(pool):
        futures = [pool.submit(slice_job, lay, op, lo, hi) for op in OPS for lay in LAYOUTS for lo, hi in bounds
                   if hi > lo]
        for f in futures:
            f.result()

    with ThreadPoolExecutor(threads) as pool:
        for _ in range(args.warmup):
            step(pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(pool)
        dt = (time.perf_counter() - t0) / args.steps
    value = 9 * RED_BYTES / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "reduction HBM GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2_reductions_8192x4096", "ops": list(OPS), "layouts": list(LAYOUTS)},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": "full X[8192x4096] per step, kept rows split over host threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------------------------
# our arm


def cpu_baseline_sample() -> dict:
    """The reference CPU carrier on a bounded sample (rank 0, N=1 only)."""
    sys.path.append(str(ROOT / "baseline" / "_ref"))
    try:
        import strideweave as sw
        from strideweave import CPU, Layout, Shape, Stride, Tensor
        kind = "reference"
    except Exception:
        sw = None
        kind = "port"
    rng = np.random.default_rng(1)
    rows = 2048  # a quarter of X: ~1/4 of the config's work per op
    x = rng.uniform(-1, 1, size=(rows, C)).astype(np.float32)
    t0 = time.perf_counter()
    if kind == "reference":
        store_a = np.ascontiguousarray(x).ravel()
        store_b = np.ascontiguousarray(x.T).ravel()
        ta = Tensor(CPU(store_a.size, pointer=store_a.ctypes.data), 0, Layout(Shape([rows, C]), Stride([C, 1])))
        tb = Tensor(CPU(store_b.size, pointer=store_b.ctypes.data), 0, Layout(Shape([rows, C]), Stride([1, rows])))
        with sw.no_grad():
            for fn in (sw.reduce_sum, sw.reduce_max, sw.argmax):
                fn(ta, "a b -> a")
                fn(tb, "a b -> a")
        n_ops = 6
    else:
        from oracle import oracle as O
        flat = np.ascontiguousarray(x).ravel()
        for k in ("sum", "max", "argmax"):
            O.reduce(k, flat, 0, [(rows, C)], [(C, 1)])
        n_ops = 3
    dt = time.perf_counter() - t0
    gbs = n_ops * (rows * C * 4 + rows * 4) / dt / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{n_ops} reductions over X[{rows}x{C}] (row-major and transposed), single-threaded kernels"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-gemm", action="store_true", help="skip the contraction measurements")
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="untimed busy time under the clock sampler before the timed region")
    ap.add_argument("--profile-case", choices=["reduce", "quantize", "dual", "mxfp8", "mxfp4", "mlp"],
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
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    from strideweave_b200 import _native as N
    from strideweave_b200 import kernels

    N.set_device(local)
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream

    rng = np.random.default_rng(1234 + rank)
    x = rng.uniform(-1, 1, size=(R, C)).astype(np.float32)
    host = {lay: storage_of(lay, x) for lay in LAYOUTS}
    dev = {lay: N.DeviceBuffer(X_BYTES) for lay in LAYOUTS}
    for lay in LAYOUTS:
        dev[lay].upload(host[lay])
    outs = {(op, lay): N.DeviceBuffer(R * 4) for op in OPS for lay in LAYOUTS}
    N.synchronize()

    # consecutive launches read different 128 MiB buffers (> L2)
    order = [(op, lay) for op in OPS for lay in LAYOUTS]

    # plans are built once: the timed loop is one C call per launch, so the
    # host stays ahead of the device
    plans = {}
    for op in OPS:
        for lay in LAYOUTS:
            kept, red, swz = plan_of(lay)
            plans[(op, lay)] = kernels.make_reduce_plan(op, 0, kept, red, swz)
    stream_arg = N.c_void_p(s)

    def launch_on(op, lay, ptr):
        N.check(N.lib.sw_reduce_f32(N.ctypes.byref(plans[(op, lay)]), N.c_void_p(ptr), R * C,
                                    N.c_void_p(outs[(op, lay)].ptr), stream_arg))

    def launch(op, lay):
        launch_on(op, lay, dev[lay].ptr)

    clocks = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        for op, lay in order:
            launch(op, lay)
    torch.cuda.synchronize()
    # keep the device busy ~1 s under the clock sampler before timing
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_seconds:
        for op, lay in order:
            launch(op, lay)
        torch.cuda.synchronize()

    # -------- timed region: device-resident inputs --------
    # One event pair brackets the K steps: an event recorded between two
    # launches costs the stream a few microseconds, which the step itself
    # does not spend.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for it in range(args.steps):
        for op, lay in order:
            launch(op, lay)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(end)
    t = torch.tensor([total_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    value = world * 9 * RED_BYTES / (ms_per_step / 1e3) / 1e9

    # -------- per-kernel durations (roofline): each kernel launched back to
    # back over rotating inputs, one event pair per run of launches --------
    # A second copy of each layout alternates with the first, so consecutive
    # launches read 256 MiB (> L2).
    spare = {lay: N.DeviceBuffer(X_BYTES) for lay in LAYOUTS}
    for lay in LAYOUTS:
        N.check(N.lib.sw_memcpy_d2d(N.c_void_p(spare[lay].ptr), N.c_void_p(dev[lay].ptr), X_BYTES, stream_arg))
    per_kernel = {}
    runs = max(6, args.steps // 3)
    for op in OPS:
        for lay in LAYOUTS:
            bufs = (dev[lay].ptr, spare[lay].ptr)
            launch_on(op, lay, bufs[0])
            k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            k0.record(stream)
            for r in range(runs):
                launch_on(op, lay, bufs[(r + 1) % 2])
            k1.record(stream)
            torch.cuda.synchronize()
            per_kernel[(op, lay)] = k0.elapsed_time(k1) / runs
    time.sleep(0.25)
    clocks.__exit__(None, None, None)

    # correctness spot check of what was timed (device vs the sequential rule)
    check = np.empty(R, dtype=np.float32)
    outs[("reduce_max", "rowmajor")].download(check)
    assert np.array_equal(check, x.max(axis=1)), "timed reduce_max disagrees with numpy"

    # -------- end-to-end: pinned host input -> device -> reduce -> host --------
    pinned = {lay: torch.from_numpy(host[lay]).pin_memory() for lay in LAYOUTS}
    res_host = torch.empty(R * 9, dtype=torch.float32).pin_memory()
    e2e_steps = max(3, args.steps // 4)

    def e2e_step():
        for lay in LAYOUTS:
            N.check(N.lib.sw_memcpy_h2d(N.c_void_p(dev[lay].ptr), N.c_void_p(pinned[lay].data_ptr()), X_BYTES,
                                        N.c_void_p(s)))
        for j, (op, lay) in enumerate(order):
            launch(op, lay)
        for j, (op, lay) in enumerate(order):
            N.check(N.lib.sw_memcpy_d2h(N.c_void_p(res_host.data_ptr() + 4 * R * j), N.c_void_p(outs[(op, lay)].ptr),
                                        R * 4, N.c_void_p(s)))

    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / e2e_steps
    e2e_value = world * 9 * RED_BYTES / (e2e_ms / 1e3) / 1e9

    # -------- contractions (configs 1 and 3) on this device --------
    contraction = None
    quantize = None
    sharded = None
    mlp = None
    if not args.no_gemm:
        quantize = bench_quantize(torch, N, kernels, s, stream)
        contraction = bench_gemm(torch, N, kernels, s, stream)
        # config 5 at this world size (strong scaling of a fixed contraction)
        sharded = {m: bench_sharded(torch, dist, N, kernels, m, world, rank) for m in ("m", "k")}
        mlp = bench_mlp(torch, N)

    if rank == 0:
        peaks = load_peaks()
        by_layout = {lay: sum(per_kernel[(op, lay)] for op in OPS) for lay in LAYOUTS}
        dominant = max(by_layout, key=by_layout.get)
        dom_ms = by_layout[dominant] / 3
        achieved = RED_BYTES / (dom_ms / 1e3) / 1e9
        line = {
            "metric": "reduction HBM GB/s",
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic U(-1,1), seeded",
            "config": {"workload": "config2_reductions_8192x4096", "ops": list(OPS), "layouts": list(LAYOUTS),
                       "step": "9 reductions (3 ops x 3 layouts)", "l2": "inputs larger than L2, rotated",
                       "parallelism": f"replicas x{world} (each rank its own X)"},
            "roofline": {"bound": "hbm", "kernel": f"sw_reduce_f32[{dominant}]", "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"], "traffic": NCU_TRAFFIC.get(dominant),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, mean of the "
                                           "layout's three kernels, from the committed --set full capture",
                         "per_layout_gbs": {lay: round(3 * RED_BYTES / (by_layout[lay] / 1e3) / 1e9, 1)
                                            for lay in LAYOUTS},
                         "per_kernel_gbs": {f"{op}/{lay}": round(RED_BYTES / (per_kernel[(op, lay)] / 1e3) / 1e9, 1)
                                            for op, lay in order}},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 3 * X_BYTES,
                    "d2h_bytes_per_step": 9 * R * 4},
            "gpu_launches": 9 * args.steps,
            "clocks": clocks.summary(),
        }
        if quantize:
            line["quantize"] = quantize
        if contraction:
            line["contraction"] = contraction
        if sharded:
            line["sharded_contraction"] = {"m_split": sharded["m"], "k_split": sharded["k"]}
        if mlp:
            line["mlp_step"] = mlp
        if world == 1:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    N.raise_device_status()
    return out


def quantize_generated(torch, N, kernels, fmt, rows, cols, seed, sigma=1.0, block=8192):
    """Device planes of a seeded N(0, sigma^2) [rows, cols] operand, generated
    and quantised in row blocks (bounded Float32 staging)."""
    rb = kernels.mx_row_bytes(fmt, cols)
    katoms = (cols // 32 + 3) // 4
    pay = N.DeviceBuffer(rows * rb)
    sc = N.DeviceBuffer(kernels.scale_bytes_tc128(rows, cols // 32))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    s = torch.cuda.current_stream().cuda_stream
    for r0 in range(0, rows, block):
        n = min(block, rows - r0)
        x = torch.randn((n, cols), generator=gen, device="cuda", dtype=torch.float32) * sigma
        kernels.mx_quantize(fmt, x.data_ptr(), n, cols, cols, 1, pay.ptr + r0 * rb, rb,
                            sc.ptr + (r0 // 128) * katoms * 512, stream=s)
        del x
    return pay, sc


def bench_sharded(torch, dist, N, kernels, mode, world, rank, steps=5, warmup=2) -> dict:
    """Config 5: sharded MXFP8 contraction M=65536, N=16384, K=16384, inputs
    N(0,1), at `world` GPUs; M-split (B replicated, no collective) or K-split
    (NCCL reduce-scatter of Float32 partials, overlapped over 8 N-chunks; the
    contractions leave 32 SMs to the collective so the two run side by side)."""
    from strideweave_b200.sharding import MXShardedContraction, ShardPlan

    M, Nn, K = 65536, 16384, 16384
    fmt = N.SW_MX_E4M3
    plan = ShardPlan(mode, world, rank, M, Nn, K, k_quantum=128, chunks=8 if mode == "k" else 1)
    rows = plan.rows_local if mode == "m" else M
    a = quantize_generated(torch, N, kernels, fmt, rows, plan.k_local, seed=7000 + rank)
    b = quantize_generated(torch, N, kernels, fmt, Nn, plan.k_local, seed=9000 + (rank if mode == "k" else 0))
    op = MXShardedContraction(plan, fmt, a, b)
    for _ in range(warmup):
        op.run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        op.run()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tflops = 2.0 * M * Nn * K / (ms / 1e3) / 1e12
    N.raise_device_status()
    del op, a, b
    torch.cuda.empty_cache()
    return {"tflops": round(tflops, 1), "ms": round(ms, 3), "n_gpus": world, "scaling": "strong",
            "config": f"MXFP8 M=65536 N=16384 K=16384, {'M-split' if mode == 'm' else 'K-split + NCCL reduce-scatter, 8 N-chunks, 32 SMs left to the collective'}"}


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
    operands, then `reps` contractions at M = N = K = 8192 (bf16 C).  mlp: the
    MLP training step, `reps` steps after one warm-up step.
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


if __name__ == "__main__":
    main()
