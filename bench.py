"""Benchmark of the easy_as hot path on B200 (one JSON line on rank 0).

Workload: the SPMD ``add_kernel`` (c = a + b with masked
tail), N = 2**28 float32 elements (1 GiB per operand), BLOCK = 1024, a and b ~
N(0,1) from a seed.  The grid is split by contiguous program-id ranges across
the ranks (one process per GPU); each GPU holds only its slice and launches the
unmodified kernel on it, so there is no data-path collective ("strong"
scaling: the total N is fixed).  Inputs are 3 GiB per step in total (> 126 MB
L2), so no L2 flush is needed between steps.

* ``value``: aggregate GB/s = 12 B/element * N / max-over-ranks device time of
  K steps (CUDA events on the launch stream, barrier + synchronize around).
* ``e2e``: the same metric through the public API with host buffers (pinned
  torch CPU tensors): every step copies a and b host->device, launches and
  copies c back (c is never loaded by the kernel, so it is not copied in).
* ``roofline``: the add kernel's achieved bytes / launch time against the
  measured HBM copy peak (MEASURED_PEAKS.json).
* ``gemm``: the fp16 ``mk.dot`` GEMM (configs C4 8192^3 and C5 batched) TFLOP/s
  on the native tcgen05 path.
* ``matmul_tiled``: config C3, the reference's fp32 tiled matmul at 2048^3 on
  the proven-GEMM FFMA path (1 GPU), with cuBLAS fp32 timed beside it and the
  opt-in 3xTF32 mode (``tf32x3``).
* ``c1_add_call``: config C1 (N = 1031), launch-bound: the cost of one call
  through the public API (numpy synced, device async, CUDA-graph replay).
* ``cpu_baseline``: numpy on the host cores on a bounded sample.

``--impl reference`` times the reference's CPU semantics instead (the CPU
oracle interpreting the reference front end's IR of the same kernel, on all
host threads) and prints the same metric.
"""

import argparse
import json
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_TOTAL = 1 << 28
BLOCK = 1024
BYTES_PER_ELEM = 12
METRIC = "add HBM GB/s"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str) -> float | None:
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md ("traffic_bytes_per_launch: X")."""
    f = ROOT / "profiles" / f"{name}.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML (read-only) every 100 ms in the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples: list[float] = []
        self.max_mhz = None
        self.reasons: set[str] = set()
        self._stop = threading.Event()
        self._ready = threading.Event()
        self._thread = None
        self.error = None

    def _loop(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            while True:
                self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
                self._ready.set()
                if self._stop.wait(0.05):
                    break
        except Exception as e:  # NVML missing: report no samples rather than failing the bench
            self.error = repr(e)
        finally:
            self._ready.set()

    def __enter__(self):
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()
        self._ready.wait(timeout=10)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.samples)}
        if self.error:
            out["error"] = self.error
        return out


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(n_total: int, block: int, world: int, rank: int) -> tuple[int, int]:
    """Element range [lo, hi) of this rank: contiguous program-id range, whole programs only (the
    library's own split, ``easy_as_b200.shard.element_range``)."""
    from easy_as_b200.shard import element_range

    return element_range(n_total, block, rank, world)


def bench_gather(c, n_total: int, world: int, rank: int) -> dict:
    """The optional collective of the sharded path, reported beside the kernel numbers: the C2
    output slices gathered into one tensor on rank 0 (``easy_as_b200.shard.gather``: batched NCCL
    send/recv over NVLink/NVSwitch), checked against each rank's slice, timed from a barrier to
    the last rank's completion (max over ranks)."""
    import torch
    import torch.distributed as dist

    from easy_as_b200.shard import gather

    counts = [hi - lo for lo, hi in (shard(n_total, BLOCK, world, r) for r in range(world))]
    full = torch.empty(n_total, device="cuda") if rank == 0 else None
    gather(c, full, counts, dst=0)                       # warm-up (NCCL connections)
    torch.cuda.synchronize()
    reps = 3
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(reps):
        gather(c, full, counts, dst=0)
    torch.cuda.synchronize()
    dt = max_over_ranks((time.perf_counter() - t0) / reps, world)
    # exact check: every slice's bit pattern summed as int64, against the same ranges of `full`
    mine = c.view(torch.int32).to(torch.int64).sum().reshape(1)
    sums = [torch.zeros(1, dtype=torch.int64, device="cuda") for _ in range(world)]
    dist.all_gather(sums, mine)
    ok = True
    if rank == 0:
        off = 0
        for r, n in enumerate(counts):
            got = full[off:off + n].view(torch.int32).to(torch.int64).sum()
            ok = ok and bool(got == sums[r][0])
            off += n
    moved = 4 * (n_total - counts[0])
    del full
    return {"bytes_into_rank0": moved, "ms": round(dt * 1e3, 3), "GBs_into_rank0": round(moved / dt / 1e9, 1),
            "checked_rank0": ok,
            "how": "easy_as_b200.shard.gather (batched NCCL send/recv) of the C2 output slices to rank 0; "
                   "wall clock from a barrier, synchronised, max over ranks"}


def make_add_kernel():
    import eas
    from eas import mk

    @eas.kernel
    def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
        offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
        mask = offs < N
        mk.store(c, offs, mk.load(a, offs, mask) + mk.load(b, offs, mask), mask)

    return add_kernel


GEMM_CONFIGS = {
    # name: (batch, M, N, K, how the work is split across ranks)
    "C4": (1, 8192, 8192, 8192, "rows of A/C split across ranks, B replicated"),
    "C5": (64, 4096, 4096, 2088, "batch split across ranks"),
}


def gemm_shard(name: str, world: int, rank: int) -> tuple[int, int, int, int]:
    batch, M, N, K, _ = GEMM_CONFIGS[name]
    if name == "C4":
        r0, r1 = M * rank // world, M * (rank + 1) // world
        return batch, r1 - r0, N, K
    b0, b1 = batch * rank // world, batch * (rank + 1) // world
    return b1 - b0, M, N, K


def last_gemm_config() -> str:
    """The tile configuration the library's last GEMM launch used, as text."""
    import ctypes

    from easy_as_b200.runtime import cuda_ext

    vals = [ctypes.c_int() for _ in range(5)]
    cuda_ext.check(cuda_ext.load().eas_gemm_last_config(*(ctypes.byref(x) for x in vals)), "gemm config")
    tm, tn, st, ks, pair = (x.value for x in vals)
    kind = "tcgen05 cta_group::2 (CTA pair)" if pair else "tcgen05 cta_group::1"
    return f"{kind}, tile {tm}x{tn}x64, {st} stages" + (f", split-K x{ks}" if ks > 1 else "")


def gemm_e2e(name, a, b, c, M, N, K, batch, world, flops_total) -> dict:
    """The GEMM leg end to end through the public API with pinned host tensors: each step copies
    A and B in, runs the kernel and copies C out, synchronised; wall clock, max over ranks.  C is
    copied in too unless the launch provably stores every element of it (the runtime keeps any
    unwritten part of a host output intact)."""
    import torch

    from examples.matmul_dot_f16 import grid, matmul_dot_f16_tuned

    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.zeros(c.shape, dtype=torch.float32).pin_memory()

    def step():
        matmul_dot_f16_tuned(ha.reshape(-1), hb.reshape(-1), hc.reshape(-1), M, N, K, _grid=grid(batch))

    step()
    ref = ha[0, :4].double() @ hb[0].double()
    err = ((hc[0, :4].double() - ref).abs().max() / ref.abs().max()).item()
    if err > 1e-4:
        raise SystemExit(f"bench: {name} e2e result off by {err:.2e}")
    steps = 2
    from easy_as_b200.runtime import get_runtime

    rt = get_runtime()
    skipped0 = rt.skipped_copy_bytes
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = max_over_ranks((time.perf_counter() - t0) / steps, world)
    skipped = (rt.skipped_copy_bytes - skipped0) // steps   # C's copy-in when the GEMM stores all of C
    per_rank_in = ha.numel() * 2 + hb.numel() * 2 + hc.numel() * 4 - skipped
    per_rank_out = hc.numel() * 4
    del ha, hb, hc
    return {"value": round(flops_total / dt / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": per_rank_in * world, "d2h_bytes_per_step": per_rank_out * world,
            "ms_per_step": round(dt * 1e3, 2),
            "how": "public API, pinned torch CPU tensors in and out (A and B copied in; C copied in only when "
                   "the launch does not store all of it; C copied out), synchronised per step; wall clock, "
                   "max over ranks; PCIe-bound"}


def run_gemm(name: str, args, world: int, rank: int, rt) -> dict:
    """fp16 mk.dot GEMM (examples/matmul_dot_f16.py) on this rank's shard; TFLOP/s aggregated over ranks."""
    import torch

    from examples.matmul_dot_f16 import grid, matmul_dot_f16_tuned

    batch, M, N, K = gemm_shard(name, world, rank)
    tb, TM, TN, TK, split = GEMM_CONFIGS[name]
    g = torch.Generator(device="cuda").manual_seed(3 + rank)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.empty(batch, M, N, device="cuda")

    def step(sync=False):
        # autotuned over BLOCK_M/N in {128, 256} x BLOCK_K in {64, 128} (first call per shape tunes)
        matmul_dot_f16_tuned(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, _grid=grid(batch), _sync=sync)

    native0 = rt.native_launches
    step(sync=True)
    cfg = matmul_dot_f16_tuned._tuned_cache.get((M, N, K))
    tuned = dict(cfg.meta) if cfg is not None else {}
    if rt.native_launches == native0:
        raise SystemExit(f"bench: {name} did not take the tcgen05 path")
    # parity spot check: rows 0..3 of the first batch against float64
    ref = a[0, :4].double() @ b[0].double()
    err = ((c[0, :4].double() - ref).abs().max() / ref.abs().max()).item()
    if err > 1e-4:
        raise SystemExit(f"bench: {name} result off by {err:.2e}")
    steps = max(2, min(args.steps, args.gemm_steps))
    for _ in range(max(args.warmup, 3)):
        step()
    rt.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    launches0 = rt.launch_count
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        e1.synchronize()
        rt.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    ms_max = max_over_ranks(ms, world)
    lib_tf = None
    if world == 1:
        # cuBLAS on the same operands (f16 in, f32 out), timed the same way, for context
        try:
            def lib_step():
                torch.bmm(a, b, out_dtype=torch.float32)
            for _ in range(3):
                lib_step()
            torch.cuda.synchronize()
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record(stream)
            for _ in range(steps):
                lib_step()
            l1.record(stream)
            l1.synchronize()
            lib_tf = round(2.0 * batch * M * N * K / (l0.elapsed_time(l1) / steps * 1e-3) / 1e12, 1)
        except (TypeError, RuntimeError):
            lib_tf = None
    kernel_desc = last_gemm_config()
    flops_total = 2.0 * tb * TM * TN * TK
    flops_local = 2.0 * batch * M * N * K
    e2e = None if args.quick else gemm_e2e(name, a, b, c, M, N, K, batch, world, flops_total)
    pk = peaks()
    local_tf = flops_local / (ms * 1e-3) / 1e12
    return {
        "metric": "fp16 mk.dot GEMM TFLOP/s", "value": round(flops_total / (ms_max * 1e-3) / 1e12, 1),
        "unit": "TFLOP/s", "ms_per_step": round(ms_max, 4), "steps": steps,
        "config": {"workload": f"{name} batch={tb} M={TM} N={TN} K={TK} f16 in, f32 acc/out", "split": split,
                   "kernel": kernel_desc, "autotuned": tuned, "spot_check_rel_err": err},
        "roofline": {"bound": "tensor", "achieved": round(local_tf, 1), "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(local_tf / pk["bf16_tflops"], 4),
                     "peak_source": ("measured burst cuBLAS bf16 (MEASURED_PEAKS.json bf16_tflops)"
                                     if pk["source"] == "measured" else "fallback"),
                     "frac_of_nominal_2250": round(local_tf / 2250.0, 4),
                     "frac_of_measured_sustained": round(local_tf / pk["bf16_tflops_sustained"], 4),
                     "traffic": profile_traffic(f"gemm_{name.lower()}_n1")},
        "cublas_f16_f32out_tflops": lib_tf,
        "e2e": e2e,
        "cpu_baseline": (cpu_gemm_baseline(min(M, 2048), N, K, 1, 5, f"one {min(M, 2048)}-row slice of one problem "
                                           f"of the {name} workload (f16 inputs upcast to f32)")
                         if world == 1 and not args.no_cpu_baseline else None),
        "gpu_launches": rt.launch_count - launches0,
        "clocks": clk.summary(),
    }


C3_SIZE = 2048


def _c3_3xtf32(rt, ck, case, args_, grid, a, b, c, flush, steps, flops) -> dict:
    """The same C3 launch in the opt-in 3xTF32 mode (EAS_FP32_MATMUL=3xtf32): split kernels
    plus one tcgen05 kind::tf32 GEMM over K' = 3K, all inside the events; error vs float64 on
    64 rows."""
    import torch

    M = N = K = C3_SIZE
    old = os.environ.get("EAS_FP32_MATMUL")
    os.environ["EAS_FP32_MATMUL"] = "3xtf32"
    try:
        for _ in range(3):
            rt.run(ck, args_, case["meta"], grid=grid, sync=False)
        torch.cuda.synchronize()
        if ck.plan.native.last_mode != "3xtf32":
            return {"error": "3xTF32 mode declined: " + ck.plan.native.last_reason}
        ref = a.view(M, K)[:64].double() @ b.view(K, N).double()
        err = ((c.view(M, N)[:64].double() - ref).abs().max() / ref.abs().max()).item()
        stream = torch.cuda.current_stream()
        total = 0.0
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            rt.run(ck, args_, case["meta"], grid=grid, sync=False)
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
    finally:
        if old is None:
            os.environ.pop("EAS_FP32_MATMUL", None)
        else:
            os.environ["EAS_FP32_MATMUL"] = old
    ms = total / steps
    return {"tflops": round(flops / (ms * 1e-3) / 1e12, 2), "ms_per_step": round(ms, 4),
            "rel_err_vs_f64": err, "tolerance": 1e-4,
            "kernels": "2x eas_split_tf32 ([hi | lo] rows) + tcgen05 kind::tf32 GEMM over 3 K/32 k-blocks (opt-in; default stays exact)"}


def run_c1(args, rt) -> dict:
    """Config C1: the reference's own test case for add_kernel (N = 1031 = 1024 + 7, BLOCK = 256,
    a, b ~ N(0, 1) from seed 0, grid ceil(N / BLOCK)); a launch-bound workload, so the metric is
    the cost of one call:

    * ``numpy_sync_us``: numpy host arrays, as the reference's tests pass them (copies in, the
      kernel, the copy of c out, synchronised), wall clock per call;
    * ``device_async_us``: torch CUDA tensors, ``_sync=False``; host cost per launch over a
      burst (the GPU drains behind it), and ``device_us_per_launch`` from CUDA events;
    * ``graph_replay_us``: 100 launches captured in one CUDA graph, per launch on replay;
    * ``cpu_baseline``: the oracle interpreting the same compiled IR (``port``, 1 thread).
    Every path is checked bit-exact against a + b first."""
    import numpy as np
    import torch

    from oracle.interp import execute

    add_kernel = make_add_kernel()
    n, block = 1031, 256
    rng = np.random.default_rng(0)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c = np.zeros_like(a)
    add_kernel(a, b, c, n, BLOCK=block)
    if not np.array_equal(c, a + b):
        raise SystemExit("bench: C1 numpy result differs from a + b")
    calls = 2000
    t0 = time.perf_counter()
    for _ in range(calls):
        add_kernel(a, b, c, n, BLOCK=block)
    numpy_us = (time.perf_counter() - t0) / calls * 1e6

    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.zeros(n, device="cuda")
    launches0 = rt.launch_count
    for _ in range(10):
        add_kernel(da, db, dc, n, BLOCK=block, _sync=False)
    torch.cuda.synchronize()
    if not torch.equal(dc.cpu(), torch.from_numpy(a + b)):
        raise SystemExit("bench: C1 device result differs from a + b")
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(calls):
        add_kernel(da, db, dc, n, BLOCK=block, _sync=False)
    e1.record(stream)
    host_us = (time.perf_counter() - t0) / calls * 1e6
    torch.cuda.synchronize()
    dev_us = e0.elapsed_time(e1) * 1e3 / calls

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(100):
            add_kernel(da, db, dc, n, BLOCK=block, _sync=False)
    dc.zero_()
    g.replay()
    torch.cuda.synchronize()
    if not torch.equal(dc.cpu(), torch.from_numpy(a + b)):
        raise SystemExit("bench: C1 graph replay differs from a + b")
    reps = 20
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    graph_us = e0.elapsed_time(e1) * 1e3 / (reps * 100)

    ck = add_kernel.compile(a, b, c, n, BLOCK=block)
    want = np.zeros_like(a)
    execute(ck.ir, {"a": a, "b": b, "c": want, "N": n})
    t0 = time.perf_counter()
    cpu_calls = 0
    while time.perf_counter() - t0 < 2.0:
        execute(ck.ir, {"a": a, "b": b, "c": want, "N": n})
        cpu_calls += 1
    cpu_us = (time.perf_counter() - t0) / cpu_calls * 1e6
    return {
        "metric": "add_kernel per-call time", "unit": "us", "higher_is_better": False,
        "numpy_sync_us": round(numpy_us, 2), "device_async_us": round(host_us, 2),
        "device_us_per_launch": round(dev_us, 2), "graph_replay_us": round(graph_us, 3),
        "config": {"workload": "C1 add_kernel N=1031 (1024+7), BLOCK=256, grid 5, a, b ~ N(0,1) seed 0",
                   "calls": calls},
        "gpu_launches": rt.launch_count - launches0,
        "cpu_baseline": {"value": round(cpu_us, 1), "unit": "us", "cores": 1, "kind": "port",
                         "sample": f"oracle interpreting the same IR, {cpu_calls} calls in 2 s"},
    }


def run_tiled(args, rt) -> dict:
    """Config C3: the reference's unmodified fp32 tiled matmul (its front end's IR, committed as
    tests/golden/reference_ir_big.json.gz), M = N = K = 2048, 32x32x32 tiles, 256 threads per
    group, A, B ~ U(-1, 1).  The runtime proves the IR is a tiled GEMM and launches the
    FFMA kernel (bit-identical to the generated kernel).  Inputs (48 MB) fit in L2, so every
    timed step follows a 512 MB L2 flush outside its CUDA events."""
    import gzip

    import torch

    from easy_as_b200.compiler import compile_ir
    from easy_as_b200.ir import ir_from_json

    with gzip.open(ROOT / "tests" / "golden" / "reference_ir_big.json.gz", "rt") as f:
        case = next(c for c in json.load(f)["cases"] if c["id"] == "matmul_tiled_c3_full")
    ck = compile_ir(ir_from_json(case["opt"]))
    M = N = K = C3_SIZE
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.rand(M * K, device="cuda", generator=g) * 2 - 1
    b = torch.rand(K * N, device="cuda", generator=g) * 2 - 1
    c = torch.empty(M * N, device="cuda")
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    grid = (N // 32, M // 32, 1)
    args_ = {"a": a, "b": b, "c": c, "M": M, "N": N}

    def step():
        rt.run(ck, args_, case["meta"], grid=grid, sync=False)

    native0 = rt.native_launches
    step()
    torch.cuda.synchronize()
    if rt.native_launches == native0:
        raise SystemExit("bench: C3 did not take the native FFMA path: " + ck.plan.native.last_reason)
    ref = a.view(M, K)[:4].double() @ b.view(K, N).double()
    err = ((c.view(M, N)[:4].double() - ref).abs().max() / ref.abs().max()).item()
    if err > 1e-4:
        raise SystemExit(f"bench: C3 result off by {err:.2e}")
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    steps = max(5, args.steps)
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    launches0 = rt.launch_count
    with ClockSampler(torch.cuda.current_device()) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
    flops = 2.0 * M * N * K
    tf = flops / (ms * 1e-3) / 1e12
    cl = clk.summary()
    tf32x3 = _c3_3xtf32(rt, ck, case, args_, grid, a, b, c, flush, steps, flops)
    mhz = cl.get("sm_mhz") or 1965.0
    peak = 148 * 128 * 2 * mhz * 1e6 / 1e12
    # cuBLAS fp32 (TF32 off) on the same operands, for context
    torch.backends.cuda.matmul.allow_tf32 = False
    A2, B2 = a.view(M, K), b.view(K, N)
    for _ in range(3):
        torch.mm(A2, B2)
    lib_ms = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        torch.mm(A2, B2)
        e1.record(stream)
        e1.synchronize()
        lib_ms.append(e0.elapsed_time(e1))
    lib_tf = flops / (sum(lib_ms) / steps * 1e-3) / 1e12
    del flush
    return {
        "metric": "fp32 tiled matmul TFLOP/s", "value": round(tf, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
        "steps": steps, "dtype": "f32",
        "config": {"workload": "C3 matmul_tiled_full_kernel (reference IR) M=N=K=2048, BM=BN=BK=32, NT=256",
                   "kernel": "proven tiled GEMM -> FFMA sgemm_ffma 64x64x32 tiles, 8x4 per thread, cp.async "
                             "2-stage (128x128x32, 8x8 per thread from 4 waves of 128-tiles up)",
                   "l2": "512 MB flush before each timed step (outside the events)", "spot_check_rel_err": err},
        "roofline": {"bound": "fp32_fma", "achieved": round(tf, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(tf / peak, 4),
                     "peak_source": "nominal 148 SM x 128 FP32 lanes x 2 at the median sampled SM clock",
                     "traffic": profile_traffic("sgemm_c3_n1")},
        "cublas_fp32_tflops": round(lib_tf, 2),
        "tf32x3": tf32x3,
        "cpu_baseline": (None if args.no_cpu_baseline else
                         cpu_gemm_baseline(M, N, K, 1, 6, "the full C3 problem")),
        "gpu_launches": rt.launch_count - launches0,
        "clocks": cl,
    }


def cpu_gemm_baseline(m: int, n: int, k: int, batch: int, seed: int, what: str, seconds: float = 3.0) -> dict:
    """numpy (OpenBLAS, all host threads) float32 A @ B on a bounded sample of the same shape:
    repeated for about ``seconds``; fp16 operands are upcast to f32 first, as the reference's
    CPU-side check does."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    a @ b
    reps, t0 = 0, time.perf_counter()
    while True:
        a @ b
        reps += 1
        dt = time.perf_counter() - t0
        if dt > seconds:
            break
    tf = 2.0 * m * n * k * reps / dt / 1e12
    return {"value": round(tf, 4), "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"numpy float32 {m}x{k} @ {k}x{n} (OpenBLAS, all threads), {reps} reps in {dt:.1f} s; {what}"}


def cpu_add_baseline(seconds: float = 10.0) -> dict:
    """numpy add on the host cores over 2**24-element chunks for ~``seconds`` (all threads)."""
    cores = os.cpu_count() or 1
    n = 1 << 24
    rng = np.random.default_rng(1)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    outs = [np.empty_like(a) for _ in range(cores)]
    stop = time.perf_counter() + seconds
    done = [0] * cores

    def work(i):
        while time.perf_counter() < stop:
            np.add(a, b, out=outs[i])
            done[i] += 1

    t0 = time.perf_counter()
    with ThreadPoolExecutor(cores) as ex:
        list(ex.map(work, range(cores)))
    dt = time.perf_counter() - t0
    gbs = sum(done) * n * BYTES_PER_ELEM / dt / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"np.add on 2^24 float32 elements, repeated on {cores} threads for {dt:.1f} s"}


def run_eas(args) -> None:
    import torch

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    import eas
    from easy_as_b200.runtime import get_runtime

    rt = get_runtime()
    if args.only == "C3":
        print(json.dumps(run_tiled(args, rt)), flush=True)
        return
    if args.only == "C1":
        print(json.dumps(run_c1(args, rt)), flush=True)
        return
    if args.only in ("C4", "C5"):
        # profiling mode: one GEMM workload only
        res = run_gemm(args.only, args, world, rank, rt)
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    add_kernel = make_add_kernel()
    lo, hi = shard(args.n, BLOCK, world, rank)
    n = hi - lo
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    a = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    b = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    c = torch.empty_like(a)

    # correctness of the slice (bit-exact vs torch's own a + b)
    add_kernel(a, b, c, n, BLOCK=BLOCK)
    torch.cuda.synchronize()
    if not torch.equal(c, a + b):
        raise SystemExit("bench: add result differs from a + b")

    stream = torch.cuda.current_stream()
    t_warm = time.perf_counter()
    w = 0
    while w < max(args.warmup, 3) or (not args.quick and time.perf_counter() - t_warm < 0.5):
        add_kernel(a, b, c, n, BLOCK=BLOCK, _sync=False)
        w += 1
        if w % 64 == 0:
            rt.synchronize()
    rt.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    launches0 = rt.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            add_kernel(a, b, c, n, BLOCK=BLOCK, _sync=False)
        e1.record(stream)
        e1.synchronize()
        rt.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    launches = rt.launch_count - launches0
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, world)
    gbs = BYTES_PER_ELEM * args.n / (ms_max * 1e-3) / 1e9
    kernel_gbs_local = BYTES_PER_ELEM * n / (ms * 1e-3) / 1e9

    gather_res = None
    if world > 1 and not args.quick:
        gather_res = bench_gather(c, args.n, world, rank)

    # end to end through the public API with pinned host buffers
    e2e = None
    if not args.quick:
        ha = a.cpu().pin_memory()
        hb = b.cpu().pin_memory()
        hc = torch.empty(n, dtype=torch.float32).pin_memory()
        add_kernel(ha, hb, hc, n, BLOCK=BLOCK)
        barrier(world)
        t0 = time.perf_counter()
        e2e_steps = max(1, min(args.steps, 5))
        for _ in range(e2e_steps):
            add_kernel(ha, hb, hc, n, BLOCK=BLOCK)  # sync launch: H2D copies, kernel, D2H copy of c
        t_e2e = (time.perf_counter() - t0) / e2e_steps
        t_e2e = max_over_ranks(t_e2e, world)
        if not torch.equal(hc, ha + hb):
            raise SystemExit("bench: e2e add result differs from a + b")
        ck = add_kernel.compile(ha, hb, hc, n, BLOCK=BLOCK)
        ew = ck.plan.elementwise
        read_only_in = sorted(ew.reads) if ew is not None else ["a", "b", "c"]
        e2e = {"value": round(BYTES_PER_ELEM * args.n / t_e2e / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": len(read_only_in) * 4 * args.n, "d2h_bytes_per_step": 4 * args.n,
               "how": f"public API with pinned torch CPU tensors; {', '.join(read_only_in)} copied in, c copied "
                      "out, chunked so both PCIe directions overlap the kernel (c is never loaded by the kernel, "
                      "so it is not copied in); wall clock, max over ranks"}

    gemm = {}
    if not args.quick and not args.no_gemm:
        del a, b, c
        torch.cuda.empty_cache()
        for name in ("C4", "C5"):
            try:
                gemm[name] = run_gemm(name, args, world, rank, rt)
            except (SystemExit, Exception) as e:
                if world > 1:   # keep the ranks' collectives aligned: fail the whole run
                    raise
                gemm[name] = {"metric": "fp16 mk.dot GEMM TFLOP/s", "error": f"{type(e).__name__}: {e}"}
    tiled = None
    if not args.quick and not args.no_gemm and world == 1:
        try:
            tiled = run_tiled(args, rt)
        except (SystemExit, Exception) as e:  # a secondary leg never suppresses the headline line
            tiled = {"metric": "fp32 tiled matmul TFLOP/s", "error": f"{type(e).__name__}: {e}"}
    c1 = None
    if not args.quick and world == 1:
        try:
            c1 = run_c1(args, rt)
        except (SystemExit, Exception) as e:
            c1 = {"metric": "add_kernel per-call time", "error": f"{type(e).__name__}: {e}"}
    if rank != 0:
        return
    pk = peaks()
    traffic = profile_traffic("add_c2_n1")
    line = {
        "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_max, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (torch.randn, seeded)",
        "config": {"workload": "C2 add_kernel N=2^28 f32, BLOCK=1024, program-id ranges split across GPUs",
                   "N": args.n, "BLOCK": BLOCK, "per_gpu_elements": n, "parallelism": f"pid-shard x{world}",
                   "l2": "inputs 3 GiB/step > 126 MB L2 (no flush needed)"},
        "e2e": e2e,
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs_local, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(kernel_gbs_local / pk["hbm_gbs"], 4),
                     "traffic": traffic, "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs)"
                     if pk["source"] == "measured" else "fallback"},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if gather_res is not None:
        line["gather"] = gather_res
    if gemm:
        line["gemm"] = gemm
    if tiled is not None:
        line["matmul_tiled"] = tiled
    if c1 is not None:
        line["c1_add_call"] = c1
    if world == 1 and not args.no_cpu_baseline and not args.quick:
        line["cpu_baseline"] = cpu_add_baseline(args.cpu_seconds)
    print(json.dumps(line), flush=True)


def run_reference(args) -> None:
    """CPU semantics of the reference (oracle interpreting the reference front end's add IR)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "tests"))
    import goldens
    from oracle.interp import execute

    case = goldens.case("add_block1024")
    ir = goldens.ir_from_json(case["opt"])
    cores = os.cpu_count() or 1
    # bounded sample per step: 2^22 elements per thread-chunk (about 0.4 s per step on 16 cores),
    # halved for every doubling of the step count past 100 so the whole run stays within minutes
    shrink = 0
    while (args.steps >> shrink) > 100 and shrink < 6:
        shrink += 1
    n = 1 << (22 - shrink)
    rng = np.random.default_rng(1)
    a = rng.standard_normal(n * cores, dtype=np.float32)
    b = rng.standard_normal(n * cores, dtype=np.float32)
    c = np.zeros_like(a)

    def chunk(i):
        sl = slice(i * n, (i + 1) * n)
        execute(ir, {"a": a[sl], "b": b[sl], "c": c[sl], "N": n})

    def step():
        with ThreadPoolExecutor(cores) as ex:
            list(ex.map(chunk, range(cores)))

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    assert np.array_equal(c, a + b)
    gbs = BYTES_PER_ELEM * n * cores / dt / 1e9
    sample = f"{cores} x 2^{22 - shrink}-element chunks of the C2 add per step (oracle interpreter, {cores} threads)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy default_rng(1))",
        "config": {"workload": "C2 add_kernel N=2^28 f32, BLOCK=1024 (bounded CPU sample)", "N": N_TOTAL,
                   "BLOCK": BLOCK},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="eas", choices=["eas", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--n", type=int, default=N_TOTAL, help="total elements (profiling runs use a smaller case)")
    ap.add_argument("--no-gemm", action="store_true", help="skip the fp16 GEMM configs (C4, C5)")
    ap.add_argument("--only", choices=["all", "C1", "C3", "C4", "C5"], default="all",
                    help="run a single secondary workload (profiling)")
    ap.add_argument("--gemm-steps", type=int, default=20)
    ap.add_argument("--quick", action="store_true",
                    help="profiling mode: no clock warm-up loop, no e2e arm, no CPU baseline")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_eas(args)
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.barrier()
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
