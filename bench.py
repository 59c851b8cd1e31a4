"""Benchmark of the easy_as hot path on B200 (one JSON line on rank 0).

Headline: the SPMD ``add_kernel`` (c = a + b with masked
tail), N = 2**28 float32 elements (1 GiB per operand), BLOCK = 1024.  Every
rank runs its contiguous program-id range of the one launch through the
library's shard path (``easy_as_b200.shard.run_shard`` with ``_buffer_base``:
each GPU allocates only its slice), so there is no data-path collective and
the total N is fixed ("strong" scaling).  Inputs are 3 GiB per step (> 126 MB
L2), so no L2 flush is needed.

The GEMM configs go through the same shard path: C4 (8192^3, autotuned over
BLOCK_M x BLOCK_N x BLOCK_K) split by rows (program_id(1)), C5 (64 x 4096^2 x
2088) by batch (program_id(2)); C3 and C1 run on one GPU.  Their compact
summaries sit in ``configs`` of the same line.  ``--impl reference`` times the
reference's CPU semantics (the oracle interpreting the reference front end's
IR of the same kernel, all host threads) on the full C2 problem.
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

    def summary(self, short: bool = False) -> dict:
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.samples)}
        if short:
            out = {"sm_mhz": out["sm_mhz"], "reasons": out["reasons"]}
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
            "checked_rank0": ok}


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
    # name: (batch, M, N, K, shard axis: 1 = rows of A and C (program_id(1)), 2 = batch (program_id(2)))
    "C4": (1, 8192, 8192, 8192, 1),
    "C5": (64, 4096, 4096, 2088, 2),
}


def last_gemm_config() -> str:
    """The tile configuration of the library's last GEMM launch, as short text."""
    import ctypes

    from easy_as_b200.runtime import cuda_ext

    vals = [ctypes.c_int() for _ in range(6)]
    cuda_ext.check(cuda_ext.load().eas_gemm_last_config(*(ctypes.byref(x) for x in vals)), "gemm config")
    tm, tn, st, ks, pair, bk = (x.value for x in vals)
    return (f"{'pair' if pair else '1sm'} {tm}x{tn}x{bk} s{st}" + (f" splitk{ks}" if ks > 1 else ""))


def _events():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def run_gemm(name: str, args, world: int, rank: int, rt) -> dict:
    """fp16 mk.dot GEMM (examples/matmul_dot_f16.py, autotuned) through ``shard.run_shard``: this
    rank's program-id range of the one launch, on buffers that hold only its slice (B whole for C4);
    TFLOP/s aggregated over ranks from the max-over-ranks device time."""
    import torch

    from easy_as_b200.shard import program_range, run_shard
    from examples.matmul_dot_f16 import grid, matmul_dot_f16_tuned as kern

    batch, M, N, K, axis = GEMM_CONFIGS[name]
    p0, p1 = program_range(M if axis == 1 else batch, rank, world)
    if axis == 1:   # rows p0..p1 of A and C; B whole
        lb, lm, base = 1, p1 - p0, {"a": p0 * K, "c": p0 * N}
        bshape = (1, K, N)
    else:           # batches p0..p1 of A, B and C
        lb, lm, base = p1 - p0, M, {"a": p0 * M * K, "b": p0 * K * N, "c": p0 * M * N}
        bshape = (lb, K, N)
    g = torch.Generator(device="cuda").manual_seed(3 + rank)
    a = (torch.randn(lb, lm, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(*bshape, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.empty(lb, lm, N, device="cuda")

    def step(sync=False):
        run_shard(kern, a, b, c, M, N, K, _grid=grid(batch), _rank=rank, _world=world, _axis=axis,
                  _buffer_base=base, _sync=sync)

    native0 = rt.native_launches
    keys0 = set(kern._tuned_cache)
    step(sync=True)                      # first call tunes (8 configs timed on this rank's range)
    if rt.native_launches == native0:
        raise SystemExit(f"bench: {name} did not take the tcgen05 path")
    new = [k for k in kern._tuned_cache if k not in keys0]
    best = dict(kern._tuned_cache[new[0]].meta) if new else {}
    times = kern._tuned_times.get(new[0], []) if new else []
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
    e0, e1 = _events()
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda._sleep(100_000)      # the first step is queued before the start event is reached
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        e1.synchronize()
    launches = rt.launch_count - launches0
    rt.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    ms_max = max_over_ranks(ms, world)
    tile = last_gemm_config()
    lib_tf = None
    if world == 1:
        # cuBLAS on the same operands (f16 in, f32 out), timed the same way, for context
        try:
            for _ in range(3):
                torch.bmm(a, b, out_dtype=torch.float32)
            torch.cuda.synchronize()
            l0, l1 = _events()
            l0.record(stream)
            for _ in range(steps):
                torch.bmm(a, b, out_dtype=torch.float32)
            l1.record(stream)
            l1.synchronize()
            lib_tf = round(2.0 * lb * lm * N * K / (l0.elapsed_time(l1) / steps * 1e-3) / 1e12, 1)
        except (TypeError, RuntimeError):
            lib_tf = None
    flops_total = 2.0 * batch * M * N * K
    local_tf = 2.0 * lb * lm * N * K / (ms * 1e-3) / 1e12
    e2e = None if args.quick else gemm_e2e(name, a, b, c, step, world, flops_total, best)
    pk = peaks()
    out = {
        "value": round(flops_total / (ms_max * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms_max, 4),
        "steps": steps,
        "roofline": {"bound": "tensor", "achieved": round(local_tf, 1), "peak": pk["bf16_tflops"],
                     "frac": round(local_tf / pk["bf16_tflops"], 4),
                     "frac_sustained": round(local_tf / pk["bf16_tflops_sustained"], 4),
                     "frac_nominal": round(local_tf / 2250.0, 4),
                     "traffic": profile_traffic(f"gemm_{name.lower()}_n1") if world == 1 else None},
        "clocks": clk.summary(short=True), "tile": tile,
        "tuned": "/".join(str(best.get(k)) for k in ("BLOCK_M", "BLOCK_N", "BLOCK_K")) if best else None,
        "tune_ms": [round(t * 1e3, 3) for _, t in times] if world == 1 else None,
        "cublas": lib_tf, "e2e": e2e, "gpu_launches": launches, "rel_err": float(f"{err:.2e}"),
    }
    if world == 1 and not args.no_cpu_baseline and not args.quick:
        out["cpu_tflops"] = cpu_gemm_baseline(min(M, 2048), N, K, 5)["value"]
    return out


def gemm_e2e(name, a, b, c, step, world, flops_total, best: dict) -> dict:
    """The GEMM end to end with pinned host tensors, synchronised per step, wall clock, max over ranks.
    One GPU: the public call with host tensors and the tuned tile configuration (the runtime
    pipelines the copies with the kernel).
    N GPUs: every rank copies its slices in, runs its range (``run_shard``) and copies its C out."""
    import torch

    from examples.matmul_dot_f16 import grid, matmul_dot_f16

    batch, M, N, K, _ = GEMM_CONFIGS[name]
    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.zeros(c.shape, dtype=torch.float32).pin_memory()
    from easy_as_b200.runtime import get_runtime

    rt = get_runtime()
    if world == 1:
        def e2e_step():
            matmul_dot_f16(ha.reshape(-1), hb.reshape(-1), hc.reshape(-1), M, N, K, **best, _grid=grid(batch))
    else:
        def e2e_step():
            a.copy_(ha, non_blocking=True)
            b.copy_(hb, non_blocking=True)
            step()
            hc.copy_(c, non_blocking=True)
            torch.cuda.synchronize()
    e2e_step()
    ref = ha[0, :4].double() @ hb[0].double()
    err = ((hc[0, :4].double() - ref).abs().max() / ref.abs().max()).item()
    if err > 1e-4:
        raise SystemExit(f"bench: {name} e2e result off by {err:.2e}")
    steps = 2
    skipped0 = rt.skipped_copy_bytes
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        e2e_step()
    dt = max_over_ranks((time.perf_counter() - t0) / steps, world)
    skipped = (rt.skipped_copy_bytes - skipped0) // steps   # C's copy-in when the GEMM stores all of C
    per_rank_in = ha.numel() * 2 + hb.numel() * 2 + (hc.numel() * 4 - skipped if world == 1 else 0)
    per_rank_out = hc.numel() * 4
    del ha, hb, hc
    return {"value": round(flops_total / dt / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(sum_over_ranks(per_rank_in, world)),
            "d2h_bytes_per_step": int(sum_over_ranks(per_rank_out, world))}


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
                         cpu_gemm_baseline(M, N, K, 6)),
        "gpu_launches": rt.launch_count - launches0,
        "clocks": cl,
    }


def cpu_gemm_baseline(m: int, n: int, k: int, seed: int, seconds: float = 3.0) -> dict:
    """numpy (OpenBLAS, all host threads) float32 A @ B on a bounded sample of the same shape,
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
            "sample": f"numpy f32 {m}x{k}@{k}x{n}, {reps} reps"}


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
            "sample": f"np.add 2^24 f32, {cores} threads, {dt:.0f} s"}


def run_add(args, world: int, rank: int, local: int, rt) -> dict:
    """Config C2 through ``shard.run_shard``: this rank's program-id range of the one N-element
    launch, on slice-only buffers (``_buffer_base``)."""
    import torch

    from easy_as_b200.shard import run_shard

    add_kernel = make_add_kernel()
    lo, hi = shard(args.n, BLOCK, world, rank)
    n = hi - lo
    base = {"a": lo, "b": lo, "c": lo}
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    a = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    b = torch.randn(n, device="cuda", dtype=torch.float32, generator=gen)
    c = torch.empty_like(a)

    def step(sync=False):
        run_shard(add_kernel, a, b, c, args.n, BLOCK=BLOCK, _rank=rank, _world=world, _buffer_base=base, _sync=sync)

    step(sync=True)
    if not torch.equal(c, a + b):            # bit-exact vs torch's own a + b
        raise SystemExit("bench: add result differs from a + b")
    stream = torch.cuda.current_stream()
    t_warm = time.perf_counter()
    w = 0
    while w < max(args.warmup, 3) or (not args.quick and time.perf_counter() - t_warm < 0.5):
        step()
        w += 1
        if w % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    launches0 = rt.launch_count
    e0, e1 = _events()
    with ClockSampler(local) as clk:
        # a ~50 us device sleep ahead of the start event, so the first step is already queued when
        # the event is reached (the timed region holds the K steps back to back, not the host's
        # latency to launch the first one)
        torch.cuda._sleep(100_000)
        e0.record(stream)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        host_us = (time.perf_counter() - t0) / args.steps * 1e6
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    launches = rt.launch_count - launches0
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, world)
    res = {"gbs": BYTES_PER_ELEM * args.n / (ms_max * 1e-3) / 1e9, "ms": ms_max, "n": n,
           "kernel_gbs": BYTES_PER_ELEM * n / (ms * 1e-3) / 1e9, "launches": launches, "clocks": clk.summary(),
           "host_us": host_us}
    if world > 1 and not args.quick:
        res["gather"] = bench_gather(c, args.n, world, rank)
    if not args.quick:
        res["e2e"] = add_e2e(args, add_kernel, a, b, c, step, world, n)
    return res


def add_e2e(args, add_kernel, a, b, c, step, world: int, n: int) -> dict:
    """C2 end to end with pinned host buffers, wall clock, max over ranks.  One GPU: the public call
    with host tensors (a and b copied in, c copied out, chunked so both PCIe directions overlap the
    kernel; c is never loaded, so it is not copied in).  N GPUs: each rank copies its slices in,
    runs its range and copies its c out."""
    import torch

    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.empty(n, dtype=torch.float32).pin_memory()
    if world == 1:
        def e2e_step():
            add_kernel(ha, hb, hc, n, BLOCK=BLOCK)   # synchronous call: copies in, kernel, copy of c out
    else:
        def e2e_step():
            a.copy_(ha, non_blocking=True)
            b.copy_(hb, non_blocking=True)
            step()
            hc.copy_(c, non_blocking=True)
            torch.cuda.synchronize()
    e2e_step()
    barrier(world)
    t0 = time.perf_counter()
    steps = max(1, min(args.steps, 5))
    for _ in range(steps):
        e2e_step()
    dt = max_over_ranks((time.perf_counter() - t0) / steps, world)
    if not torch.equal(hc, ha + hb):
        raise SystemExit("bench: e2e add result differs from a + b")
    return {"value": round(BYTES_PER_ELEM * args.n / dt / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": 8 * args.n, "d2h_bytes_per_step": 4 * args.n}


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def compact_c3(r: dict) -> dict:
    if "error" in r:
        return r
    out = {"value": r["value"], "unit": "TFLOP/s", "ms_per_step": r["ms_per_step"], "steps": r["steps"],
           "roofline": {"bound": "fp32_fma", "achieved": r["value"], "peak": r["roofline"]["peak"],
                        "frac": r["roofline"]["frac"], "traffic": r["roofline"]["traffic"]},
           "clocks": {k: r["clocks"].get(k) for k in ("sm_mhz", "reasons")}, "cublas": r["cublas_fp32_tflops"],
           "gpu_launches": r["gpu_launches"], "rel_err": float(f"{r['config']['spot_check_rel_err']:.2e}")}
    t = r.get("tf32x3") or {}
    if "tflops" in t:
        out["tf32x3"] = {"value": t["tflops"], "rel_err": float(f"{t['rel_err_vs_f64']:.2e}")}
    if r.get("cpu_baseline"):
        out["cpu_tflops"] = r["cpu_baseline"]["value"]
    return out


def compact_c1(r: dict) -> dict:
    if "error" in r:
        return r
    return {"unit": "us", "higher_is_better": False, "numpy_sync_us": r["numpy_sync_us"],
            "device_async_us": r["device_async_us"], "device_us_per_launch": r["device_us_per_launch"],
            "graph_replay_us": r["graph_replay_us"], "gpu_launches": r["gpu_launches"],
            "cpu_us": r["cpu_baseline"]["value"]}


def run_eas(args) -> None:
    import torch

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    import eas  # noqa: F401
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
    add = run_add(args, world, rank, local, rt)
    configs: dict = {}
    if not args.quick and not args.no_gemm:
        torch.cuda.empty_cache()
        for name in ("C4", "C5"):
            try:
                configs[name] = run_gemm(name, args, world, rank, rt)
            except (SystemExit, Exception) as e:
                if world > 1:   # keep the ranks' collectives aligned: fail the whole run
                    raise
                configs[name] = {"error": f"{type(e).__name__}: {e}"[:200]}
            torch.cuda.empty_cache()
    if not args.quick and not args.no_gemm and world == 1:
        try:
            configs["C3"] = compact_c3(run_tiled(args, rt))
        except (SystemExit, Exception) as e:  # a secondary leg never suppresses the headline line
            configs["C3"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    if not args.quick and world == 1:
        try:
            configs["C1"] = compact_c1(run_c1(args, rt))
        except (SystemExit, Exception) as e:
            configs["C1"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    if rank != 0:
        return
    pk = peaks()
    line = {
        "metric": METRIC, "value": round(add["gbs"], 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(add["ms"], 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (torch.randn, seeded)",
        "config": {"workload": "C2 add_kernel N=2^28 f32 BLOCK=1024 via shard.run_shard", "N": args.n,
                   "BLOCK": BLOCK, "per_gpu_elements": add["n"], "parallelism": f"pid-range x{world}",
                   "l2": "3 GiB/step inputs > L2, no flush"},
        "e2e": add.get("e2e"),
        "roofline": {"bound": "hbm", "achieved": round(add["kernel_gbs"], 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(add["kernel_gbs"] / pk["hbm_gbs"], 4),
                     "traffic": profile_traffic("add_c2_n1") if world == 1 else None, "peak_source": pk["source"]},
        "gpu_launches": add["launches"], "host_us_per_launch": round(add["host_us"], 1),
        "clocks": add["clocks"],
    }
    if world == 1 and not args.no_cpu_baseline and not args.quick:
        line["cpu_baseline"] = cpu_add_baseline(args.cpu_seconds)
    if "gather" in add:
        line["gather"] = add["gather"]
    if configs:
        line["configs"] = configs
    print(json.dumps(line, separators=(",", ":")), flush=True)


def run_reference(args) -> None:
    """CPU semantics of the reference: the oracle interpreting the reference front end's IR of the
    same add kernel, on all host threads, over the whole C2 problem (N = 2**28) per step."""
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
    n_total = args.n
    # sampled (not the full N) only when the full problem at this step count would take many minutes
    budget_steps = args.steps + max(args.warmup, 1)
    while n_total > (1 << 22) and budget_steps * n_total * BYTES_PER_ELEM / 2.0e9 > 240:
        n_total //= 2
    chunk = 1 << 22
    nchunks = -(-n_total // chunk)
    rng = np.random.default_rng(1)
    a = rng.standard_normal(n_total, dtype=np.float32)
    b = rng.standard_normal(n_total, dtype=np.float32)
    c = np.zeros_like(a)

    def run_chunk(i):
        sl = slice(i * chunk, min((i + 1) * chunk, n_total))
        execute(ir, {"a": a[sl], "b": b[sl], "c": c[sl], "N": sl.stop - sl.start})

    def step():
        with ThreadPoolExecutor(cores) as ex:
            list(ex.map(run_chunk, range(nchunks)))

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    assert np.array_equal(c, a + b)
    gbs = BYTES_PER_ELEM * n_total / dt / 1e9
    full = n_total == args.n
    sample = (f"{'the full' if full else 'a sampled'} C2 add, {n_total} elements per step in 2^22-element chunks "
              f"(oracle interpreter, {cores} threads)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (numpy default_rng(1))",
        "config": {"workload": "C2 add_kernel N=2^28 f32 BLOCK=1024 via shard.run_shard", "N": args.n,
                   "BLOCK": BLOCK, "sampled_N": None if full else n_total},
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
    ap.add_argument("--no-gemm", action="store_true", help="skip the GEMM configs (C3, C4, C5)")
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
