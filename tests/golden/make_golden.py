"""Generate tests/golden/reference_ir.json(.gz) from the reference front end.

Run where a reference checkout is readable, its location in $EAS_REFERENCE:

    EAS_REFERENCE=<path to the easy_as checkout> python tests/golden/make_golden.py

For every case below this script imports the reference package ``eas`` and
the reference module that defines the kernel (examples/*.py, tests/*.py),
then records, using the reference's own code only:

* ``raw``: the IR returned by the reference tracer ``eas.compiler.trace_to_ir``;
* ``opt``: the IR after the reference pass pipeline ``eas.compiler._optimize_ir``;
* ``block_size``, ``launch_mode``, ``writes`` from ``Kernel.compile``;
* the launch configuration (buffer sizes/dtypes, scalar values, grid options)
  the parity tests use to execute the IR.

Nothing from the reference's source text is stored: only the IR data its
front end produces.  The tests replay that IR through this repository's
passes, CUDA emitter and runtime (GPU) and through the CPU oracle.
"""

from __future__ import annotations

import gzip
import importlib.util
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("EAS_REFERENCE"):
    raise SystemExit("make_golden.py: set EAS_REFERENCE to a checkout of the reference (easy_as)")
REF = Path(os.environ["EAS_REFERENCE"])


def B(dtype: str, n: int) -> dict:
    return {"buffer": dtype, "n": int(n)}


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


# id, reference file, kernel attribute, positional runtime args, meta, launch options
CASES: list[tuple[str, str, str, list, dict, dict]] = [
    # examples/add.py — configs C1 (N=1031, BLOCK=256) and the C2 block size
    ("add_c1", "examples/add.py", "add_kernel", [B("f32", 1031), B("f32", 1031), B("f32", 1031), 1031],
     {"BLOCK": 256}, {}),
    ("add_block1024", "examples/add.py", "add_kernel", [B("f32", 5000), B("f32", 5000), B("f32", 5000), 5000],
     {"BLOCK": 1024}, {}),
    # examples/matmul.py — naive thread-mode matmul, constexpr K unrolled
    ("matmul_naive", "examples/matmul.py", "matmul_kernel",
     [B("f32", 40 * 16), B("f32", 16 * 70), B("f32", 40 * 70), 40, 70], {"BLOCK": 32, "K": 16}, {}),
    # examples/matmul_tiled.py — masked and interior kernels
    ("matmul_tiled_masked", "examples/matmul_tiled.py", "matmul_tiled_kernel",
     [B("f32", 50 * 64), B("f32", 64 * 70), B("f32", 50 * 70), 50, 70, 0, 0],
     {"BM": 16, "BN": 64, "BK": 16, "K": 64, "NT": 256}, {"grid": [cdiv(70, 64), cdiv(50, 16), 1]}),
    ("matmul_tiled_full", "examples/matmul_tiled.py", "matmul_tiled_full_kernel",
     [B("f32", 64 * 64), B("f32", 64 * 128), B("f32", 64 * 128), 64, 128],
     {"BM": 32, "BN": 32, "BK": 32, "K": 64, "NT": 256}, {"grid": [4, 2, 1]}),
    # examples/matmul_simdgroup.py — simdgroup 8x8 MMA through threadgroup f16 tiles
    ("matmul_simdgroup", "examples/matmul_simdgroup.py", "matmul_simdgroup_mma_kernel",
     [B("f32", 40 * 32), B("f32", 32 * 36), B("f32", 40 * 36), 40, 36],
     {"BM": 16, "BN": 16, "BK": 16, "K": 32, "NT": 128}, {"grid": [cdiv(36, 16), cdiv(40, 16), 1]}),
    # reference unit-test kernels
    ("t_add", "tests/test_add.py", "add_kernel", [B("f32", 4099), B("f32", 4099), B("f32", 4099), 4099],
     {"BLOCK": 256}, {}),
    ("t_fma_simple", "tests/test_fma.py", "simple_fma_kernel",
     [B("f32", 300), B("f32", 300), B("f32", 300), B("f32", 300), 300], {"BLOCK": 256}, {}),
    ("t_fma_matmul", "tests/test_fma.py", "matmul_with_fma",
     [B("f32", 32 * 8), B("f32", 8 * 64), B("f32", 32 * 64), 32, 64], {"BLOCK": 32, "K": 8},
     {"grid": [32, 2, 1]}),
    ("t_local_id", "tests/test_local_and_lane_id.py", "local_id_kernel", [B("f32", 384), 384], {"BLOCK": 128}, {}),
    ("t_lane_id", "tests/test_local_and_lane_id.py", "lane_id_kernel", [B("f32", 256), 256], {"BLOCK": 256}, {}),
    ("t_tg_copy", "tests/test_threadgroup_memory.py", "tg_copy_kernel",
     [B("f32", 4103), B("f32", 4103), 4103], {"BLOCK": 256}, {}),
    ("t_tg_copy_masked", "tests/test_threadgroup_memory.py", "tg_copy_kernel_masked",
     [B("f32", 515), B("f32", 515), 515], {"BLOCK": 256}, {}),
    ("t_tptg", "tests/test_tptg_override.py", "tptg_independent_kernel", [B("f32", 1031), 1031], {"BLOCK": 256}, {}),
    ("t_callable_grid", "tests/test_callable_grid.py", "grid_callable_kernel", [B("f32", 50), 5, 10], {"BLOCK": 4},
     {"grid": [3, 5, 1]}),
    ("t_gemv_dot", "tests/test_dot_dynamic_k.py", "gemv_dot_kernel",
     [B("f32", 33 * 31), B("f32", 31), B("f32", 33), 33, 31, 33], {"BLOCK": 64}, {"nthreads": 33}),
    ("t_matmul", "tests/test_matmul.py", "matmul_kernel",
     [B("f32", 32 * 16), B("f32", 16 * 100), B("f32", 32 * 100), 32, 100], {"BLOCK": 64, "K": 16},
     {"grid": [32, 2, 1]}),
    ("t_matmul_tiled", "tests/test_matmul_tiled.py", "matmul_tiled_kernel_test",
     [B("f32", 17 * 31), B("f32", 31 * 130), B("f32", 17 * 130), 17, 130],
     {"BM": 16, "BN": 64, "BK": 16, "K": 31, "NT": 256}, {"grid": [cdiv(130, 64), cdiv(17, 16), 1]}),
    # the other two shapes of the reference test's device check (tests/test_matmul_tiled.py:128-178)
    ("t_matmul_tiled_33x65x48", "tests/test_matmul_tiled.py", "matmul_tiled_kernel_test",
     [B("f32", 33 * 48), B("f32", 48 * 65), B("f32", 33 * 65), 33, 65],
     {"BM": 16, "BN": 64, "BK": 16, "K": 48, "NT": 256}, {"grid": [cdiv(65, 64), cdiv(33, 16), 1]}),
    ("t_matmul_tiled_64x64x32", "tests/test_matmul_tiled.py", "matmul_tiled_kernel_test",
     [B("f32", 64 * 32), B("f32", 32 * 64), B("f32", 64 * 64), 64, 64],
     {"BM": 16, "BN": 64, "BK": 16, "K": 32, "NT": 256}, {"grid": [cdiv(64, 64), cdiv(64, 16), 1]}),
    ("t_grid_hw", "tests/test_grid_infer.py", "add2d_hw_kernel",
     [B("f32", 17 * 103), B("f32", 17 * 103), B("f32", 17 * 103), 17, 103], {"BLOCK": 32}, {}),
    ("t_bool_simplify", "tests/test_bool_simplify.py", "bool_simplify_kernel", [B("f32", 256), 128], {"BLOCK": 256},
     {"nthreads": 256}),
    ("t_bool_chain", "tests/test_bool_simplify.py", "bool_chain_mask_kernel", [B("f32", 256), 128],
     {"BLOCK": 256}, {"nthreads": 256}),
    ("t_in_tile_fold", "tests/test_interval_lt_fold.py", "_in_tile_store_kernel", [B("f32", 64), B("f32", 64)],
     {"LIMIT": 64, "NT": 16}, {"nthreads": 16}),
    ("t_in_tile_keep", "tests/test_interval_lt_fold.py", "_in_tile_store_kernel", [B("f32", 80), B("f32", 80)],
     {"LIMIT": 70, "NT": 16}, {"nthreads": 16}),
    ("t_many_dot", "tests/test_dot_codegen_unique_vars.py", "many_dot_kernel", [B("f32", 1)], {"K": 16, "BLOCK": 32},
     {"nthreads": 32}),
    ("t_axpy", "tests/test_kernel_cache.py", "axpy_kernel", [B("f32", 1027), B("f32", 1027), B("f32", 1027), 1027, 2.0],
     {"BLOCK": 256}, {}),
]

# bench-scale IR of the unmodified tiled kernel (config C3: 2048^3, 32x32x32 tiles, NT=256)
BIG_CASES = [
    ("matmul_tiled_c3_full", "examples/matmul_tiled.py", "matmul_tiled_full_kernel",
     [B("f32", 1), B("f32", 1), B("f32", 1), 2048, 2048],
     {"BM": 32, "BN": 32, "BK": 32, "K": 2048, "NT": 256}, {"grid": [64, 64, 1]}),
    # the simdgroup-MMA example's own default run (examples/matmul_simdgroup.py:138-160): 512^3,
    # BM=16 BN=32 BK=8, NT=(BM/8)(BN/8)*32
    ("matmul_simdgroup_512", "examples/matmul_simdgroup.py", "matmul_simdgroup_mma_kernel",
     [B("f32", 512 * 512), B("f32", 512 * 512), B("f32", 512 * 512), 512, 512],
     {"BM": 16, "BN": 32, "BK": 8, "K": 512, "NT": 256}, {"grid": [512 // 32, 512 // 16, 1]}),
]


def _load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    spec.loader.exec_module(mod)
    return mod


def _ser_arg(a):
    from eas.ir import DType, ValueRef  # reference package

    if isinstance(a, ValueRef):
        return {"v": [a.id, a.dtype.value, a.lanes]}
    if isinstance(a, DType):
        return {"dt": a.value}
    if isinstance(a, bool) or a is None or isinstance(a, (int, float, str)):
        return a
    raise TypeError(type(a))


def ser_ir(ir) -> dict:
    return {
        "name": ir.name,
        "args": [[a.name, a.dtype.value, a.kind] for a in ir.args],
        "insts": [[i.op, None if i.out is None else [i.out.id, i.out.dtype.value, i.out.lanes],
                   [_ser_arg(x) for x in i.args]] for i in ir.insts],
    }


def _runtime_values(spec: list, np):
    out = []
    for a in spec:
        if isinstance(a, dict):
            out.append(np.zeros(a["n"], dtype=np.float32 if a["buffer"] == "f32" else np.float16))
        else:
            out.append(a)
    return out


def build(cases) -> list[dict]:
    sys.path.insert(0, str(REF))
    import numpy as np

    import eas  # the reference package
    from eas.compiler import _optimize_ir, trace_to_ir

    records = []
    modules: dict[str, object] = {}
    for cid, rel, attr, args, meta, launch in cases:
        if rel not in modules:
            modules[rel] = _load_module(REF / rel, "ref_" + rel.replace("/", "_").replace(".py", ""))
        kern = getattr(modules[rel], attr)
        values = _runtime_values(args, np)
        meta_b, rt_args = kern._bind_and_split(*values, **meta)
        raw = trace_to_ir(kern.fn, rt_args, meta_b)
        opt = _optimize_ir(raw)
        ck = kern.compile(*values, **meta)
        assert ser_ir(ck.ir) == ser_ir(opt)
        records.append({
            "id": cid, "source": f"{rel}:{attr}", "meta": meta, "args": args,
            "arg_names": list(rt_args.keys()), "launch": launch,
            "block_size": ck.block_size, "launch_mode": ck.launch_mode, "writes": sorted(ck.writes),
            "raw": ser_ir(raw), "opt": ser_ir(opt),
        })
    _ = eas
    return records


def main() -> None:
    small = build(CASES)
    (HERE / "reference_ir.json").write_text(json.dumps({"generator": "tests/golden/make_golden.py",
                                                         "cases": small}, indent=None, separators=(",", ":")))
    big = build(BIG_CASES)
    with gzip.open(HERE / "reference_ir_big.json.gz", "wt") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": big}, f, separators=(",", ":"))
    print(f"wrote {len(small)} small and {len(big)} large cases")


if __name__ == "__main__":
    main()
