"""Load the reference-IR fixtures in tests/golden and rebuild them as IR objects."""

from __future__ import annotations

import gzip
import json
from functools import lru_cache
from pathlib import Path
from typing import Any

import numpy as np

from easy_as_b200.ir import Arg, DType, IRModule, Inst, ValueRef

GOLDEN = Path(__file__).resolve().parent / "golden"


def _arg(x: Any) -> Any:
    if isinstance(x, dict) and "v" in x:
        i, dt, lanes = x["v"]
        return ValueRef(int(i), DType(dt), int(lanes))
    if isinstance(x, dict) and "dt" in x:
        return DType(x["dt"])
    return x


def ir_from_json(d: dict) -> IRModule:
    args = tuple(Arg(n, DType(dt), kind) for n, dt, kind in d["args"])
    insts = []
    for op, out, a in d["insts"]:
        o = None if out is None else ValueRef(int(out[0]), DType(out[1]), int(out[2]))
        insts.append(Inst(op, o, tuple(_arg(x) for x in a)))
    return IRModule(d["name"], args, tuple(insts))


def ir_to_json(ir: IRModule) -> dict:
    def ser(a: Any) -> Any:
        if isinstance(a, ValueRef):
            return {"v": [a.id, a.dtype.value, a.lanes]}
        if isinstance(a, DType):
            return {"dt": a.value}
        return a

    return {"name": ir.name, "args": [[a.name, a.dtype.value, a.kind] for a in ir.args],
            "insts": [[i.op, None if i.out is None else [i.out.id, i.out.dtype.value, i.out.lanes],
                       [ser(x) for x in i.args]] for i in ir.insts]}


@lru_cache(maxsize=None)
def cases() -> tuple[dict, ...]:
    return tuple(json.loads((GOLDEN / "reference_ir.json").read_text())["cases"])


@lru_cache(maxsize=None)
def big_cases() -> tuple[dict, ...]:
    with gzip.open(GOLDEN / "reference_ir_big.json.gz", "rt") as f:
        return tuple(json.load(f)["cases"])


def case(cid: str) -> dict:
    for c in cases() + big_cases():
        if c["id"] == cid:
            return c
    raise KeyError(cid)


def make_inputs(c: dict, seed: int = 0) -> dict[str, Any]:
    """Seeded runtime arguments for a fixture case (buffers ~ N(0,1), outputs zeroed)."""
    rng = np.random.default_rng(seed)
    out: dict[str, Any] = {}
    for name, spec in zip(c["arg_names"], c["args"]):
        if isinstance(spec, dict):
            dt = np.float32 if spec["buffer"] == "f32" else np.float16
            if name in c["writes"]:
                out[name] = np.zeros(spec["n"], dtype=dt)
            else:
                out[name] = rng.standard_normal(spec["n"]).astype(dt)
        else:
            out[name] = spec
    return out


def launch_opts(c: dict) -> dict[str, Any]:
    lo = c["launch"]
    return {"grid": tuple(lo["grid"]) if "grid" in lo else None, "nthreads": lo.get("nthreads"),
            "shape": tuple(lo["shape"]) if "shape" in lo else None}
