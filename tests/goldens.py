"""Load the reference-IR fixtures in tests/golden and rebuild them as IR objects."""

from __future__ import annotations

import gzip
import json
from functools import lru_cache
from pathlib import Path
from typing import Any

import numpy as np

from easy_as_b200.ir import ir_from_json, ir_to_json  # noqa: F401  (re-exported for the tests)

GOLDEN = Path(__file__).resolve().parent / "golden"


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
