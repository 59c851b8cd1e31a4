"""The front end reproduces the reference front end's IR exactly.

Golden IR comes from the reference's own tracer and passes
(tests/golden/make_golden.py).  Two checks per case:

* this repository's pass pipeline applied to the reference's *traced* IR
  gives the reference's *optimised* IR (pins the passes,
  reference eas/compiler.py:648-1272);
* where the reference checkout is present, the unmodified reference kernel
  function traced by this repository's front end gives the same raw and
  optimised IR (pins the tracer, reference eas/compiler.py:132-617).
"""

from __future__ import annotations

import importlib.util

import numpy as np
import pytest

import goldens
from conftest import REFERENCE
from easy_as_b200.analysis import infer_writes
from easy_as_b200.codegen.cuda import infer_block_and_mode
from easy_as_b200.compiler import optimize_ir, trace_to_ir
from easy_as_b200.ir import validate_ir

CASES = goldens.cases()


@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_passes_reproduce_reference(c):
    raw = goldens.ir_from_json(c["raw"])
    validate_ir(raw)
    opt = optimize_ir(raw)
    assert goldens.ir_to_json(opt) == c["opt"]
    validate_ir(opt)
    assert infer_block_and_mode(opt) == (c["block_size"], c["launch_mode"])
    assert sorted(infer_writes(opt)) == c["writes"]


@pytest.mark.parametrize("c", goldens.big_cases(), ids=[c["id"] for c in goldens.big_cases()])
def test_big_case_passes(c):
    opt = optimize_ir(goldens.ir_from_json(c["raw"]))
    assert goldens.ir_to_json(opt) == c["opt"]


def _ref_kernel(c):
    rel, attr = c["source"].split(":")
    path = REFERENCE / rel
    spec = importlib.util.spec_from_file_location("refk_" + c["id"], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # its `import eas` resolves to easy_as_b200
    return getattr(mod, attr)


@pytest.mark.skipif(REFERENCE is None or not REFERENCE.exists(), reason="EAS_REFERENCE not set to a reference checkout")
@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_tracer_reproduces_reference(c):
    kern = _ref_kernel(c)
    vals = []
    for spec in c["args"]:
        if isinstance(spec, dict):
            vals.append(np.zeros(spec["n"], np.float32 if spec["buffer"] == "f32" else np.float16))
        else:
            vals.append(spec)
    meta, rt = kern._bind_and_split(*vals, **c["meta"])
    raw = trace_to_ir(kern.fn, rt, meta)
    assert goldens.ir_to_json(raw) == c["raw"]
    ck = kern.compile(*vals, **c["meta"])
    assert goldens.ir_to_json(ck.ir) == c["opt"]
    assert (ck.block_size, ck.launch_mode) == (c["block_size"], c["launch_mode"])
