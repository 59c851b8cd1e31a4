"""GPU: the bounds-checked lowering (EAS_BOUNDS_CHECK=1) on the device.

(a) The reference's own kernels (IR from its front end), lowered with checks, give the same bits
    as their unchecked lowering on identical inputs (a check only skips accesses outside a
    buffer, and these kernels make none), and within the same tolerance as the unchecked parity
    tests for the simdgroup-MMA kernel.
(b) The out-of-bounds corpus (tests/oob_kernels.py) runs on buffers that are views into the middle
    of larger allocations, with 4096 guard elements on each side holding a sentinel.  The
    corpus's stray accesses are a few elements past a view, so every one of them would still land
    in memory this process owns; the checked kernel skips them, and each launch must raise the
    IndexError that names the buffer and the kind of access the oracle reports, and leave every
    guard element as it was.  No launch here touches memory outside its allocations."""

from __future__ import annotations

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from oob_kernels import OOB_CASES

pytestmark = pytest.mark.gpu
PAD = 4096
SENTINEL = 1234.5
CASES = [c for c in goldens.cases() if c["id"] not in ("t_many_dot",)]  # t_many_dot reads unwritten smem


@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_checked_reference_kernels_match_unchecked(cuda_rt, c, monkeypatch):
    ir = goldens.ir_from_json(c["opt"])
    monkeypatch.delenv("EAS_BOUNDS_CHECK", raising=False)
    plain = compile_ir(ir)
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "1")
    checked = compile_ir(ir)
    assert checked.plan.checked and not plain.plan.checked
    outs = []
    for ck in (plain, checked):
        inp = goldens.make_inputs(c, 11)
        cuda_rt.run(ck, inp, c["meta"], sync=True, **goldens.launch_opts(c))
        outs.append(inp)
    tol = 5e-3 if c["id"] == "matmul_simdgroup" else 0.0
    for name in c["writes"]:
        if tol:
            np.testing.assert_allclose(outs[1][name], outs[0][name], rtol=tol, atol=tol)
        else:
            np.testing.assert_array_equal(outs[1][name], outs[0][name], err_msg=f"{c['id']}:{name}")


def _guarded(x: np.ndarray):
    import torch

    dt = torch.float32 if x.dtype == np.float32 else torch.float16
    full = torch.full((x.size + 2 * PAD,), SENTINEL, dtype=dt, device="cuda")
    full[PAD:PAD + x.size] = torch.from_numpy(x).cuda()
    return full, full[PAD:PAD + x.size]


@pytest.mark.parametrize("case", OOB_CASES, ids=[c[0] for c in OOB_CASES])
def test_out_of_bounds_accesses_are_skipped_and_reported(cuda_rt, case, monkeypatch):
    import torch

    _cid, kernel, make, meta, grid, buf, kind = case
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "1")
    args = make()
    fulls, views = [], []
    for a in args:
        if isinstance(a, np.ndarray):
            full, view = _guarded(a)
            fulls.append(full)
            views.append(view)
        else:
            views.append(a)
    verb = "load from" if kind == "load" else "store to"
    where = f"{buf!r}" if buf else "threadgroup allocation"
    opts = {"_grid": grid} if grid else {}
    with pytest.raises(IndexError, match=f"out-of-bounds {verb} {where}"):
        kernel(*views, **meta, **opts)
    torch.cuda.synchronize()
    for full in fulls:
        guard = torch.cat([full[:PAD], full[-PAD:]]).float()
        assert torch.all(guard == SENTINEL), "a guard element changed: an access was not skipped"
