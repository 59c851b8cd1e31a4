"""CPU: the out-of-bounds corpus (tests/oob_kernels.py) against the oracle and the checked lowering.

The oracle raises on the first access outside a buffer; each case must trip it with the expected
buffer and access kind, and its checked lowering must guard that buffer and compile for sm_100a."""

from __future__ import annotations

import ctypes

import pytest

from easy_as_b200.codegen.cuda import ir_to_cuda
from easy_as_b200.runtime import cuda_ext
from oob_kernels import OOB_CASES
from oracle.interp import OracleError, execute


@pytest.mark.parametrize("case", OOB_CASES, ids=[c[0] for c in OOB_CASES])
def test_oracle_reports_the_expected_access(case):
    _cid, kernel, make, meta, grid, buf, kind = case
    args = make()
    ck = kernel.compile(*args, **meta)
    names = [a.name for a in ck.ir.args]
    verb = "load from" if kind == "load" else "store to"
    with pytest.raises(OracleError, match=f"out-of-bounds {verb}" + (f" {buf!r}" if buf else "")):
        execute(ck.ir, dict(zip(names, args)), grid=grid)


@pytest.mark.parametrize("case", OOB_CASES, ids=[c[0] for c in OOB_CASES])
def test_checked_lowering_guards_the_buffer_and_compiles(case):
    _cid, kernel, make, meta, _grid, buf, kind = case
    args = make()
    ck = kernel.compile(*args, **meta)
    lo = ir_to_cuda(ck.ir, checked=True)
    if buf is not None:
        slot = [a.name for a in ck.ir.args].index(buf)
        assert f"eas_lo_{buf}, eas_n_{buf}, eas_err, {2 * slot + (kind == 'store')}u)" in lo.src
    else:
        assert "0ull, 32ull, eas_err" in lo.src
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(lo.src.encode(), (lo.kernel_name + ".cu").encode(), None, 0, ctypes.byref(img),
                         ctypes.byref(size))
    assert rc == 0, cuda_ext.last_error()
    lib.eas_free_host(img)
