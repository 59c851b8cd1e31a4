"""libeas_cuda.so: loads without a GPU, exports every entry point of include/eas_cuda.h,
compiles generated CUDA with NVRTC for sm_100a, and honours host-side fault injection."""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

import pytest

import goldens
from easy_as_b200.codegen.cuda import ir_to_cuda
from easy_as_b200.runtime import cuda_ext

HEADER = Path(__file__).resolve().parent.parent / "include" / "eas_cuda.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|const char\*)\s+(eas_[a-z0-9_]+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "eas_compile" in names and "eas_launch" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    lib = cuda_ext.load()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared()) <= set(cuda_ext.SIGNATURES)


def test_unavailable_is_reported_not_raised():
    lib = cuda_ext.load()
    avail = lib.eas_is_available()
    assert avail in (0, 1)
    if not avail:
        assert cuda_ext.last_error()


def _compile(src: str, name: str) -> int:
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(src.encode(), (name + ".cu").encode(), None, 0, ctypes.byref(img), ctypes.byref(size))
    if rc == 0:
        lib.eas_free_host(img)
    return rc


def test_nvrtc_compiles_generated_add():
    lo = ir_to_cuda(goldens.ir_from_json(goldens.case("add_c1")["opt"]))
    assert _compile(lo.src, lo.kernel_name) == 0


def test_compile_error_carries_nvrtc_log():
    rc = _compile('extern "C" __global__ void k() { this is not cuda; }', "bad")
    assert rc == cuda_ext.EAS_ERR_COMPILE
    assert "CUDA compile failed" in cuda_ext.last_error()


def test_fault_injection_on_compile():
    lib = cuda_ext.load()
    lo = ir_to_cuda(goldens.ir_from_json(goldens.case("t_tptg")["opt"]))
    assert lib.eas_fault_inject(b"compile", 2) == 0
    assert _compile(lo.src, lo.kernel_name) == 0
    assert _compile(lo.src, lo.kernel_name) == cuda_ext.EAS_ERR_INJECTED
    assert "injected" in cuda_ext.last_error()
    assert _compile(lo.src, lo.kernel_name) == 0
    assert lib.eas_fault_inject(b"bogus", 1) == cuda_ext.EAS_ERR_VALUE


def test_check_maps_status_to_exception_types():
    with pytest.raises(ValueError):
        cuda_ext.check(cuda_ext.EAS_ERR_VALUE)
    with pytest.raises(MemoryError):
        cuda_ext.check(cuda_ext.EAS_ERR_MEMORY)
    with pytest.raises(RuntimeError):
        cuda_ext.check(cuda_ext.EAS_ERR_LAUNCH)



def test_build_is_keyed_on_a_source_hash():
    """The library's stamp records the sha256 of the sources and nvcc flags it was built from; a
    changed source (not a newer file time) is what makes ``needs_build`` true."""
    from easy_as_b200 import build

    assert build.STAMP.exists(), "build() writes the stamp beside the library"
    assert build.STAMP.read_text().strip() == build.source_hash()
    assert not build.needs_build()
    os.utime(build.sources()[0])          # touching a file changes nothing
    assert not build.needs_build()
