"""ctypes binding of ``libeas_cuda.so`` (C ABI in ``include/eas_cuda.h``).

This module plays the part of the reference's ``eas/runtime/metal_ext.py``
(which imports the ObjC++ extension ``eas._metal`` and checks its method
table, ``metal_ext.py:22-33``): it loads the native library from the package's
``_lib`` directory, declares every entry point, and turns status codes into
the exception classes the reference raises (``RuntimeError`` for compile and
execution failures, ``ValueError`` for bad sizes, ``MemoryError`` for
allocation failures).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any

LIB_PATH = Path(__file__).resolve().parent.parent / "_lib" / "libeas_cuda.so"

EAS_OK = 0
EAS_ERR_UNAVAILABLE = 1
EAS_ERR_COMPILE = 2
EAS_ERR_LAUNCH = 3
EAS_ERR_VALUE = 4
EAS_ERR_MEMORY = 5
EAS_ERR_INJECTED = 6
EAS_ERR_TIMEOUT = 7

_vp = ctypes.c_void_p
_int = ctypes.c_int
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32
_PINT = ctypes.POINTER(ctypes.c_int)

#: every exported entry point: name -> (restype, argtypes)
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "eas_last_error": (ctypes.c_char_p, []),
    "eas_is_available": (_int, []),
    "eas_device_count": (_int, [_PINT]),
    "eas_set_device": (_int, [_int]),
    "eas_device_capability": (_int, [_int, _PINT, _PINT]),
    "eas_versions": (_int, [_PINT, _PINT]),
    "eas_compile": (_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), _int,
                           ctypes.POINTER(_vp), ctypes.POINTER(_sz)]),
    "eas_free_host": (None, [_vp]),
    "eas_pipeline_load": (_int, [_int, _vp, _sz, ctypes.c_char_p, _int, ctypes.POINTER(_vp)]),
    "eas_pipeline_free": (_int, [_vp]),
    "eas_pipeline_attrs": (_int, [_vp, _PINT, _PINT, _PINT]),
    "eas_launch": (_int, [_vp, ctypes.POINTER(_u32), ctypes.POINTER(_u32), _u32, _vp, _vp, ctypes.POINTER(_u32),
                          _u32]),
    "eas_launch_pdl": (_int, [_vp, ctypes.POINTER(_u32), ctypes.POINTER(_u32), _u32, _vp, _vp, ctypes.POINTER(_u32),
                          _u32]),
    "eas_alloc_buffer": (_int, [_int, _sz, ctypes.POINTER(_vp)]),
    "eas_free_buffer": (_int, [_vp]),
    "eas_copy_from_host": (_int, [_vp, _vp, _sz, _vp]),
    "eas_copy_to_host": (_int, [_vp, _vp, _sz, _vp]),
    "eas_copy_device": (_int, [_vp, _vp, _sz, _vp]),
    "eas_memset_d8": (_int, [_vp, _int, _sz, _vp]),
    "eas_copy_from_host_async": (_int, [_vp, _vp, _sz, _vp]),
    "eas_copy_to_host_async": (_int, [_vp, _vp, _sz, _vp]),
    "eas_host_is_pinned": (_int, [_vp, _PINT]),
    "eas_alloc_pinned": (_int, [_sz, ctypes.POINTER(ctypes.c_void_p)]),
    "eas_free_pinned": (_int, [_vp]),
    "eas_pinned_device_pointer": (_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "eas_stream_wait_event": (_int, [_vp, _vp]),
    "eas_stream_synchronize": (_int, [_vp]),
    "eas_device_synchronize": (_int, [_int]),
    "eas_stream_is_capturing": (_int, [_vp, _PINT]),
    "eas_stream_create": (_int, [_int, ctypes.POINTER(_vp)]),
    "eas_stream_destroy": (_int, [_vp]),
    "eas_event_create": (_int, [ctypes.POINTER(_vp)]),
    "eas_event_destroy": (_int, [_vp]),
    "eas_event_record": (_int, [_vp, _vp]),
    "eas_event_synchronize": (_int, [_vp]),
    "eas_event_query": (_int, [_vp, _PINT]),
    "eas_event_elapsed_ms": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_float)]),
    "eas_fault_inject": (_int, [ctypes.c_char_p, _int]),
    "eas_gemm_f16": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                            ctypes.c_uint64, ctypes.c_uint64, _int, ctypes.c_uint64, ctypes.c_uint64, _int, _vp]),
    "eas_gemm_status": (_int, [_int, _PINT]),
    "eas_gemm_f16_tile": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                                 ctypes.c_uint64, ctypes.c_uint64, _int, ctypes.c_uint64, ctypes.c_uint64, _int, _int,
                                 _int, _vp]),
    "eas_gemm_last_config": (_int, [_PINT, _PINT, _PINT, _PINT, _PINT, _PINT]),
    "eas_gemm_f16_plan": (_int, [_u32, _u32, _u32, _u32, _int, _int, _int, _int, _int, _int, _PINT, _PINT, _PINT,
                                 _PINT, _PINT, _PINT]),
    "eas_gemm_tf32": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                             ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _int, _vp]),
    "eas_gemm_3xtf32": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                               ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _int, _vp]),
    "eas_split_tf32": (_int, [_vp, _vp, _u32, _u32, ctypes.c_uint64, _u32, _u32, _u32, ctypes.c_uint64, _int, _vp]),
    "eas_wait_selftest": (_int, [ctypes.c_longlong, _vp]),
    "eas_cast_f32_f16_2d": (_int, [_vp, _vp, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64, _u32, _u32, _u32,
                                   ctypes.c_uint64, ctypes.c_uint64, _vp]),
    "eas_pad_f16_2d": (_int, [_vp, _vp, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64, _u32, _u32, _u32,
                                   ctypes.c_uint64, ctypes.c_uint64, _vp]),
    "eas_sgemm_f32_tiled": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                                   ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _int,
                                   _u32, _u32, _u32, _u32, _vp]),
    "eas_gemm_f16_noalloc": (_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, ctypes.c_uint64, ctypes.c_uint64,
                                    ctypes.c_uint64, ctypes.c_uint64, _int, ctypes.c_uint64, ctypes.c_uint64, _int,
                                    _vp, _PINT]),
}

_lib: ctypes.CDLL | None = None
_load_error: str | None = None


def load(*, require: bool = True) -> ctypes.CDLL | None:
    """Load the native library once; raise (``require=True``) or return None when it is missing."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("EAS_CUDA_LIB", str(LIB_PATH)))
    stale = None
    if path == LIB_PATH and path.exists():
        from .. import build as _build

        if _build.STAMP.exists() and _build.STAMP.read_text().strip() != _build.source_hash():
            stale = (f"native library {path} was built from other sources than the ones beside it; "
                     "rebuild with `python -m easy_as_b200.build`")
    if not path.exists():
        _load_error = (f"native library {path} is not built; run `python -m easy_as_b200.build` "
                       "(nvcc for sm_100a)")
    elif stale:
        _load_error = stale
    else:
        try:
            lib = ctypes.CDLL(str(path))
            missing = [n for n in SIGNATURES if not hasattr(lib, n)]
            if missing:
                raise RuntimeError("libeas_cuda.so is missing entry points: " + ", ".join(missing))
            for name, (res, argt) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = argt
            _lib = lib
            return lib
        except OSError as e:
            _load_error = f"cannot load {path}: {e}"
    if require:
        raise RuntimeError(_load_error)
    return None


def load_error() -> str | None:
    return _load_error


def last_error() -> str:
    lib = load()
    msg = lib.eas_last_error()
    return msg.decode(errors="replace") if msg else ""


class CudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def check(rc: int, what: str = "") -> None:
    if rc == EAS_OK:
        return
    msg = last_error()
    text = f"{what}: {msg}" if what else msg
    if rc == EAS_ERR_VALUE:
        raise ValueError(text)
    if rc == EAS_ERR_MEMORY:
        raise MemoryError(text)
    raise CudaError(rc, text)
