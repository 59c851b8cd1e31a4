"""DLPack exchange: ``from_dlpack`` / ``to_dlpack`` and the CUDA capsule codec.

Public behaviour follows easy_as ``eas/dlpack.py:16-82``: CPU tensors go
through numpy's own DLPack support; device tensors are exchanged zero-copy.
On this backend the device type is ``kDLCUDA`` (2) instead of ``kDLMetal``
(8).  The capsule codec below reads and writes the DLPack v0.x
``DLManagedTensor`` layout with ctypes, so no compiled Python extension is
involved; the reference did this in ObjC++ (``_metal.mm:530-639,710-822``).
"""

from __future__ import annotations

import ctypes
import threading
from typing import Any

import numpy as np

KDL_CPU = 1
KDL_CUDA = 2
KDL_FLOAT = 2


class DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class DLTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("device", DLDevice), ("ndim", ctypes.c_int32),
                ("dtype", DLDataType), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("strides", ctypes.POINTER(ctypes.c_int64)), ("byte_offset", ctypes.c_uint64)]


class DLManagedTensor(ctypes.Structure):
    pass


_DELETER = ctypes.CFUNCTYPE(None, ctypes.POINTER(DLManagedTensor))
DLManagedTensor._fields_ = [("dl_tensor", DLTensor), ("manager_ctx", ctypes.c_void_p), ("deleter", _DELETER)]

_api = ctypes.pythonapi
_api.PyCapsule_New.restype = ctypes.py_object
_api.PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
_api.PyCapsule_IsValid.restype = ctypes.c_int
_api.PyCapsule_IsValid.argtypes = [ctypes.py_object, ctypes.c_char_p]
_api.PyCapsule_GetPointer.restype = ctypes.c_void_p
_api.PyCapsule_GetPointer.argtypes = [ctypes.py_object, ctypes.c_char_p]
_api.PyCapsule_SetName.restype = ctypes.c_int
_api.PyCapsule_SetName.argtypes = [ctypes.py_object, ctypes.c_char_p]

_NAME = b"dltensor"
_USED = b"used_dltensor"
_name_buf = ctypes.create_string_buffer(_NAME)
_used_buf = ctypes.create_string_buffer(_USED)

# exported tensors alive in some consumer: id(managed struct) -> (struct, shape array, owner)
_live: dict[int, tuple[Any, Any, Any]] = {}
_live_lock = threading.Lock()


@_DELETER
def _managed_deleter(mt: Any) -> None:
    addr = ctypes.addressof(mt.contents)
    with _live_lock:
        _live.pop(addr, None)


_CAPSULE_DESTRUCTOR = ctypes.CFUNCTYPE(None, ctypes.c_void_p)
# raw-pointer views of the capsule API: a capsule being destroyed must not be
# turned back into a Python reference
_capsule_is_valid_raw = ctypes.PYFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p)(
    ("PyCapsule_IsValid", ctypes.pythonapi))
_capsule_pointer_raw = ctypes.PYFUNCTYPE(ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p)(
    ("PyCapsule_GetPointer", ctypes.pythonapi))


@_CAPSULE_DESTRUCTOR
def _capsule_destructor(cap_ptr: int) -> None:
    if _capsule_is_valid_raw(cap_ptr, _NAME):  # never consumed: we still own it
        p = _capsule_pointer_raw(cap_ptr, _NAME)
        mt = ctypes.cast(p, ctypes.POINTER(DLManagedTensor))
        mt.contents.deleter(mt)


def export_capsule(ptr: int, shape: tuple[int, ...], itemsize: int, device_type: int, device_id: int,
                   owner: Any) -> Any:
    """A ``dltensor`` capsule viewing ``ptr`` (float16/float32, C-contiguous); keeps ``owner`` alive."""
    mt = DLManagedTensor()
    shp = (ctypes.c_int64 * max(len(shape), 1))(*shape)
    mt.dl_tensor.data = ptr
    mt.dl_tensor.device = DLDevice(device_type, device_id)
    mt.dl_tensor.ndim = len(shape)
    mt.dl_tensor.dtype = DLDataType(KDL_FLOAT, itemsize * 8, 1)
    mt.dl_tensor.shape = ctypes.cast(shp, ctypes.POINTER(ctypes.c_int64))
    mt.dl_tensor.strides = None
    mt.dl_tensor.byte_offset = 0
    mt.manager_ctx = None
    mt.deleter = _managed_deleter
    addr = ctypes.addressof(mt)
    with _live_lock:
        _live[addr] = (mt, shp, owner)
    return _api.PyCapsule_New(addr, _name_buf, ctypes.cast(_capsule_destructor, ctypes.c_void_p))


class ImportedDLPack:
    """Keeps a consumed ``DLManagedTensor`` alive; calls its deleter when freed."""

    def __init__(self, capsule: Any):
        if not _api.PyCapsule_IsValid(capsule, _NAME):
            raise TypeError("expected an unconsumed 'dltensor' capsule")
        p = _api.PyCapsule_GetPointer(capsule, _NAME)
        self._mt = ctypes.cast(p, ctypes.POINTER(DLManagedTensor))
        _api.PyCapsule_SetName(capsule, _used_buf)
        t = self._mt.contents.dl_tensor
        self.device_type = int(t.device.device_type)
        self.device_id = int(t.device.device_id)
        if t.dtype.code != KDL_FLOAT or t.dtype.bits not in (16, 32) or t.dtype.lanes != 1:
            self.close()
            raise TypeError(f"unsupported dlpack dtype (code={t.dtype.code}, bits={t.dtype.bits})")
        self.bits = int(t.dtype.bits)
        self.shape = tuple(int(t.shape[i]) for i in range(t.ndim))
        if t.strides:
            expect = 1
            for i in range(t.ndim - 1, -1, -1):
                if self.shape[i] != 1 and int(t.strides[i]) != expect:
                    self.close()
                    raise ValueError("only C-contiguous DLPack tensors are supported")
                expect *= self.shape[i]
        self.ptr = int(t.data or 0) + int(t.byte_offset)

    def close(self) -> None:
        mt, self._mt = self._mt, None
        if mt is not None and mt.contents.deleter:
            mt.contents.deleter(mt)

    def __del__(self) -> None:  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _as_capsule(x: Any) -> Any:
    if type(x).__name__ == "PyCapsule":
        return x
    fn = getattr(x, "__dlpack__", None)
    if not callable(fn):
        raise TypeError("object does not implement the DLPack protocol (__dlpack__)")
    return fn()


def from_dlpack(x: Any, *, device: str | None = None) -> Any:
    """Wrap a DLPack producer as an ``eas.Tensor``.

    ``device="cuda"`` imports a ``kDLCUDA`` tensor zero-copy (a torch CUDA
    tensor, or any capsule/producer); otherwise numpy's importer is used.
    """
    from .tensor import Tensor, _normalize_device, tensor as _tensor

    dev = _normalize_device(device)
    if dev == "cuda":
        try:
            import torch  # type: ignore

            if isinstance(x, torch.Tensor):
                return _tensor(x, device="cuda")
        except ImportError:  # pragma: no cover
            pass
        imp = ImportedDLPack(_as_capsule(x))
        if imp.device_type != KDL_CUDA:
            imp.close()
            raise TypeError(f"expected a kDLCUDA tensor, got device type {imp.device_type}")
        dtype = np.float16 if imp.bits == 16 else np.float32
        return Tensor._from_cuda_ptr(imp.ptr, imp.shape, dtype, imp.device_id, owner=imp)
    try:
        arr = np.from_dlpack(x)
    except Exception as e:
        raise TypeError("object does not support DLPack import via numpy.from_dlpack") from e
    if arr.dtype not in (np.float16, np.float32):
        raise TypeError("only float16/float32 tensors are supported")
    return _tensor(np.ascontiguousarray(arr), device=dev)


def to_dlpack(x: Any) -> Any:
    """Export an ``eas.Tensor`` as a raw ``PyCapsule`` (torch-style)."""
    from .tensor import Tensor

    if not isinstance(x, Tensor):
        raise TypeError(f"to_dlpack expects eas.Tensor, got {type(x)!r}")
    return x.__dlpack__()
