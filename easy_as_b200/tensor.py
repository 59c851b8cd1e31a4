"""``eas.Tensor``: a float16/float32 buffer on the host or on a CUDA device.

Same public surface as easy_as ``eas/tensor.py`` (``Tensor``, ``tensor``,
``empty``, ``empty_like``; properties ``device/dtype/shape/nbytes``;
``numpy()``, ``to()``, ``to_torch()``, ``__dlpack__``, ``__dlpack_device__``)
with the device ``"cuda"`` in place of ``"mps"``:

* CPU storage is a numpy array (kept zero-copy when wrapping numpy or a torch
  CPU tensor, as ``tensor.py:296-328`` does);
* CUDA storage is a device pointer owned by a ``DeviceBuffer`` or borrowed from
  its producer (a torch CUDA tensor, or an imported DLPack capsule) whose
  lifetime the tensor extends;
* ``__dlpack_device__`` answers ``(2, device_index)`` (``kDLCUDA``), and
  ``__dlpack__`` exports the device pointer zero-copy, ordering the
  consumer's stream after queued launches on the device (the reference
  synchronised its whole queue on the host, ``_metal.mm:788-793``).

``"cuda:N"`` selects device ``N``; ``"mps"``/``"metal"`` are rejected.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

from .dlpack import KDL_CPU, KDL_CUDA, export_capsule


def _torch() -> Any:
    try:
        import torch  # type: ignore

        return torch
    except Exception:
        return None


def _parse_device(device: Any) -> tuple[str, int]:
    if device is None:
        return "cpu", 0
    s = str(device).lower()
    if s == "cpu":
        return "cpu", 0
    if s == "cuda":
        return "cuda", _default_cuda_device()
    if s.startswith("cuda:") and s[5:].isdigit():
        return "cuda", int(s[5:])
    raise ValueError(f"unsupported device: {device!r} (expected 'cpu'|'cuda'|'cuda:N')")


def _normalize_device(device: Any) -> str:
    return _parse_device(device)[0]


def _default_cuda_device() -> int:
    from .runtime.cuda import CudaRuntime

    return CudaRuntime().default_device()


def _require_supported_dtype(dtype: Any) -> np.dtype:
    d = np.dtype(dtype)
    if d not in (np.float16, np.float32):
        raise TypeError(f"only float16/float32 tensors are supported (got {d})")
    return d


def _numel(shape: tuple[int, ...]) -> int:
    n = 1
    for d in shape:
        if d < 0:
            raise ValueError("negative dimensions are not allowed")
        n *= int(d)
    return n


@dataclass(frozen=True, slots=True)
class _CudaStorage:
    ptr: int
    nbytes: int
    device: int
    owner: Any  # DeviceBuffer, torch tensor or ImportedDLPack keeping ptr alive


def _runtime() -> Any:
    from .runtime import _cuda_runtime

    return _cuda_runtime()


class Tensor:
    __eas_tensor__ = True

    def __init__(self, *, shape: tuple[int, ...], dtype: Any, device: str, cpu: np.ndarray | None = None,
                 cuda: _CudaStorage | None = None) -> None:
        self._shape = tuple(int(d) for d in shape)
        self._dtype = _require_supported_dtype(dtype)
        self._device = device
        self._cpu = cpu
        self._cuda = cuda
        if device == "cpu":
            if cpu is None or cuda is not None:
                raise ValueError("cpu tensor requires cpu storage only")
        elif device == "cuda":
            if cuda is None or cpu is not None:
                raise ValueError("cuda tensor requires cuda storage only")
        else:
            raise ValueError(f"unsupported device: {device!r}")

    # -- construction helpers ------------------------------------------------
    @classmethod
    def _from_cuda_ptr(cls, ptr: int, shape: tuple[int, ...], dtype: Any, device: int, owner: Any) -> "Tensor":
        d = _require_supported_dtype(dtype)
        nbytes = _numel(tuple(shape)) * d.itemsize
        return cls(shape=tuple(shape), dtype=d, device="cuda", cuda=_CudaStorage(int(ptr), nbytes, int(device), owner))

    # -- properties ------------------------------------------------------------
    @property
    def device(self) -> str:
        return self._device

    @property
    def dtype(self) -> np.dtype:
        return self._dtype

    @property
    def shape(self) -> tuple[int, ...]:
        return self._shape

    @property
    def nbytes(self) -> int:
        return _numel(self._shape) * self._dtype.itemsize

    def __repr__(self) -> str:  # pragma: no cover
        dev = self._device if self._device == "cpu" else f"cuda:{self._cuda.device}"
        return f"eas.Tensor(shape={self._shape}, dtype={self._dtype.name}, device={dev!r})"

    def _cuda_ptr(self) -> int:
        if self._cuda is None:
            raise TypeError("expected a cuda tensor")
        return self._cuda.ptr

    def _cuda_device(self) -> int:
        if self._cuda is None:
            raise TypeError("expected a cuda tensor")
        return self._cuda.device

    # -- host views --------------------------------------------------------------
    def __array__(self, dtype: Any | None = None, copy: Any | None = None) -> np.ndarray:
        if self._device != "cpu":
            raise TypeError("cannot convert a cuda tensor to numpy without .numpy()")
        arr = self._cpu
        return arr if dtype is None else arr.astype(dtype, copy=False)

    def numpy(self) -> np.ndarray:
        if self._device == "cpu":
            return self._cpu  # type: ignore[return-value]
        out = np.empty(self._shape, dtype=self._dtype)
        from .runtime import cuda_ext

        rt = _runtime()
        rt.synchronize()
        lib = cuda_ext.load()
        cuda_ext.check(lib.eas_set_device(self._cuda.device), "set_device")
        cuda_ext.check(lib.eas_copy_to_host(out.ctypes.data, self._cuda.ptr, out.nbytes, 0), "copy_to_host")
        return out

    # -- DLPack ----------------------------------------------------------------------
    def __dlpack__(self, stream: Any | None = None, **_kw: Any) -> Any:
        """Export for a DLPack consumer.

        CUDA tensors: with ``stream=None`` all queued launches are waited for on
        the host.  With a consumer stream (DLPack convention: 1 = legacy default
        stream, 2 = per-thread default stream, otherwise a ``cudaStream_t``) the
        consumer stream is made to wait on the device for every queued launch,
        so the export does not block the host; ``stream=-1`` asks for no
        synchronisation at all.
        """
        if self._device == "cpu":
            return self._cpu.__dlpack__()  # type: ignore[union-attr]
        rt = _runtime()
        if stream is None:
            rt.synchronize()
        elif int(stream) != -1:
            s = int(stream)
            rt.stream_wait_pending({1: 0, 2: 2}.get(s, s))
        return export_capsule(self._cuda.ptr, self._shape, self._dtype.itemsize, KDL_CUDA, self._cuda.device, self)

    def __dlpack_device__(self) -> tuple[int, int]:
        if self._device == "cpu":
            return (KDL_CPU, 0)
        return (KDL_CUDA, self._cuda.device)

    # -- conversions -------------------------------------------------------------------
    def to_torch(self, device: str | None = None) -> Any:
        torch = _torch()
        if torch is None:
            raise RuntimeError("torch is not available; install it to use Tensor.to_torch()")
        target = device if device is not None else ("cpu" if self._device == "cpu" else f"cuda:{self._cuda.device}")
        kind, idx = _parse_device(target)
        if kind == "cpu":
            return torch.from_numpy(self.numpy())
        if self._device == "cuda" and idx == self._cuda.device:
            return torch.from_dlpack(self)
        return torch.from_numpy(self.numpy()).to(f"cuda:{idx}")

    def to(self, device: Any) -> "Tensor":
        kind, idx = _parse_device(device)
        if kind == self._device and (kind == "cpu" or idx == self._cuda.device):
            return self
        if kind == "cpu":
            return Tensor(shape=self._shape, dtype=self._dtype, device="cpu", cpu=self.numpy())
        host = self.numpy() if self._device == "cuda" else self._cpu
        from .runtime.cuda import DeviceBuffer

        buf = DeviceBuffer(max(self.nbytes, 1), idx)
        buf.copy_from_host(host)
        return Tensor(shape=self._shape, dtype=self._dtype, device="cuda",
                      cuda=_CudaStorage(buf.ptr, self.nbytes, idx, buf))


def tensor(data: Any, *, device: Any | None = None, dtype: Any | None = None) -> Tensor:
    kind, idx = _parse_device(device)
    torch = _torch()
    if torch is not None and isinstance(data, torch.Tensor):
        t = data.detach()
        if dtype is not None:
            want = torch.float16 if _require_supported_dtype(dtype) == np.float16 else torch.float32
            if t.dtype != want:
                t = t.to(dtype=want)
        elif t.dtype not in (torch.float16, torch.float32):
            t = t.to(dtype=torch.float32)
        if kind == "cuda" and t.device.type == "cuda" and int(t.device.index or 0) == idx:
            t = t.contiguous()
            return Tensor._from_cuda_ptr(int(t.data_ptr()), tuple(t.shape), np.float16 if t.dtype == torch.float16
                                         else np.float32, idx, owner=t)
        if t.device.type != "cpu":
            t = t.to("cpu")
        arr = t.contiguous().numpy()
        return Tensor(shape=arr.shape, dtype=arr.dtype, device="cpu", cpu=arr).to(device if kind == "cuda" else "cpu")
    if isinstance(data, Tensor):
        out = data
        if dtype is not None and np.dtype(dtype) != out.dtype:
            out = Tensor(shape=out.shape, dtype=_require_supported_dtype(dtype), device="cpu",
                         cpu=out.numpy().astype(dtype, copy=True))
        return out.to(device if kind == "cuda" else "cpu")
    if dtype is None:
        arr = np.asarray(data)
        if arr.dtype not in (np.float16, np.float32):
            arr = arr.astype(np.float32)
    else:
        arr = np.asarray(data, dtype=_require_supported_dtype(dtype))
    if not arr.flags.c_contiguous:
        arr = np.ascontiguousarray(arr)
    cpu_t = Tensor(shape=arr.shape, dtype=arr.dtype, device="cpu", cpu=arr)
    return cpu_t.to(device if kind == "cuda" else "cpu")


def empty(shape: int | tuple[int, ...], *, device: Any | None = None, dtype: Any | None = None) -> Tensor:
    kind, idx = _parse_device(device)
    d = _require_supported_dtype(np.float32 if dtype is None else dtype)
    shp = (int(shape),) if isinstance(shape, int) else tuple(int(x) for x in shape)
    if kind == "cpu":
        return Tensor(shape=shp, dtype=d, device="cpu", cpu=np.empty(shp, dtype=d))
    from .runtime.cuda import DeviceBuffer

    nbytes = _numel(shp) * d.itemsize
    buf = DeviceBuffer(max(nbytes, 1), idx)
    return Tensor(shape=shp, dtype=d, device="cuda", cuda=_CudaStorage(buf.ptr, nbytes, idx, buf))


def empty_like(x: Tensor, *, device: Any | None = None) -> Tensor:
    if device is None:
        device = x.device if x.device == "cpu" else f"cuda:{x._cuda_device()}"
    return empty(x.shape, device=device, dtype=x.dtype)
