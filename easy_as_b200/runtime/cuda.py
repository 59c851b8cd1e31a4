"""CUDA runtime: the B200 counterpart of the reference's ``MetalRuntime``.

Same public methods and launch semantics as easy_as ``eas/runtime/metal.py``:

* ``run(ck, runtime_args, meta, *, sync, nthreads, grid, tptg, shape)``
  (``metal.py:244-352``): checks ``tptg`` against the launch mode, derives the
  grid with the reference's rules (``grid.py``; thread mode 1D without
  ``_grid`` runs exactly ``N`` threads), resolves every buffer argument to a
  device pointer, packs the kernel parameters, launches, and either waits
  (``sync=True``) or queues an event, keeping at most ``EAS_MAX_IN_FLIGHT``
  (default 256) launches in flight (``metal.py:52-67,346-352``).
* ``synchronize()`` drains the queue (``metal.py:354-360``).
* ``benchmark(...)`` times ``repeat`` launches after ``warmup`` with CUDA
  events on the launch stream and returns seconds per launch
  (``metal.py:362-506`` used wall-clock time around a command buffer).

Buffer arguments may be torch CUDA tensors (zero copy, launched on torch's
current stream), ``eas.Tensor(device="cuda")``, or host arrays (numpy, torch
CPU, ``eas.Tensor(device="cpu")``), which are bridged through temporary device
buffers and copied back when written (``metal.py:209-233,337-344``).

There is no CPU fallback: without the native library or a GPU every entry
point raises.
"""

from __future__ import annotations

import hashlib
import math
import os
import struct
from collections import deque
from pathlib import Path
from typing import Any, Mapping

import numpy as np

from ..ir import DType
from ..tensor import Tensor
from . import cuda_ext
from .grid import grid_rank, infer_1d_grid, infer_grid, infer_nthreads

ALL_THREADS = 0xFFFFFFFF
MAX_GRID_YZ = 65535


def _torch() -> Any:
    try:
        import torch  # type: ignore

        return torch
    except Exception:
        return None


class DeviceBuffer:
    """Owning handle of one ``cudaMalloc`` allocation on one device."""

    __slots__ = ("ptr", "nbytes", "device", "__weakref__")

    def __init__(self, nbytes: int, device: int = 0):
        lib = cuda_ext.load()
        p = cuda_ext.ctypes.c_void_p()
        cuda_ext.check(lib.eas_alloc_buffer(int(device), int(nbytes), cuda_ext.ctypes.byref(p)), "alloc_buffer")
        self.ptr = int(p.value or 0)
        self.nbytes = int(nbytes)
        self.device = int(device)

    def free(self) -> None:
        if self.ptr:
            lib = cuda_ext.load(require=False)
            if lib is not None:
                lib.eas_free_buffer(self.ptr)
            self.ptr = 0

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.free()
        except Exception:
            pass

    def copy_from_host(self, arr: Any, stream: int = 0) -> None:
        a = np.ascontiguousarray(arr)
        if a.nbytes > self.nbytes:
            raise ValueError(f"copy_from_host: {a.nbytes} bytes do not fit a {self.nbytes}-byte buffer")
        lib = cuda_ext.load()
        cuda_ext.check(lib.eas_copy_from_host(self.ptr, a.ctypes.data, a.nbytes, stream), "copy_from_host")

    def copy_to_host(self, out: Any, stream: int = 0) -> None:
        if not isinstance(out, np.ndarray):  # bytearray, memoryview, ...: any writable buffer
            out = np.frombuffer(out, dtype=np.uint8)
            if not out.flags.writeable:
                raise ValueError("copy_to_host needs a writable destination")
        if not out.flags.c_contiguous:
            raise ValueError("copy_to_host needs a C-contiguous destination")
        if out.nbytes > self.nbytes:
            raise ValueError(f"copy_to_host: {out.nbytes} bytes exceed the {self.nbytes}-byte buffer")
        lib = cuda_ext.load()
        cuda_ext.check(lib.eas_copy_to_host(out.ctypes.data, self.ptr, out.nbytes, stream), "copy_to_host")


# ---------------------------------------------------------------------------
# kernel parameter packing
# ---------------------------------------------------------------------------

_PACK_PTR = struct.Struct("<Q").pack_into
_SCALAR_FMT = {DType.U32: ("<I", 4), DType.F32: ("<f", 4), DType.F16: ("<H", 2), DType.BOOL: ("<?", 1)}


class ParamLayout:
    """Byte layout of a generated kernel's parameters (natural alignment, in order)."""

    def __init__(self, params: list[Any]):
        self.entries: list[tuple[Any, int, str]] = []
        off = 0
        for p in params:
            if p.kind in ("buffer", "check"):   # pointers; the u64 bounds of the checked mode
                fmt, size = "<Q", 8
            else:
                fmt, size = _SCALAR_FMT[p.dtype]
            off = -(-off // size) * size
            self.entries.append((p, off, fmt))
            off += size
        self.size = -(-off // 8) * 8
        self.offsets = (cuda_ext.ctypes.c_uint32 * max(len(self.entries), 1))(*[o for _p, o, _f in self.entries])
        self.count = len(self.entries)
        # one struct for the whole block: explicit pad bytes reproduce the natural alignment above
        fmt, pos = "<", 0
        for _p, o, f in self.entries:
            fmt += "x" * (o - pos) + f[1:]
            pos = o + struct.calcsize(f)
        fmt += "x" * (self.size - pos)
        self._struct = struct.Struct(fmt)
        self.block = None  # ctypes uint32[3] of the CUDA block shape, set by the runtime

    def pack(self, values: Mapping[str, Any], pointers: Mapping[str, int], hidden: Mapping[str, int]) -> bytes:
        vals = []
        for p, _off, _fmt in self.entries:
            if p.kind == "buffer":
                vals.append(pointers[p.arg])
            elif p.kind in ("hidden", "check"):
                vals.append(hidden[p.name])
            else:
                vals.append(_scalar_bits(p.dtype, values[p.arg], p.arg))
        return self._struct.pack(*vals)


def _scalar_bits(dt: DType, v: Any, name: str) -> Any:
    if dt == DType.U32:
        iv = int(v)
        if not 0 <= iv < (1 << 32):
            raise ValueError(f"scalar {name!r}={iv} does not fit u32")
        return iv
    if dt == DType.F32:
        return float(v)
    if dt == DType.F16:
        return int(np.array(v, dtype=np.float16).view(np.uint16))
    return bool(v)


def _elem_count(v: Any) -> int:
    """Elements of a buffer argument (numpy array, torch tensor or eas.Tensor)."""
    if isinstance(v, np.ndarray):
        return int(v.size)
    numel = getattr(v, "numel", None)
    if callable(numel):
        return int(numel())
    return int(v.nbytes) // np.dtype(v.dtype).itemsize


def _describe_violation(ck: Any, what: int, index: int, bounds: Mapping[str, tuple[int, int]]) -> str:
    """Message for the error record (2 * slot + is_store, index) of a bounds-checked kernel."""
    from ..codegen.cuda import CHECK_TG_SLOT

    slot, store = divmod(what, 2)
    verb = "store to" if store else "load from"
    kernel = ck.plan.kernel_name
    if slot >= CHECK_TG_SLOT:
        n = [int(i.args[0]) for i in ck.ir.insts if i.op == "alloc_tg"][slot - CHECK_TG_SLOT]
        return (f"{kernel}: out-of-bounds {verb} threadgroup allocation #{slot - CHECK_TG_SLOT} at element "
                f"{index} (it holds {n} elements)")
    name = ck.ir.args[slot].name
    lo, n = bounds.get(name, (0, 0))
    return f"{kernel}: out-of-bounds {verb} {name!r} at element {index} (valid elements: [{lo}, {lo + n}))"


# ---------------------------------------------------------------------------
# launch geometry
# ---------------------------------------------------------------------------


def launch_geometry(ck: Any, runtime_args: Mapping[str, Any], *, nthreads: int | None,
                    grid: tuple[int, int, int] | None, tptg: tuple[int, int, int] | None,
                    shape: tuple[int, ...] | None) -> tuple[tuple[int, int, int], int] | None:
    """Programs per axis and active-thread count, or None when there is nothing to run.

    Thread mode: one program = one block of ``block_size`` threads.
    SPMD mode: one program = ``block_size`` lanes.  Follows ``metal.py:257-326``.
    """
    bs = int(ck.block_size)
    thread_mode = ck.launch_mode == "thread"
    expected = (bs, 1, 1) if thread_mode else (1, 1, 1)
    if tptg is not None and tuple(int(x) for x in tptg) != expected:
        raise ValueError(f"tptg must match kernel launch mode: expected {expected}, "
                         f"got ({tptg[0]}, {tptg[1]}, {tptg[2]})")
    if grid is None:
        plan = getattr(ck, "plan", None)
        rank = getattr(plan, "grid_rank", None) if plan is not None else None
        if plan is not None and rank is None:
            rank = plan.grid_rank = grid_rank(ck.ir)
        inferred = infer_grid(ck.ir, runtime_args, bs, shape=shape, rank=rank)
        if inferred is None:
            n = infer_nthreads(runtime_args, nthreads=nthreads)
            if n == 0:
                return None
            if thread_mode:
                return (math.ceil(n / bs), 1, 1), n
            return (infer_1d_grid(runtime_args, bs, nthreads=nthreads), 1, 1), ALL_THREADS
        dims = tuple(int(x) for x in inferred)
    else:
        dims = tuple(int(x) for x in grid)
        if min(dims) < 0:
            raise ValueError("grid dims must be >= 0")
    if min(dims) == 0:
        return None
    return dims, ALL_THREADS  # type: ignore[return-value]


# ---------------------------------------------------------------------------
# runtime
# ---------------------------------------------------------------------------


def _cache_dir() -> Path | None:
    d = os.environ.get("EAS_CACHE_DIR", str(Path.home() / ".cache" / "easy_as_b200"))
    if d in ("", "0", "off", "none"):
        return None
    return Path(d)


class _Arg:
    """A buffer argument resolved to a device pointer."""

    __slots__ = ("ptr", "device", "keep", "host", "dev_buf", "torch_stream", "bounce", "deferred", "zero_copy")

    def __init__(self, ptr: int, device: int | None, keep: Any = None, host: np.ndarray | None = None,
                 dev_buf: DeviceBuffer | None = None, torch_stream: bool = False, bounce: int | None = None):
        self.ptr, self.device, self.keep, self.host = ptr, device, keep, host
        self.dev_buf, self.torch_stream, self.bounce = dev_buf, torch_stream, bounce
        self.deferred = False  # copy-in not made yet (a write-only host output; see _settle_deferred)
        self.zero_copy = False  # the kernel works on the page-locked bounce buffer in place


class _FastLaunch:
    """A launch prepared once for repeated calls whose inputs differ only in buffer contents or
    pointers (the same kernel, meta, scalars, grid and buffer kinds, shapes and dtypes): the
    pipeline, grid, block and the packed parameter block are fixed, so a call patches the buffer
    pointers into the block and makes one driver call.

    mode ``"device"``: every buffer is a contiguous CUDA torch tensor or a CUDA eas.Tensor;
    ``ptr_slots`` holds (byte offset, argument position, is torch tensor).
    mode ``"zerocopy"``: every buffer is a small host numpy array of an elementwise kernel; the
    kernel works on the pinned bounce buffer in place (pointers fixed), ``copy_in`` /
    ``copy_out`` hold (argument position, bounce offset, bytes).
    """

    __slots__ = ("rt", "lib", "mode", "pipe", "grid", "block", "dyn", "buf", "offsets", "count", "launch",
                 "device", "torch_stream", "ptr_slots", "bounce", "copy_in", "copy_out", "bounds_env")

class _Bounce:
    """Page-locked host buffer and its device twin, for launches with small host arrays."""

    __slots__ = ("host_ptr", "view", "dev", "nbytes", "mapped")

    def __init__(self, nbytes: int, device: int):
        lib = cuda_ext.load()
        p = cuda_ext.ctypes.c_void_p()
        cuda_ext.check(lib.eas_alloc_pinned(nbytes, cuda_ext.ctypes.byref(p)), "pinned bounce buffer")
        self.host_ptr = int(p.value)
        self.view = np.ctypeslib.as_array((cuda_ext.ctypes.c_uint8 * nbytes).from_address(self.host_ptr))
        self.dev = DeviceBuffer(nbytes, device)
        self.nbytes = nbytes
        m = cuda_ext.ctypes.c_void_p()   # device address of the pinned buffer (zero-copy launches)
        cuda_ext.check(lib.eas_pinned_device_pointer(self.host_ptr, cuda_ext.ctypes.byref(m)), "mapped bounce buffer")
        self.mapped = int(m.value or 0)

    def free(self) -> None:
        if self.host_ptr:
            lib = cuda_ext.load(require=False)
            if lib is not None:
                lib.eas_free_pinned(self.host_ptr)
            self.host_ptr = 0
            self.view = None
        self.dev.free()


class CudaRuntime:
    def __init__(self) -> None:
        self._available: bool | None = None
        self._reason = ""
        self._pipelines: dict[tuple[str, str, int, int], int] = {}
        self._pending: deque[tuple[int, int, Any]] = deque()
        self._max_in_flight: int | None = None
        self._staging: dict[tuple[int, int], list[DeviceBuffer]] = {}
        self._bounce: dict[int, _Bounce] = {}
        self._check_records: dict[int, DeviceBuffer] = {}   # per device: error record of checked kernels
        self._pdl_on: bool | None = None
        self.skipped_copy_bytes = 0  # host->device bytes not copied because a launch stores all of them
        self._bucket_keep: list[Any] = []
        self._pending_n = 0
        self._bucket_n = 0
        self._bucket_stream = 0
        self._event_pool: list[int] = []
        self.launch_count = 0  # kernels launched through this runtime (generic + native)
        self.native_launches = 0  # of which pattern-lowered native kernels
        self._scratch_bufs: dict[tuple[int, int, str], DeviceBuffer] = {}

    def scratch(self, device: int, stream: int, tag: str, nbytes: int) -> tuple[int, Any] | None:
        """Device scratch of at least ``nbytes`` for a native launch on ``stream``: (pointer, owner);
        keep ``owner`` until the launch is enqueued.  With torch, the block comes from torch's
        caching allocator on ``stream`` (stream-ordered reuse; inside a CUDA-graph capture, from the
        graph's private pool, kept for its replays).  Without torch: one cached buffer per
        (device, stream, tag), grown after the stream drained; None when that would have to happen
        inside a capture (the caller then declines)."""
        try:
            import torch  # type: ignore
        except Exception:  # pragma: no cover - torch is part of the image
            torch = None
        if torch is not None and torch.cuda.is_available():
            with torch.cuda.device(int(device)):
                ctx = (torch.cuda.stream(torch.cuda.ExternalStream(int(stream), device=int(device))) if stream
                       else torch.cuda.stream(torch.cuda.default_stream(int(device))))
                with ctx:
                    t = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=f"cuda:{int(device)}")
            return int(t.data_ptr()), t
        key = (int(device), int(stream), tag)
        buf = self._scratch_bufs.get(key)
        if buf is not None and buf.nbytes >= nbytes:
            return buf.ptr, buf
        capturing = cuda_ext.ctypes.c_int(0)
        if stream:
            cuda_ext.check(self.lib().eas_stream_is_capturing(stream, cuda_ext.ctypes.byref(capturing)), "capture state")
        if capturing.value:
            return None
        if buf is not None:
            cuda_ext.check(self.lib().eas_stream_synchronize(stream), "scratch resize")
            buf.free()
        buf = DeviceBuffer(max(int(nbytes), 256), int(device))
        self._scratch_bufs[key] = buf
        return buf.ptr, buf

    # -- availability ----------------------------------------------------------
    def is_available(self) -> bool:
        if self._available is None:
            lib = cuda_ext.load(require=False)
            if lib is None:
                self._available, self._reason = False, cuda_ext.load_error() or "native library missing"
            else:
                self._available = bool(lib.eas_is_available())
                self._reason = "" if self._available else cuda_ext.last_error()
        return self._available

    def unavailable_reason(self) -> str:
        self.is_available()
        return self._reason

    @staticmethod
    def lib() -> Any:
        return cuda_ext.load()

    def default_device(self) -> int:
        t = _torch()
        if t is not None and t.cuda.is_available() and t.cuda.is_initialized():
            return int(t.cuda.current_device())
        return int(os.environ.get("EAS_DEVICE", "0"))

    def _pdl(self) -> bool:
        """EAS_PDL: launch generated kernels with programmatic dependent launch (see eas_launch_pdl)."""
        if self._pdl_on is None:
            self._pdl_on = os.environ.get("EAS_PDL", "1") not in ("0", "off", "")
        return self._pdl_on

    def _max_flight(self) -> int:
        if self._max_in_flight is None:
            try:
                v = int(os.environ.get("EAS_MAX_IN_FLIGHT", "256").strip() or 256)
            except ValueError:
                v = 256
            self._max_in_flight = max(v, 0)
        return self._max_in_flight

    # -- compile / pipelines ---------------------------------------------------------
    def compile_cubin(self, src: str, name: str) -> bytes:
        lib = self.lib()
        drv, nvrtc = cuda_ext.ctypes.c_int(), cuda_ext.ctypes.c_int()
        lib.eas_versions(cuda_ext.ctypes.byref(drv), cuda_ext.ctypes.byref(nvrtc))
        key = hashlib.sha256(f"sm_100a|nvrtc{nvrtc.value}|{name}|".encode() + src.encode()).hexdigest()
        cdir = _cache_dir()
        if cdir is not None:
            f = cdir / f"{key}.cubin"
            if f.exists():
                return f.read_bytes()
        img, size = cuda_ext.ctypes.c_void_p(), cuda_ext.ctypes.c_size_t()
        rc = lib.eas_compile(src.encode(), f"{name}.cu".encode(), None, 0, cuda_ext.ctypes.byref(img),
                             cuda_ext.ctypes.byref(size))
        if rc != cuda_ext.EAS_OK:
            msg = cuda_ext.last_error()
            if rc == cuda_ext.EAS_ERR_COMPILE:
                raise RuntimeError(f"CUDA compile failed: {msg}")
            cuda_ext.check(rc, "compile")
        try:
            data = cuda_ext.ctypes.string_at(img.value, size.value)
        finally:
            lib.eas_free_host(img)
        if cdir is not None:
            try:
                cdir.mkdir(parents=True, exist_ok=True)
                tmp = cdir / f"{key}.{os.getpid()}.tmp"
                tmp.write_bytes(data)
                os.replace(tmp, cdir / f"{key}.cubin")
            except OSError:
                pass
        return data

    def pipeline(self, src: str, name: str, device: int, dyn_smem: int) -> int:
        key = (src, name, device, dyn_smem)
        p = self._pipelines.get(key)
        if p is None:
            cubin = self.compile_cubin(src, name)
            lib = self.lib()
            h = cuda_ext.ctypes.c_void_p()
            cuda_ext.check(lib.eas_pipeline_load(device, cubin, len(cubin), name.encode(),
                                                 dyn_smem if dyn_smem > 48 * 1024 else 0,
                                                 cuda_ext.ctypes.byref(h)), "pipeline_load")
            p = int(h.value)
            self._pipelines[key] = p
        return p

    def _pipeline_for(self, ck: Any, device: int) -> int:
        plan = ck.plan
        return self.pipeline(ck.src, plan.kernel_name, device, plan.dyn_smem)

    # -- arguments ---------------------------------------------------------------------
    def _resolve(self, ck: Any, runtime_args: Mapping[str, Any], *, allow_host: bool = True,
                 allow_bounce: bool = True) -> tuple[dict[str, _Arg], int, int]:
        torch = _torch()
        resolved: dict[str, _Arg] = {}
        device: int | None = None
        torch_stream = False
        host_pending: list[tuple[str, np.ndarray]] = []
        for a in ck.ir.args:
            if a.kind != "buffer":
                continue
            v = runtime_args[a.name]
            want = np.float32 if a.dtype == DType.F32 else np.float16
            if type(v) is Tensor and v._device == "cuda" and v._dtype == want:
                dev = v._cuda_device()
                if device is not None and dev != device:
                    raise ValueError(f"buffers on different devices: {device} and {dev}")
                device = dev
                resolved[a.name] = _Arg(v._cuda_ptr(), dev, keep=v)
                continue
            if torch is not None and type(v) is torch.Tensor and v.is_cuda and not v.requires_grad:
                # common case first: a contiguous CUDA tensor of the right dtype
                if v.dtype == (torch.float32 if a.dtype == DType.F32 else torch.float16) and v.is_contiguous():
                    dev = v.get_device()
                    if device is not None and dev != device:
                        raise ValueError(f"buffers on different devices: {device} and {dev}")
                    device = dev
                    resolved[a.name] = _Arg(v.data_ptr(), dev, keep=v)
                    torch_stream = True
                    continue
            if torch is not None and isinstance(v, torch.Tensor):
                t = v.detach()
                tdt = torch.float32 if a.dtype == DType.F32 else torch.float16
                if t.dtype != tdt:
                    raise TypeError(f"{a.name!r} must be {tdt}, got {t.dtype}")
                if t.device.type == "cuda":
                    if not t.is_contiguous():
                        if a.name in ck.writes:
                            raise ValueError(f"{a.name!r} is written by the kernel and must be contiguous")
                        t = t.contiguous()
                    dev = int(t.device.index or 0)
                    if device is not None and dev != device:
                        raise ValueError(f"buffers on different devices: {device} and {dev}")
                    device = dev
                    resolved[a.name] = _Arg(int(t.data_ptr()), dev, keep=t)
                    torch_stream = True
                    continue
                if t.device.type != "cpu":
                    raise TypeError(f"unsupported torch device for {a.name!r}: {t.device!s}")
                v = t.contiguous().numpy()
            if getattr(v, "__eas_tensor__", False):
                if np.dtype(v.dtype) != np.dtype(want):
                    raise TypeError(f"{a.name!r} dtype mismatch: expected {np.dtype(want)}, got {v.dtype}")
                if v.device == "cuda":
                    dev = v._cuda_device()
                    if device is not None and dev != device:
                        raise ValueError(f"buffers on different devices: {device} and {dev}")
                    device = dev
                    resolved[a.name] = _Arg(v._cuda_ptr(), dev, keep=v)
                    continue
                v = v.numpy()
            if isinstance(v, np.ndarray):
                if v.dtype != want:
                    raise TypeError(f"{a.name!r} must be {np.dtype(want)}, got {v.dtype}")
                if not v.flags.c_contiguous:
                    raise ValueError(f"{a.name!r} must be C-contiguous for MVP")
                if not allow_host:
                    raise ValueError("benchmark() with numpy inputs is not supported; use eas.Tensor(device='cuda') "
                                     "or torch CUDA tensors for device-native timing")
                host_pending.append((a.name, v))
                continue
            raise TypeError(f"expected numpy.ndarray, torch.Tensor or eas.Tensor for {a.name!r}, got {type(v)!r}")
        if device is None:
            device = self.default_device()
        stream = 0
        if torch_stream and torch is not None:
            raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
            stream = int(raw(device)) if raw is not None else int(torch.cuda.current_stream(device).cuda_stream)
        if host_pending and allow_bounce and self._bounce_resolve(ck, host_pending, resolved, device, stream):
            return resolved, device, stream
        # host arrays: one temporary device buffer per distinct array object.  An array the kernel
        # only writes, under a single name, is not copied in yet: the launch may store every element
        # of it (_settle_deferred decides before the launch)
        staged: dict[int, DeviceBuffer] = {}
        names_of: dict[int, list[str]] = {}
        for name, arr in host_pending:
            names_of.setdefault(id(arr), []).append(name)
        reads = getattr(ck.plan, "reads", None)
        for name, arr in host_pending:
            buf = staged.get(id(arr))
            names = names_of[id(arr)]
            defer = (reads is not None and len(names) == 1 and name in ck.writes and name not in reads)
            if buf is None:
                buf = self._stage(device, max(arr.nbytes, 1))
                if not defer:
                    buf.copy_from_host(arr, stream)
                staged[id(arr)] = buf
            a = _Arg(buf.ptr, device, keep=arr, host=arr if name in ck.writes else None, dev_buf=buf)
            a.deferred = defer
            resolved[name] = a
        return resolved, device, stream

    def _settle_deferred(self, ck: Any, runtime_args: Mapping[str, Any], args: dict[str, _Arg], stream: int,
                         programs: tuple[int, int, int], ntx: int) -> None:
        """Make the copy-in of write-only host outputs unless the launch provably stores every
        element of them (a native GEMM plan's output rectangle covering the whole buffer; the
        generated kernel stores the same elements, so this holds whichever kernel runs)."""
        native = getattr(ck.plan, "native", None)
        for name, a in args.items():
            if not a.deferred:
                continue
            a.deferred = False
            covers = getattr(native, "covers", None)
            if covers is not None and covers(runtime_args, programs, ntx, name, int(a.host.size)):
                self.skipped_copy_bytes += int(a.host.nbytes)
                continue
            a.dev_buf.copy_from_host(a.host, stream)

    # -- small host arrays: one pinned bounce buffer ----------------------------------
    BOUNCE_MAX_BYTES = 4 << 20   # host arrays up to this total go through the bounce buffer
    ZERO_COPY_MAX_BYTES = 256 << 10  # elementwise launches up to this total run on the bounce buffer in place
    _BOUNCE_ALIGN = 256

    def _bounce_resolve(self, ck: Any, host_pending: list[tuple[str, np.ndarray]], resolved: dict[str, _Arg],
                        device: int, stream: int) -> bool:
        """Pack the distinct host arrays into the device's pinned bounce buffer and copy them in
        with ONE asynchronous copy (instead of a synchronous copy per array).  False when they
        are too large: the caller stages them one by one."""
        distinct: dict[int, np.ndarray] = {}
        for _name, arr in host_pending:
            distinct.setdefault(id(arr), arr)
        al = self._BOUNCE_ALIGN
        total = sum(-(-max(a.nbytes, 1) // al) * al for a in distinct.values())
        if total > self.BOUNCE_MAX_BYTES:
            return False
        bb = self._bounce.get(device)
        if bb is None or bb.nbytes < total:
            if bb is not None:
                cuda_ext.check(self.lib().eas_stream_synchronize(stream), "bounce resize")
                bb.free()
            bb = self._bounce[device] = _Bounce(max(64 << 10, 1 << (total - 1).bit_length()), device)
        offs: dict[int, int] = {}
        cur = 0
        for key, arr in distinct.items():
            n = arr.nbytes
            if n:
                bb.view[cur:cur + n] = arr.reshape(-1).view(np.uint8)
            offs[key] = cur
            cur += -(-max(n, 1) // al) * al
        # an elementwise launch touches each element once: it reads and writes the page-locked buffer
        # in place over PCIe (no copies); other kernels may re-read, so they get the device copy
        # (small launches only: a kernel reaching host memory over PCIe makes many small requests,
        # so beyond a few hundred KiB one bulk copy each way is faster)
        zero_copy = (getattr(ck.plan, "elementwise", None) is not None and bb.mapped
                     and cur <= self.ZERO_COPY_MAX_BYTES
                     and os.environ.get("EAS_ZERO_COPY", "1") not in ("0", "off"))
        base = bb.mapped if zero_copy else bb.dev.ptr
        if not zero_copy:
            cuda_ext.check(self.lib().eas_copy_from_host_async(bb.dev.ptr, bb.host_ptr, cur, stream), "copy in")
        for name, arr in host_pending:
            o = offs[id(arr)]
            a = _Arg(base + o, device, keep=arr, host=arr if name in ck.writes else None, bounce=o)
            a.zero_copy = zero_copy
            resolved[name] = a
        return True

    def _finish_host_copies(self, host_args: list[_Arg], device: int, stream: int) -> None:
        """After the launch: copy written host arrays back (one asynchronous copy per array through
        the bounce buffer, or a synchronous copy per staged buffer), wait once, unpack."""
        lib = self.lib()
        bb = self._bounce.get(device)
        out: dict[int, _Arg] = {}
        for a in host_args:
            if a.host is not None and id(a.host) not in out:
                out[id(a.host)] = a
        for a in out.values():
            if a.bounce is not None and a.host.nbytes and not a.zero_copy:
                cuda_ext.check(lib.eas_copy_to_host_async(bb.host_ptr + a.bounce, bb.dev.ptr + a.bounce, a.host.nbytes,
                                                          stream), "copy out")
        cuda_ext.check(lib.eas_stream_synchronize(stream), "kernel execution")
        self._check_native_status(device)
        for a in out.values():
            if a.bounce is not None:
                if a.host.nbytes:
                    a.host.reshape(-1).view(np.uint8)[:] = bb.view[a.bounce:a.bounce + a.host.nbytes]
            else:
                a.dev_buf.copy_to_host(a.host, stream)

    # -- host staging buffers ----------------------------------------------------------
    def _stage(self, device: int, nbytes: int) -> DeviceBuffer:
        free = self._staging.get((device, nbytes))
        return free.pop() if free else DeviceBuffer(nbytes, device)

    def _unstage(self, args: dict[str, _Arg]) -> None:
        """Return staging buffers of host arguments to the pool (after the launch has completed)."""
        seen: set[int] = set()
        for a in args.values():
            b = a.dev_buf
            if b is not None and id(b) not in seen:
                seen.add(id(b))
                free = self._staging.setdefault((b.device, b.nbytes), [])
                if len(free) < 4:
                    free.append(b)
                a.dev_buf = None

    # -- launch -------------------------------------------------------------------------
    def _launch_generic(self, ck: Any, runtime_args: Mapping[str, Any], args: dict[str, _Arg], device: int,
                        stream: int, programs: tuple[int, int, int], ntx: int,
                        pid_base: tuple[int, int, int] = (0, 0, 0),
                        elem_base: Mapping[str, int] | None = None) -> None:
        plan = ck.plan
        if plan.checked:
            self._launch_checked(ck, runtime_args, args, device, stream, programs, ntx, pid_base, elem_base or {})
            return
        self._launch_generic_raw(ck, runtime_args, args, device, stream, programs, ntx, pid_base, None)

    def _launch_generic_raw(self, ck: Any, runtime_args: Mapping[str, Any], args: dict[str, _Arg], device: int,
                            stream: int, programs: tuple[int, int, int], ntx: int, pid_base: tuple[int, int, int],
                            extra: Mapping[str, int] | None) -> None:
        plan = ck.plan
        pipe = self._pipeline_for(ck, device)
        layout = plan.layout
        if layout is None:
            layout = plan.layout = ParamLayout(plan.params)
            layout.block = (cuda_ext.ctypes.c_uint32 * 3)(plan.cuda_threads, 1, 1)
        ptrs = {n: a.ptr for n, a in args.items()}
        lib = self.lib()
        gx, gy, gz = programs
        block = layout.block
        for z0 in range(0, gz, MAX_GRID_YZ):
            for y0 in range(0, gy, MAX_GRID_YZ):
                hidden = {"eas_ntx": ntx, "eas_pid_x": pid_base[0], "eas_pid_y": pid_base[1] + y0,
                          "eas_pid_z": pid_base[2] + z0}
                if extra:
                    hidden.update(extra)
                blob = layout.pack(runtime_args, ptrs, hidden)
                g = (cuda_ext.ctypes.c_uint32 * 3)(gx, min(MAX_GRID_YZ, gy - y0), min(MAX_GRID_YZ, gz - z0))
                launch = lib.eas_launch_pdl if self._pdl() else lib.eas_launch
                cuda_ext.check(launch(pipe, g, block, plan.dyn_smem, stream, blob, layout.offsets, layout.count),
                               f"launch {plan.kernel_name}")
                self.launch_count += 1

    # -- bounds-checked kernels (EAS_BOUNDS_CHECK) ---------------------------------------
    def _launch_checked(self, ck: Any, runtime_args: Mapping[str, Any], args: dict[str, _Arg], device: int,
                        stream: int, programs: tuple[int, int, int], ntx: int, pid_base: tuple[int, int, int],
                        elem_base: Mapping[str, int]) -> None:
        """Launch a bounds-checked kernel: pass each buffer's element range, clear the error record
        before and read it after the launch (the stream is synchronised), and raise IndexError
        for the first access outside its buffer.  The access itself was skipped on the device."""
        capturing = cuda_ext.ctypes.c_int(0)
        self.lib().eas_stream_is_capturing(stream, cuda_ext.ctypes.byref(capturing))
        if capturing.value:
            raise ValueError("bounds-checked kernels (EAS_BOUNDS_CHECK=1) cannot be captured in a CUDA graph")
        rec = self._check_records.get(device)
        if rec is None:
            rec = self._check_records[device] = DeviceBuffer(16, device)
        zero = np.zeros(4, np.uint32)
        rec.copy_from_host(zero, stream)
        extra: dict[str, int] = {"eas_err": rec.ptr}
        bounds: dict[str, tuple[int, int]] = {}
        for p in ck.plan.params:
            if p.kind == "check" and p.arg is not None and p.arg not in bounds:
                lo = int(elem_base.get(p.arg, 0))
                bounds[p.arg] = (lo, _elem_count(runtime_args[p.arg]))
        for p in ck.plan.params:
            if p.kind == "check" and p.arg is not None:
                lo, n = bounds[p.arg]
                extra[p.name] = lo if p.name.startswith("eas_lo_") else n
        self._launch_generic_raw(ck, runtime_args, args, device, stream, programs, ntx, pid_base, extra)
        cuda_ext.check(self.lib().eas_stream_synchronize(stream), "kernel execution")
        out = np.zeros(4, np.uint32)
        rec.copy_to_host(out, stream)
        if out[0]:
            raise IndexError(_describe_violation(ck, int(out[1]), int(out[2]), bounds))

    def _dispatch(self, ck: Any, runtime_args: Mapping[str, Any], args: dict[str, _Arg], device: int, stream: int,
                  programs: tuple[int, int, int], ntx: int) -> None:
        native = getattr(ck.plan, "native", None)
        if native is not None and native.try_launch(self, ck, runtime_args, args, device, stream, programs, ntx):
            return
        self._launch_generic(ck, runtime_args, args, device, stream, programs, ntx)

    def run(self, ck: Any, runtime_args: Mapping[str, Any], meta: Mapping[str, Any], *, sync: bool = True,
            nthreads: int | None = None, grid: tuple[int, int, int] | None = None,
            tptg: tuple[int, int, int] | None = None, shape: tuple[int, ...] | None = None) -> None:
        _ = meta
        geo = launch_geometry(ck, runtime_args, nthreads=nthreads, grid=grid, tptg=tptg, shape=shape)
        if geo is None:
            return
        if not self.is_available():
            raise RuntimeError("CUDA runtime is not available: " + self._reason)
        hosts = self._pipeline_candidates(ck, runtime_args, geo)
        if hosts is not None:
            self._run_pipelined(ck, runtime_args, geo, hosts)
            return
        gp = self._gemm_pipeline_plan(ck, runtime_args, geo)
        if gp is not None:
            self._run_gemm_pipelined(ck, runtime_args, geo, gp)
            return
        # the shared bounce buffer only serves calls that wait before returning: an asynchronous call
        # could still be waiting for its copy when the next call refills the buffer
        args, device, stream = self._resolve(ck, runtime_args, allow_bounce=sync)
        host_copies = [a for a in args.values() if a.host is not None]
        if any(a.deferred for a in host_copies):
            self._settle_deferred(ck, runtime_args, args, stream, *geo)
        lib = self.lib()
        capturing = cuda_ext.ctypes.c_int(0)
        if stream:
            lib.eas_stream_is_capturing(stream, cuda_ext.ctypes.byref(capturing))
        if capturing.value:
            # inside CUDA graph capture: enqueue only (the graph keeps raw pointers: callers keep buffers alive)
            if sync or host_copies:
                raise ValueError("inside CUDA graph capture launch with _sync=False and device buffers only")
            self._dispatch(ck, runtime_args, args, device, stream, *geo)
            return
        self._dispatch(ck, runtime_args, args, device, stream, *geo)
        if sync or host_copies:
            self._finish_host_copies(host_copies, device, stream)
            self._unstage(args)
            return
        # asynchronous launch: keep the arguments alive until a completion event covers it.
        # One (pooled) event per group of launches; at most EAS_MAX_IN_FLIGHT stay unfinished.
        if self._bucket_n and stream != self._bucket_stream:
            self._close_bucket()
        self._bucket_keep.append((args, runtime_args))
        self._bucket_n += 1
        self._bucket_stream = stream
        limit = self._max_flight()
        if self._bucket_n >= (max(1, limit // 16) if limit else 64):
            self._close_bucket()
        while limit and self.in_flight() > limit:
            if not self._pending:
                self._close_bucket()
            self._wait_one()

    # -- prepared repeated launches (Kernel.__call__ fast path) ------------------------
    def fast_prepare(self, ck: Any, runtime_args: Mapping[str, Any], opts: Mapping[str, Any],
                     positions: Mapping[str, int], axis: int = 0, lo: int | None = None, hi: int | None = None,
                     buffer_base: Mapping[str, int] | None = None) -> _FastLaunch | None:
        """A :class:`_FastLaunch` for this launch, or None when it needs the general path (a
        native plan, a bounds-checked kernel, host arrays other than small elementwise ones, a
        grid split into several launches, ...).  Call after an identical :meth:`run` succeeded.
        With ``lo``/``hi`` it is the :meth:`run_range` launch of programs ``[lo, hi)`` on ``axis``
        (device buffers only; ``buffer_base`` as there)."""
        plan = ck.plan
        if plan.checked or getattr(plan, "native", None) is not None or not self._available:
            return None
        geo = launch_geometry(ck, runtime_args, nthreads=opts.get("nthreads"), grid=opts.get("grid"),
                              tptg=opts.get("tptg"), shape=opts.get("shape"))
        if geo is None:
            return None
        (gx, gy, gz), ntx = geo
        pid = [0, 0, 0]
        if lo is not None:
            dims = [gx, gy, gz]
            lo, hi = max(0, int(lo)), min(int(hi), dims[axis])
            if hi <= lo:
                return None
            dims[axis] = hi - lo
            pid[axis] = lo
            gx, gy, gz = dims
        if gy > MAX_GRID_YZ or gz > MAX_GRID_YZ:
            return None
        torch = _torch()
        fl = _FastLaunch()
        bufs = [a for a in ck.ir.args if a.kind == "buffer"]
        if any(a.name not in positions for a in bufs):
            return None
        kinds = set()
        device = None
        slots: dict[str, tuple[int, bool]] = {}
        for a in bufs:
            v = runtime_args[a.name]
            want_np = np.float32 if a.dtype == DType.F32 else np.float16
            if type(v) is Tensor and v._device == "cuda" and v._dtype == want_np:
                kinds.add("device")
                dev = v._cuda_device()
                slots[a.name] = (positions[a.name], False)
            elif (torch is not None and type(v) is torch.Tensor and v.is_cuda and not v.requires_grad
                  and v.is_contiguous() and v.dtype == (torch.float32 if a.dtype == DType.F32 else torch.float16)):
                kinds.add("device")
                kinds.add("torch")
                dev = v.get_device()
                slots[a.name] = (positions[a.name], True)
            elif type(v) is np.ndarray and v.dtype == want_np and v.flags.c_contiguous:
                kinds.add("host")
                dev = self.default_device()
            else:
                return None
            if device is not None and dev != device:
                return None
            device = dev
        if device is None or ("host" in kinds and "device" in kinds) or ("host" in kinds and lo is not None):
            return None
        layout = plan.layout
        if layout is None:
            layout = plan.layout = ParamLayout(plan.params)
            layout.block = (cuda_ext.ctypes.c_uint32 * 3)(plan.cuda_threads, 1, 1)
        hidden = {"eas_ntx": ntx, "eas_pid_x": pid[0], "eas_pid_y": pid[1], "eas_pid_z": pid[2]}
        if "host" in kinds:
            # small elementwise launches on the pinned bounce buffer, in place (as _bounce_resolve)
            if (getattr(plan, "elementwise", None) is None
                    or os.environ.get("EAS_ZERO_COPY", "1") in ("0", "off")):
                return None
            bb = self._bounce.get(device)
            if bb is None or not bb.mapped:
                return None
            al = self._BOUNCE_ALIGN
            offs: dict[int, int] = {}
            cur = 0
            copy_in = []
            for a in bufs:
                arr = runtime_args[a.name]
                if id(arr) in offs:
                    continue
                offs[id(arr)] = cur
                copy_in.append((positions[a.name], cur, arr.nbytes))
                cur += -(-max(arr.nbytes, 1) // al) * al
            if cur > self.ZERO_COPY_MAX_BYTES or cur > bb.nbytes:
                return None
            ptrs = {a.name: bb.mapped + offs[id(runtime_args[a.name])] for a in bufs}
            seen = set()
            copy_out = []
            for a in bufs:
                arr = runtime_args[a.name]
                if a.name in ck.writes and id(arr) not in seen:
                    seen.add(id(arr))
                    copy_out.append((positions[a.name], offs[id(arr)], arr.nbytes))
            fl.mode, fl.bounce, fl.copy_in, fl.copy_out, fl.ptr_slots = "zerocopy", bb, copy_in, copy_out, ()
        else:
            ptrs = {a.name: 0 for a in bufs}
            fl.mode, fl.bounce, fl.copy_in, fl.copy_out = "device", None, (), ()
            base = buffer_base or {}
            item = {a.name: (4 if a.dtype == DType.F32 else 2) for a in bufs}
            fl.ptr_slots = tuple((off, slots[p.arg][0], slots[p.arg][1], int(base.get(p.arg, 0)) * item[p.arg])
                                 for p, off, _f in layout.entries if p.kind == "buffer")
        fl.rt, fl.lib = self, self.lib()
        fl.pipe = self._pipeline_for(ck, device)
        fl.grid = (cuda_ext.ctypes.c_uint32 * 3)(gx, gy, gz)
        fl.block = layout.block
        fl.dyn = plan.dyn_smem
        blob = layout.pack(runtime_args, ptrs, hidden)
        fl.buf = cuda_ext.ctypes.create_string_buffer(blob, len(blob))
        fl.offsets, fl.count = layout.offsets, layout.count
        fl.launch = fl.lib.eas_launch_pdl if self._pdl() else fl.lib.eas_launch
        fl.device = device
        fl.torch_stream = "torch" in kinds
        return fl

    def fast_run(self, fl: _FastLaunch, args: tuple[Any, ...], sync: bool) -> bool:
        """Launch ``fl`` with the buffers of ``args``; False (nothing done) when the general path
        must take the call (the runtime's library or bounce buffer changed since it was prepared,
        or the stream is being captured)."""
        lib = fl.lib
        if cuda_ext._lib is not lib:
            return False
        buf = fl.buf
        if fl.mode == "device":
            for off, pos, is_torch, back in fl.ptr_slots:
                v = args[pos]
                _PACK_PTR(buf, off, (v.data_ptr() if is_torch else v._cuda_ptr()) - back)
            stream = 0
            if fl.torch_stream:
                stream = int(_torch()._C._cuda_getCurrentRawStream(fl.device))
                if stream:
                    cap = cuda_ext.ctypes.c_int(0)
                    lib.eas_stream_is_capturing(stream, cuda_ext.ctypes.byref(cap))
                    if cap.value:
                        return False
            rc = fl.launch(fl.pipe, fl.grid, fl.block, fl.dyn, stream, buf, fl.offsets, fl.count)
            if rc:
                cuda_ext.check(rc, "launch")
            self.launch_count += 1
            if sync:
                cuda_ext.check(lib.eas_stream_synchronize(stream), "kernel execution")
                return True
            if self._bucket_n and stream != self._bucket_stream:
                self._close_bucket()
            self._bucket_keep.append(args)
            self._bucket_n += 1
            self._bucket_stream = stream
            limit = self._max_flight()
            if self._bucket_n >= (max(1, limit // 16) if limit else 64):
                self._close_bucket()
            while limit and self.in_flight() > limit:
                if not self._pending:
                    self._close_bucket()
                self._wait_one()
            return True
        bb = fl.bounce
        if self._bounce.get(fl.device) is not bb:
            return False
        view = bb.view
        for pos, off, n in fl.copy_in:
            if n:
                view[off:off + n] = args[pos].reshape(-1).view(np.uint8)
        rc = fl.launch(fl.pipe, fl.grid, fl.block, fl.dyn, 0, buf, fl.offsets, fl.count)
        if rc:
            cuda_ext.check(rc, "launch")
        self.launch_count += 1
        cuda_ext.check(lib.eas_stream_synchronize(0), "kernel execution")
        for pos, off, n in fl.copy_out:
            if n:
                args[pos].reshape(-1).view(np.uint8)[:] = view[off:off + n]
        return True

    def _close_bucket(self) -> None:
        if not self._bucket_n:
            return
        lib = self.lib()
        if self._event_pool:
            ev = self._event_pool.pop()
        else:
            e = cuda_ext.ctypes.c_void_p()
            cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e)), "event_create")
            ev = int(e.value)
        cuda_ext.check(lib.eas_event_record(ev, self._bucket_stream), "event_record")
        self._pending.append((ev, self._bucket_n, self._bucket_keep))
        self._pending_n += self._bucket_n
        self._bucket_keep, self._bucket_n = [], 0

    def _wait_one(self) -> None:
        ev, n, _keep = self._pending.popleft()
        self._pending_n -= n
        try:
            cuda_ext.check(self.lib().eas_event_synchronize(ev), "kernel execution")
        finally:
            self._event_pool.append(ev)

    def synchronize(self) -> None:
        self._close_bucket()
        while self._pending:
            self._wait_one()
        if self.native_launches:
            for dev in range(8):
                self._check_native_status(dev)

    def stream_wait_pending(self, stream: int) -> None:
        """Make ``stream`` wait (device side, no host block) for every launch queued so far."""
        self._close_bucket()
        lib = self.lib()
        for ev, _n, _keep in self._pending:
            cuda_ext.check(lib.eas_stream_wait_event(stream, ev), "stream_wait_event")

    def in_flight(self) -> int:
        return self._pending_n + self._bucket_n

    # -- pipelined host-buffer path ----------------------------------------------------
    PIPELINE_CHUNK_ELEMS = 1 << 23      # elements per operand per chunk (32 MiB of f32)
    PIPELINE_SLOTS = 3

    @staticmethod
    def _first_buffer_on_device(ck: Any, runtime_args: Mapping[str, Any]) -> bool:
        """The first buffer argument is device memory (a CUDA torch tensor or a CUDA eas.Tensor):
        the host-pipelined paths, which need every buffer on the host, cannot apply."""
        first = next((runtime_args[a.name] for a in ck.ir.args if a.kind == "buffer"), None)
        if type(first) is Tensor:
            return first._device == "cuda"
        torch = _torch()
        return torch is not None and type(first) is torch.Tensor and first.is_cuda

    def _pipeline_candidates(self, ck: Any, runtime_args: Mapping[str, Any], geo: Any) -> dict[str, np.ndarray] | None:
        """Host arrays of an elementwise kernel, when the pipelined copy path applies.

        Applies when every buffer argument is a page-locked host array (a
        pinned torch CPU tensor, or memory registered with CUDA), the kernel is
        elementwise (program p touches only elements [p*BLOCK, (p+1)*BLOCK)),
        the launch is 1D and the data is large enough to be worth splitting.
        """
        ew = getattr(ck.plan, "elementwise", None)
        if ew is None:
            return None
        if self._first_buffer_on_device(ck, runtime_args):
            return None  # device tensors: nothing to copy
        min_bytes = int(os.environ.get("EAS_PIPELINE_MIN_BYTES", str(64 << 20)))
        if sum(getattr(runtime_args[a.name], "nbytes", 0) for a in ck.ir.args if a.kind == "buffer") < min_bytes:
            return None  # small calls: the bounce buffer or per-array staging serves them
        torch = _torch()
        if os.environ.get("EAS_PIPELINE", "1") in ("0", "off"):
            return None
        (gx, gy, gz), _ntx = geo
        if gy != 1 or gz != 1:
            return None
        hosts: dict[str, np.ndarray] = {}
        total = 0
        for a in ck.ir.args:
            if a.kind != "buffer":
                continue
            v = runtime_args[a.name]
            if torch is not None and isinstance(v, torch.Tensor):
                if v.device.type != "cpu" or not v.is_contiguous():
                    return None
                v = v.detach().numpy()
            elif getattr(v, "__eas_tensor__", False):
                if v.device != "cpu":
                    return None
                v = v.numpy()
            if not isinstance(v, np.ndarray) or not v.flags.c_contiguous:
                return None
            want = np.float32 if a.dtype == DType.F32 else np.float16
            if v.dtype != want:
                return None
            hosts[a.name] = v
            total += v.nbytes
        if not hosts or total < min_bytes:
            return None
        lib = self.lib()   # only large calls pay for the page-lock queries
        pinned = cuda_ext.ctypes.c_int(0)
        for v in hosts.values():
            lib.eas_host_is_pinned(v.ctypes.data, cuda_ext.ctypes.byref(pinned))
            if not pinned.value:
                return None
        return hosts

    def _streams(self, device: int) -> tuple[int, int, int]:
        key = ("pipeline_streams", device)
        st = self._pipelines.get(key)  # type: ignore[arg-type]
        if st is None:
            lib = self.lib()
            out = []
            for _ in range(3):
                h = cuda_ext.ctypes.c_void_p()
                cuda_ext.check(lib.eas_stream_create(device, cuda_ext.ctypes.byref(h)), "stream_create")
                out.append(int(h.value))
            st = tuple(out)
            self._pipelines[key] = st  # type: ignore[index]
        return st  # type: ignore[return-value]

    def _run_pipelined(self, ck: Any, runtime_args: Mapping[str, Any], geo: Any, hosts: dict[str, np.ndarray]) -> None:
        """H2D copy, kernel and D2H copy of successive program ranges overlap on three streams.

        Buffers the kernel never loads are not copied in; only the elements a
        store can reach (below its mask bound) are copied back, so host
        elements the kernel leaves alone are untouched.  Returns after the
        last copy has landed (the launch is synchronous).
        """
        ew = ck.plan.elementwise
        (gx, _, _), ntx = geo
        B = ew.block
        device = self.default_device()
        lib = self.lib()
        s_in, s_run, s_out = self._streams(device)
        progs = max(1, self.PIPELINE_CHUNK_ELEMS // B)
        chunk = progs * B
        distinct: dict[tuple[int, int], tuple[np.ndarray, bool, bool, list[str]]] = {}
        for name, arr in hosts.items():
            arr_id = (arr.ctypes.data, arr.nbytes)  # the same memory passed twice is staged once
            _, r, w, names = distinct.get(arr_id, (arr, False, False, []))
            distinct[arr_id] = (arr, r or name in ew.reads, w or name in ew.writes, names + [name])
        write_limit: dict[str, int] = {}
        for name, b in ew.store_bounds:
            lim = hosts[name].size if b is None else (
                int(runtime_args[b[1]]) if b[0] == "arg" else int(b[1]))
            write_limit[name] = max(write_limit.get(name, 0), min(lim, hosts[name].size))
        R = self.PIPELINE_SLOTS
        slots: dict[tuple[int, int], list[DeviceBuffer]] = {}
        for key, (arr, _r, _w, _n) in distinct.items():
            slots[key] = [self._stage(device, chunk * arr.itemsize) for _ in range(R)]
        evs = []
        for _ in range(3 * R):
            e = cuda_ext.ctypes.c_void_p()
            cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e)), "event_create")
            evs.append(int(e.value))
        ev_in, ev_run, ev_free = evs[:R], evs[R:2 * R], evs[2 * R:]
        try:
            for i, p0 in enumerate(range(0, gx, progs)):
                p1 = min(gx, p0 + progs)
                s = i % R
                lo = p0 * B
                if i >= R:
                    cuda_ext.check(lib.eas_stream_wait_event(s_in, ev_free[s]), "stream_wait_event")
                for key, (arr, reads, _w, _n) in distinct.items():
                    n = min(p1 * B, arr.size) - lo
                    if reads and n > 0:
                        cuda_ext.check(lib.eas_copy_from_host_async(slots[key][s].ptr, arr.ctypes.data + lo * arr.itemsize,
                                                                    n * arr.itemsize, s_in), "pipelined copy in")
                cuda_ext.check(lib.eas_event_record(ev_in[s], s_in), "event_record")
                cuda_ext.check(lib.eas_stream_wait_event(s_run, ev_in[s]), "stream_wait_event")
                args = {}
                for key, (arr, _r, _w, names) in distinct.items():
                    for name in names:
                        args[name] = _Arg(slots[key][s].ptr - lo * arr.itemsize, device)
                self._launch_generic(ck, runtime_args, args, device, s_run, (p1 - p0, 1, 1), ntx, (p0, 0, 0))
                cuda_ext.check(lib.eas_event_record(ev_run[s], s_run), "event_record")
                cuda_ext.check(lib.eas_stream_wait_event(s_out, ev_run[s]), "stream_wait_event")
                for key, (arr, _r, writes, names) in distinct.items():
                    if not writes:
                        continue
                    lim = max(write_limit.get(nm, 0) for nm in names)
                    n = min(p1 * B, lim) - lo
                    if n > 0:
                        cuda_ext.check(lib.eas_copy_to_host_async(arr.ctypes.data + lo * arr.itemsize, slots[key][s].ptr,
                                                                  n * arr.itemsize, s_out), "pipelined copy out")
                cuda_ext.check(lib.eas_event_record(ev_free[s], s_out), "event_record")
            cuda_ext.check(lib.eas_stream_synchronize(s_out), "kernel execution")
            cuda_ext.check(lib.eas_stream_synchronize(s_run), "kernel execution")
        finally:
            for e in evs:
                lib.eas_event_destroy(e)
            for key, bufs in slots.items():
                for b in bufs:
                    free = self._staging.setdefault((b.device, b.nbytes), [])
                    if len(free) < 4 * R:
                        free.append(b)

    # -- pipelined host-buffer path for batched GEMMs ------------------------------------
    GEMM_PIPELINE_SLICE_BYTES = 96 << 20   # input bytes (A + B) per batch slice

    def _gemm_pipeline_plan(self, ck: Any, runtime_args: Mapping[str, Any], geo: Any) -> dict[str, Any] | None:
        """Batch slices of a batched fp16 dot GEMM on page-locked host arrays, when the pipeline
        applies: a native dot-GEMM plan whose batch is program_id(2), that stores every element of
        C (so C is never copied in), on host buffers large enough to split, with at least two
        slices."""
        native = getattr(ck.plan, "native", None)
        if native is None or not hasattr(native, "map_launch") or not hasattr(native, "covers"):
            return None
        if self._first_buffer_on_device(ck, runtime_args):
            return None
        if os.environ.get("EAS_PIPELINE", "1") in ("0", "off"):
            return None
        if os.environ.get("EAS_DISABLE_NATIVE", "0") not in ("", "0"):
            return None
        torch = _torch()
        names = [a.name for a in ck.ir.args if a.kind == "buffer"]
        if sorted(names) != sorted({native.a_arg, native.b_arg, native.c_arg}):
            return None
        hosts: dict[str, np.ndarray] = {}
        lib = self.lib()
        for n in names:
            v = runtime_args[n]
            if torch is not None and isinstance(v, torch.Tensor):
                if v.device.type != "cpu" or not v.is_contiguous():
                    return None
                v = v.detach().numpy()
            if not isinstance(v, np.ndarray) or not v.flags.c_contiguous:
                return None
            pinned = cuda_ext.ctypes.c_int(0)
            if v.nbytes == 0 or lib.eas_host_is_pinned(v.ctypes.data, cuda_ext.ctypes.byref(pinned)) or not pinned.value:
                return None
            hosts[n] = v
        if len({id(h) for h in hosts.values()}) != 3:
            return None
        (gx, gy, gz), ntx = geo
        scalars = {f"${a.name}": int(runtime_args[a.name]) for a in ck.ir.args if a.kind == "scalar"}
        m = native.map_launch(scalars, (gx, gy, gz), ntx)
        if m is None or m.get("empty") or m["batch"] < 2 or gz != m["batch"]:
            return None
        if not native.covers(runtime_args, (gx, gy, gz), ntx, native.c_arg, hosts[native.c_arg].size):
            return None
        m1 = native.map_launch(scalars, (gx, gy, 1), ntx, (0, 0, 1))  # batch 1 alone: program_id(2) is the batch
        if (m1 is None or m1.get("empty") or m1["batch"] != 1 or m1["a0"] != m["a0"] + m["a_bs"]
                or m1["b0"] != m["b0"] + m["b_bs"] or m1["c0"] != m["c0"] + m["c_bs"]):
            return None
        M, N, K = m["M"], m["N"], m["K"]
        spans = {native.a_arg: (m["a0"], m["a_bs"], (M - 1) * m["lda"] + K),
                 native.b_arg: (m["b0"], m["b_bs"], ((N - 1) * m["ldb"] + K) if m["b_kmajor"] else ((K - 1) * m["ldb"] + N)),
                 native.c_arg: (m["c0"], m["c_bs"], (M - 1) * m["ldc"] + N)}
        per_batch_in = 2 * (m["a_bs"] + m["b_bs"])
        S = max(1, self.GEMM_PIPELINE_SLICE_BYTES // max(per_batch_in, 1))
        if -(-m["batch"] // S) < 2:
            return None
        return {"hosts": hosts, "spans": spans, "batch": m["batch"], "S": S, "c": native.c_arg,
                "item": {native.a_arg: 2, native.b_arg: 2, native.c_arg: 4}}

    def _run_gemm_pipelined(self, ck: Any, runtime_args: Mapping[str, Any], geo: Any, gp: dict[str, Any]) -> None:
        """Copy-in of batch slice i+1, the GEMM of slice i and the copy-out of slice i-1 overlap on
        three streams.  Each slice runs as a program sub-range (program_id(2) in [z0, z1)) on
        slot buffers holding only its elements (pointers rebased, as run_range does), natively
        or, if the native kernel declines, with the generated kernel."""
        (gx, gy, _gz), ntx = geo
        device = self.default_device()
        lib = self.lib()
        s_in, s_run, s_out = self._streams(device)
        hosts, spans, item, S, B = gp["hosts"], gp["spans"], gp["item"], gp["S"], gp["batch"]
        R = self.PIPELINE_SLOTS
        slot_elems = {n: (S - 1) * bs + span for n, (_x0, bs, span) in spans.items()}
        slots = {n: [self._stage(device, slot_elems[n] * item[n]) for _ in range(R)] for n in spans}
        evs = []
        for _ in range(3 * R):
            e = cuda_ext.ctypes.c_void_p()
            cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e)), "event_create")
            evs.append(int(e.value))
        ev_in, ev_run, ev_free = evs[:R], evs[R:2 * R], evs[2 * R:]
        native = ck.plan.native
        try:
            for i, z0 in enumerate(range(0, B, S)):
                z1 = min(B, z0 + S)
                k = i % R
                if i >= R:
                    cuda_ext.check(lib.eas_stream_wait_event(s_in, ev_free[k]), "stream_wait_event")
                lo: dict[str, int] = {}
                for n, (x0, bs, span) in spans.items():
                    lo[n] = x0 + z0 * bs
                    if n != gp["c"]:
                        cnt = (z1 - 1 - z0) * bs + span
                        cuda_ext.check(lib.eas_copy_from_host_async(slots[n][k].ptr, hosts[n].ctypes.data + lo[n] * item[n],
                                                                    cnt * item[n], s_in), "pipelined GEMM copy in")
                cuda_ext.check(lib.eas_event_record(ev_in[k], s_in), "event_record")
                cuda_ext.check(lib.eas_stream_wait_event(s_run, ev_in[k]), "stream_wait_event")
                args = {n: _Arg(slots[n][k].ptr - lo[n] * item[n], device) for n in spans}
                if not native.try_launch(self, ck, runtime_args, args, device, s_run, (gx, gy, z1 - z0), ntx,
                                         pid_base=(0, 0, z0), elem_base=dict(lo)):
                    self._launch_generic(ck, runtime_args, args, device, s_run, (gx, gy, z1 - z0), ntx, (0, 0, z0))
                cuda_ext.check(lib.eas_event_record(ev_run[k], s_run), "event_record")
                cuda_ext.check(lib.eas_stream_wait_event(s_out, ev_run[k]), "stream_wait_event")
                c = gp["c"]
                _x0, bs, span = spans[c]
                cnt = (z1 - 1 - z0) * bs + span
                cuda_ext.check(lib.eas_copy_to_host_async(hosts[c].ctypes.data + lo[c] * item[c], slots[c][k].ptr,
                                                          cnt * item[c], s_out), "pipelined GEMM copy out")
                cuda_ext.check(lib.eas_event_record(ev_free[k], s_out), "event_record")
            cuda_ext.check(lib.eas_stream_synchronize(s_out), "kernel execution")
            cuda_ext.check(lib.eas_stream_synchronize(s_run), "kernel execution")
            self._check_native_status(device)
            self.skipped_copy_bytes += int(hosts[gp["c"]].nbytes)   # C is stored in full, never copied in
        finally:
            for e in evs:
                lib.eas_event_destroy(e)
            for bufs in slots.values():
                for b in bufs:
                    free = self._staging.setdefault((b.device, b.nbytes), [])
                    if len(free) < 4 * R:
                        free.append(b)

    def run_range(self, ck: Any, runtime_args: Mapping[str, Any], meta: Mapping[str, Any], *, axis: int,
                  lo: int, hi: int, grid: tuple[int, int, int] | None = None, nthreads: int | None = None,
                  shape: tuple[int, ...] | None = None, buffer_base: Mapping[str, int] | None = None,
                  sync: bool = True) -> None:
        """Run only programs ``lo <= program_id(axis) < hi`` of the launch ``run`` would make.

        The programs keep their global ids (the kernel's hidden program-id
        offsets), so an unmodified kernel computes exactly its share.  With
        ``buffer_base={name: e}`` buffer ``name`` holds only the elements from
        global index ``e`` on: the kernel receives its pointer moved back by
        ``e`` elements, and must only touch indices ``>= e`` in it (true for a
        program-id shard whose programs address disjoint element ranges).
        Used by :mod:`easy_as_b200.shard` to split a grid across GPUs.  A kernel with a native
        plan (fp16 dot GEMM, tiled fp32 GEMM) runs it on the sub-range when the plan applies.
        """
        geo = launch_geometry(ck, runtime_args, nthreads=nthreads, grid=grid, tptg=None, shape=shape)
        if geo is None:
            return
        programs, ntx = geo
        if not 0 <= axis <= 2:
            raise ValueError("axis must be 0, 1 or 2")
        lo, hi = max(0, int(lo)), min(int(hi), programs[axis])
        if hi <= lo:
            return
        sub = list(programs)
        sub[axis] = hi - lo
        base = [0, 0, 0]
        base[axis] = lo
        # per-array staging: a range launch may stay in flight, so no shared bounce buffer
        args, device, stream = self._resolve(ck, runtime_args, allow_bounce=False)
        for name, e in (buffer_base or {}).items():
            item = 4 if next(a for a in ck.ir.args if a.name == name).dtype == DType.F32 else 2
            args[name].ptr -= int(e) * item
        host_copies = [a for a in args.values() if a.host is not None]
        if host_copies:
            raise ValueError("run_range needs device buffers (torch CUDA tensors or eas.Tensor on cuda)")
        native = getattr(ck.plan, "native", None)
        if native is None or not native.try_launch(self, ck, runtime_args, args, device, stream, tuple(sub), ntx,
                                                   pid_base=tuple(base), elem_base=dict(buffer_base or {})):
            self._launch_generic(ck, runtime_args, args, device, stream, tuple(sub), ntx, tuple(base),
                                 dict(buffer_base or {}))
        if sync:
            cuda_ext.check(self.lib().eas_stream_synchronize(stream), "kernel execution")
            self._check_native_status(device)

    def _check_native_status(self, device: int) -> None:
        if not self.native_launches:
            return
        code = cuda_ext.ctypes.c_int()
        self.lib().eas_gemm_status(device, cuda_ext.ctypes.byref(code))
        if code.value:
            raise RuntimeError(f"native kernel on device {device} reported status {code.value} "
                               "(a bounded pipeline wait expired; results are incomplete)")

    # -- timing ---------------------------------------------------------------------------
    def benchmark_range(self, ck: Any, runtime_args: Mapping[str, Any], meta: Mapping[str, Any], *, axis: int,
                        lo: int, hi: int, repeat: int, warmup: int = 0, grid: tuple[int, int, int] | None = None,
                        nthreads: int | None = None, shape: tuple[int, ...] | None = None,
                        buffer_base: Mapping[str, int] | None = None) -> float:
        """Mean seconds per :meth:`run_range` launch of programs ``[lo, hi)`` on ``axis`` (CUDA
        events on the launch stream, after ``warmup`` launches)."""
        if repeat <= 0:
            raise ValueError("repeat must be > 0")
        kw = dict(axis=axis, lo=lo, hi=hi, grid=grid, nthreads=nthreads, shape=shape, buffer_base=buffer_base)
        for _ in range(max(warmup, 0)):
            self.run_range(ck, runtime_args, meta, sync=False, **kw)
        self.synchronize()
        _, device, stream = self._resolve(ck, runtime_args, allow_bounce=False)
        lib = self.lib()
        e0, e1 = cuda_ext.ctypes.c_void_p(), cuda_ext.ctypes.c_void_p()
        cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e0)), "event_create")
        cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e1)), "event_create")
        try:
            cuda_ext.check(lib.eas_event_record(e0, stream), "event_record")
            for _ in range(repeat):
                self.run_range(ck, runtime_args, meta, sync=False, **kw)
            cuda_ext.check(lib.eas_event_record(e1, stream), "event_record")
            cuda_ext.check(lib.eas_event_synchronize(e1), "kernel execution")
            ms = cuda_ext.ctypes.c_float()
            cuda_ext.check(lib.eas_event_elapsed_ms(e0, e1, cuda_ext.ctypes.byref(ms)), "elapsed")
        finally:
            lib.eas_event_destroy(e0)
            lib.eas_event_destroy(e1)
        self._check_native_status(device)
        return float(ms.value) * 1e-3 / repeat

    def benchmark(self, ck: Any, runtime_args: Mapping[str, Any], meta: Mapping[str, Any], *, repeat: int,
                  warmup: int = 0, nthreads: int | None = None, grid: tuple[int, int, int] | None = None,
                  tptg: tuple[int, int, int] | None = None, shape: tuple[int, ...] | None = None,
                  **_ignored: Any) -> float:
        """Mean seconds per launch over ``repeat`` launches (CUDA events), after ``warmup``."""
        _ = meta
        if repeat <= 0:
            raise ValueError("repeat must be > 0")
        if warmup < 0:
            raise ValueError("warmup must be >= 0")
        self.synchronize()
        geo = launch_geometry(ck, runtime_args, nthreads=nthreads, grid=grid, tptg=tptg, shape=shape)
        if geo is None:
            return 0.0
        args, device, stream = self._resolve(ck, runtime_args, allow_host=False)
        for _ in range(warmup):
            self._dispatch(ck, runtime_args, args, device, stream, *geo)
        lib = self.lib()
        e0, e1 = cuda_ext.ctypes.c_void_p(), cuda_ext.ctypes.c_void_p()
        cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e0)), "event_create")
        cuda_ext.check(lib.eas_event_create(cuda_ext.ctypes.byref(e1)), "event_create")
        try:
            cuda_ext.check(lib.eas_event_record(e0, stream), "event_record")
            for _ in range(repeat):
                self._dispatch(ck, runtime_args, args, device, stream, *geo)
            cuda_ext.check(lib.eas_event_record(e1, stream), "event_record")
            cuda_ext.check(lib.eas_event_synchronize(e1), "kernel execution")
            ms = cuda_ext.ctypes.c_float()
            cuda_ext.check(lib.eas_event_elapsed_ms(e0, e1, cuda_ext.ctypes.byref(ms)), "elapsed")
        finally:
            lib.eas_event_destroy(e0)
            lib.eas_event_destroy(e1)
        return float(ms.value) * 1e-3 / repeat

