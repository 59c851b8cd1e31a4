"""Runtime selection.

There is one backend, CUDA on sm_100a.  ``EAS_BACKEND`` accepts ``auto`` and
``cuda``; the reference's names for its GPU backend (``mps``/``metal``) are
refused with a message, and ``cpu`` is refused as in the reference
(easy_as ``eas/runtime/__init__.py:18-44``): there is no CPU fallback.
"""

from __future__ import annotations

import os
from typing import Any

from .base import Runtime

__all__ = ["get_runtime", "Runtime"]

_cuda: Any = None


def _cuda_runtime() -> Any:
    global _cuda
    if _cuda is None:
        from .cuda import CudaRuntime

        _cuda = CudaRuntime()
    return _cuda


# the process environment as CPython keeps it (bytes keys and values on POSIX): a lookup there costs
# a dict access, against about 0.7 us for os.environ.get, and sees every os.environ change
_ENV_DATA = getattr(os.environ, "_data", None)
if _ENV_DATA is not None and not all(type(k) is bytes for k in list(_ENV_DATA)[:1]):
    _ENV_DATA = None   # not the POSIX layout: use os.environ


def env_bytes(key: bytes) -> bytes | None:
    """The raw value of environment variable ``key`` (bytes), or None; for the launch path."""
    if _ENV_DATA is not None:
        return _ENV_DATA.get(key)
    v = os.environ.get(key.decode())
    return None if v is None else v.encode()


def get_runtime(backend: str | None = None) -> Runtime:
    if backend is None and _cuda is not None and _cuda._available:
        raw = env_bytes(b"EAS_BACKEND")
        if raw is None or raw in (b"auto", b"cuda", b"AUTO", b"CUDA"):
            return _cuda  # launch-path shortcut: already probed and available
    name = (backend or os.environ.get("EAS_BACKEND", "auto")).lower()
    if name in ("auto", "cuda") and _cuda is not None and _cuda._available:
        return _cuda  # launch-path shortcut: already probed and available
    if name in ("auto", "cuda"):
        rt = _cuda_runtime()
        if not rt.is_available():
            raise RuntimeError("CUDA runtime is not available: " + rt.unavailable_reason()
                               + ". Build the native library with `python -m easy_as_b200.build`.")
        return rt
    if name == "cpu":
        raise ValueError("unsupported backend: 'cpu' (there is no CPU runtime; use 'cuda' or 'auto')")
    if name in ("mps", "metal"):
        raise ValueError(f"unsupported backend: {name!r} (this build targets CUDA sm_100a; use 'cuda' or 'auto')")
    raise ValueError(f"unsupported backend: {name!r} (expected 'auto'|'cuda')")
