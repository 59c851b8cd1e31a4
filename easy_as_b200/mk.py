"""Kernel-language primitives (``eas.mk``), trace-only.

Every function records one instruction into the tracer that is active on this
thread; none of them computes anything.  The operator set of :class:`val`
is the reference's (easy_as ``eas/mk.py:37-85``): ``+ * // % < & | ~`` and
their reflected forms.  There is deliberately no ``-``, ``/`` or ``>``.
"""

from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass
from typing import Any, Iterator

from .ir import DType, ValueRef


class _TraceState(threading.local):
    builder: Any = None


_state = _TraceState()


@contextlib.contextmanager
def _trace(builder: Any) -> Iterator[None]:
    saved = _state.builder
    _state.builder = builder
    try:
        yield
    finally:
        _state.builder = saved


def _b() -> Any:
    if _state.builder is None:
        raise RuntimeError("eas.mk is only valid inside an @eas.kernel trace/launch")
    return _state.builder


def _binary(method: str, reflected: bool = False):
    if reflected:
        return lambda self, other: getattr(_b(), method)(other, self)
    return lambda self, other: getattr(_b(), method)(self, other)


@dataclass(frozen=True, slots=True)
class val:
    """A traced SSA value."""

    ref: ValueRef

    @property
    def dtype(self) -> DType:
        return self.ref.dtype

    __add__ = _binary("add")
    __radd__ = _binary("add", True)
    __mul__ = _binary("mul")
    __rmul__ = _binary("mul", True)
    __floordiv__ = _binary("floordiv")
    __rfloordiv__ = _binary("floordiv", True)
    __mod__ = _binary("mod")
    __rmod__ = _binary("mod", True)
    __lt__ = _binary("lt")
    __and__ = _binary("and_")
    __rand__ = _binary("and_", True)
    __or__ = _binary("or_")
    __ror__ = _binary("or_", True)

    def __invert__(self) -> "val":
        return _b().not_(self)


# ---- ids -----------------------------------------------------------------
def program_id(axis: int) -> val:
    return _b().program_id(axis)


def local_id(axis: int) -> val:
    return _b().local_id(axis)


def lane_id() -> val:
    return _b().lane_id()


def sg_id() -> val:
    return _b().sg_id()


def arange(start: int, size: int) -> val:
    """Lane vector ``start .. start+size-1`` of one program (SPMD mode)."""
    return _b().arange(start, size)


def tid(start: int, size: int) -> val:
    """Per-thread local index; ``size`` is the threads per block (thread mode)."""
    return _b().tid(start, size)


# ---- block-shared memory ---------------------------------------------------
def alloc_tg(size: int) -> val:
    return _b().alloc_tg(size)


def alloc_tg_f16(size: int) -> val:
    return _b().alloc_tg(size, dtype=DType.F16)


def barrier() -> None:
    _b().barrier()


# ---- memory and arithmetic -------------------------------------------------
def load(buffer: Any, offset: Any, mask: Any | None = None) -> val:
    return _b().load(buffer, offset, mask)


def store(buffer: Any, offset: Any, value: Any, mask: Any | None = None) -> None:
    _b().store(buffer, offset, value, mask)


def where(cond: Any, a: Any, b: Any) -> val:
    return _b().where(cond, a, b)


def fma(a: Any, b: Any, c: Any) -> val:
    return _b().fma(a, b, c)


def to_f32(x: Any) -> val:
    return _b().cast(x, DType.F32)


def to_f16(x: Any) -> val:
    return _b().cast(x, DType.F16)


def to_u32(x: Any) -> val:
    return _b().cast(x, DType.U32)


def and_(a: Any, b: Any) -> val:
    return _b().and_(a, b)


def or_(a: Any, b: Any) -> val:
    return _b().or_(a, b)


def not_(x: Any) -> val:
    return _b().not_(x)


# ---- contractions ----------------------------------------------------------
def dot(a_buffer: Any, a_base: Any, a_stride: Any, b_buffer: Any, b_base: Any,
        b_stride: Any, K: Any) -> val:
    """f32 sum over ``k < K`` of ``a[a_base + k*a_stride] * b[b_base + k*b_stride]``."""
    return _b().dot(a_buffer, a_base, a_stride, b_buffer, b_base, b_stride, K)


def mma_zero() -> val:
    return _b().mma_zero()


def mma(a_buffer: Any, a_base: Any, a_stride: Any, b_buffer: Any, b_base: Any,
        b_stride: Any, acc: Any) -> val:
    """Warp-cooperative 8x8x8 multiply-accumulate into an 8x8 f32 fragment."""
    return _b().mma(a_buffer, a_base, a_stride, b_buffer, b_base, b_stride, acc)


def mma_store(buffer: Any, base: Any, stride: Any, frag: Any) -> None:
    _b().mma_store(buffer, base, stride, frag)
