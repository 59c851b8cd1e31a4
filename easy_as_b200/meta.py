"""Compile-time parameter marker (easy_as ``eas/meta.py:5-10``)."""

from __future__ import annotations


class constexpr:
    """Annotate a kernel parameter as compile-time.

    ``constexpr`` parameters are not kernel arguments: their values are bound as
    Python literals while the kernel body is traced, so they specialise the
    generated CUDA code and form part of the compile-cache key.
    """
