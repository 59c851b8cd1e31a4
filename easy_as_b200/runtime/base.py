"""Runtime protocol shared by the CUDA runtime and test doubles (easy_as ``eas/runtime/base.py:9-24``)."""

from __future__ import annotations

from collections.abc import Mapping
from typing import Any, Protocol


class Runtime(Protocol):
    def is_available(self) -> bool: ...

    def run(self, ck: Any, runtime_args: Mapping[str, Any], meta: Mapping[str, Any], *,
            sync: bool = True, nthreads: int | None = None, grid: tuple[int, int, int] | None = None,
            tptg: tuple[int, int, int] | None = None, shape: tuple[int, ...] | None = None) -> None: ...

    def synchronize(self) -> None: ...
