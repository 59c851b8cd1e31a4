"""``@eas.autotune`` configuration objects (easy_as ``eas/autotune.py:9-57``).

The decorator only records an :class:`AutotuneSpec` on the kernel; the search
itself runs in :meth:`easy_as_b200.kernel.Kernel._autotune_select`, which times
each config with the runtime's ``benchmark`` (CUDA events on the launch stream).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Mapping, Sequence


@dataclass(frozen=True, slots=True)
class Config:
    meta: Mapping[str, Any]


@dataclass(frozen=True, slots=True)
class AutotuneSpec:
    configs: tuple[Config, ...]
    key: tuple[str, ...]
    warmup: int
    repeat: int


def autotune(*, configs: Sequence[Config], key: Sequence[str], warmup: int = 5,
             repeat: int = 25) -> Callable[[Any], Any]:
    checks = (
        (bool(configs), "autotune(configs=...) must be non-empty"),
        (bool(key), "autotune(key=...) must be non-empty"),
        (warmup >= 0, "autotune(warmup=...) must be >= 0"),
        (repeat > 0, "autotune(repeat=...) must be > 0"),
    )
    for ok, msg in checks:
        if not ok:
            raise ValueError(msg)
    spec = AutotuneSpec(tuple(configs), tuple(str(k) for k in key), int(warmup), int(repeat))

    def attach(target: Any) -> Any:
        setter = getattr(target, "_set_autotune_spec", None)
        if callable(setter):
            setter(spec)
        elif callable(target):
            target.__eas_autotune_spec__ = spec
        else:
            raise TypeError(f"@eas.autotune expects a callable or Kernel, got {type(target)!r}")
        return target

    return attach
