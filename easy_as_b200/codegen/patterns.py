"""Recognise IR shapes that map onto hand-written native kernels.

``match_native(ir, lowered)`` returns a plan object with a
``try_launch(runtime, ck, runtime_args, args, device, stream, programs, ntx)``
method, or None.  A plan launches its native kernel only when the runtime
values fit it and returns False otherwise, in which case the generic
NVRTC-compiled kernel runs; both compute the same IR semantics.
"""

from __future__ import annotations

from typing import Any

from ..ir import IRModule


def match_native(ir: IRModule, lowered: Any) -> Any:
    return None
