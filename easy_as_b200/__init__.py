"""easy_as_b200: the easy_as kernel DSL on NVIDIA B200 (CUDA sm_100a).

Public API (same names as the reference package ``eas``):
``kernel``, ``Kernel``, ``constexpr``, ``autotune``, ``Config``, ``mk``,
``Tensor``, ``tensor``, ``empty``, ``empty_like``, ``from_dlpack``,
``to_dlpack``, ``from_torch``, ``to_torch``.  ``import eas`` resolves to this
package (see the top-level ``eas`` shim), so existing kernels run unchanged.
"""

from __future__ import annotations

from . import mk  # noqa: F401
from .autotune import Config, autotune
from .dlpack import from_dlpack, to_dlpack
from .kernel import Kernel, kernel
from .meta import constexpr
from .tensor import Tensor, empty, empty_like, tensor
from .torch import from_torch, to_torch

__all__ = [
    "Config", "Kernel", "Tensor", "autotune", "constexpr", "from_dlpack", "empty", "empty_like",
    "from_torch", "kernel", "mk", "tensor", "to_dlpack", "to_torch",
]
