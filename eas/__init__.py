"""``import eas`` for kernels written against the reference package.

This module replaces itself in ``sys.modules`` with :mod:`easy_as_b200` and
registers every submodule under the ``eas.`` prefix too, so that
``from eas import mk``, ``import eas.runtime.grid`` or
``mock.patch("eas.kernel.get_runtime")`` all reach the same module objects.
"""

import importlib
import sys

import easy_as_b200 as _pkg

for _name in ("ir", "mk", "meta", "autotune", "analysis", "compiler", "kernel", "tensor", "dlpack", "torch",
              "codegen", "codegen.cuda", "codegen.patterns", "runtime", "runtime.base", "runtime.grid",
              "runtime.cuda", "runtime.cuda_ext", "shard"):
    try:
        _mod = importlib.import_module(f"easy_as_b200.{_name}")
    except ModuleNotFoundError:
        continue
    sys.modules[f"eas.{_name}"] = _mod

sys.modules[__name__] = _pkg
