"""Test-only pytest plugin: run the reference's own test files unmodified on this backend.

The reference's device tests ask for the Metal backend by name (``get_runtime("mps")``,
``EAS_BACKEND=mps``, ``eas.tensor(..., device="mps")``, e.g. easy_as ``tests/test_add.py:24-66``).
The library refuses those names on purpose; this plugin, loaded with ``-p mps_alias`` only by
``tests/test_gpu_reference_suite.py``, maps them to CUDA for the duration of one pytest process.
It changes nothing else: the kernels, runtime and checks are the reference tests' own.
"""

from __future__ import annotations

import os


def _alias(name):
    return "cuda" if isinstance(name, str) and name.lower() in ("mps", "metal") else name


def pytest_configure(config):
    import importlib

    # by module path: the package also exports functions named `kernel` and `tensor`
    kernel_mod = importlib.import_module("easy_as_b200.kernel")
    runtime_mod = importlib.import_module("easy_as_b200.runtime")
    tensor_mod = importlib.import_module("easy_as_b200.tensor")

    orig_get = runtime_mod.get_runtime

    def get_runtime(backend=None):
        if backend is None:
            backend = _alias(os.environ.get("EAS_BACKEND", "auto"))
        return orig_get(_alias(backend))

    runtime_mod.get_runtime = get_runtime
    kernel_mod.get_runtime = get_runtime

    orig_parse = tensor_mod._parse_device

    def parse_device(device):
        return orig_parse(_alias(str(device)) if device is not None else device)

    tensor_mod._parse_device = parse_device
