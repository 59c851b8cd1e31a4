import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

import eas  # noqa: E402,F401  (registers the `eas` alias before tests import kernels)

# a checkout of the reference (easy_as), only where EAS_REFERENCE names one; tests that read it skip otherwise
_REF_ENV = os.environ.get("EAS_REFERENCE", "")
REFERENCE = Path(_REF_ENV) if _REF_ENV else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_rt():
    from easy_as_b200.runtime import _cuda_runtime

    rt = _cuda_runtime()
    if not rt.is_available():
        pytest.fail("GPU test on a box without a usable CUDA runtime: " + rt.unavailable_reason())
    return rt
