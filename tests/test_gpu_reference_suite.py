"""GPU: the reference's own test files, unmodified, against this backend.

Runs where ``EAS_REFERENCE`` names a checkout of the reference (easy_as); skipped otherwise.  Each
file runs in its own pytest process with the test-only plugin ``tests/mps_alias.py``, which maps
the reference tests' Metal device names (``"mps"``) to CUDA.  Every test in the listed files must
pass; a skip counts as a failure (the reference tests skip when their device is unavailable, so a
skip would mean they did not run on the GPU).  ``import eas`` resolves to this repository's ``eas``
alias package (the process runs from the repository root)."""

from __future__ import annotations

import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import REFERENCE

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
FILES = ["test_add.py", "test_matmul.py", "test_matmul_tiled.py", "test_dot_dynamic_k.py", "test_callable_grid.py",
         "test_tptg_override.py", "test_local_and_lane_id.py", "test_threadgroup_memory.py"]


@pytest.mark.skipif(REFERENCE is None or not (REFERENCE / "tests").is_dir(),
                    reason="EAS_REFERENCE not set to a reference checkout")
@pytest.mark.parametrize("name", FILES)
def test_reference_test_file_passes(cuda_rt, name):
    path = REFERENCE / "tests" / name
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT), str(ROOT / "tests")]))
    env.pop("EAS_BACKEND", None)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "mps_alias", "-p", "no:cacheprovider",
                        "--rootdir", str(path.parent), str(path), "-rs"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    out = r.stdout[-3000:] + r.stderr[-2000:]
    assert r.returncode == 0, out
    summary = r.stdout.strip().splitlines()[-1]
    assert re.search(r"\d+ passed", summary), out
    assert "skipped" not in summary, out
