"""GPU: the reference's own test files, unmodified, against this backend.

Runs where ``EAS_REFERENCE`` names a checkout of the reference (easy_as); skipped otherwise.  Each
file runs in its own pytest process with the test-only plugin ``tests/mps_alias.py``, which maps
the reference tests' Metal device names (``"mps"``) to CUDA.  Every test in the listed files must
pass; a skip counts as a failure (the reference tests skip when their device is unavailable, so a
skip would mean they did not run on the GPU).  Five tests of those files check the text of the
generated Metal source (``ck.msl`` must contain MSL syntax such as ``threadgroup float v1[256];``,
``[[thread_position_in_threadgroup]]`` or ``packed_float4``); this backend generates CUDA C++, so
they are deselected by name and listed in ``MSL_TEXT``.  ``import eas`` resolves to this repository's ``eas``
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
MSL_TEXT = ["test_packed_float4_emitted_for_dot_group", "test_msl_contains_for_loop", "test_msl_declares_hidden_params",
            "test_msl_contains_threadgroup_alloc_and_barrier", "test_barrier_not_in_mask_guard"]
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
                        "--rootdir", str(path.parent), str(path), "-rs",
                        "-k", " and ".join(f"not {t}" for t in MSL_TEXT)],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    out = r.stdout[-3000:] + r.stderr[-2000:]
    assert r.returncode == 0, out
    summary = r.stdout.strip().splitlines()[-1]
    assert re.search(r"\d+ passed", summary), out
    assert "skipped" not in summary, out
