"""Build libeas_cuda.so in-tree with nvcc for sm_100a.

Run ``python -m easy_as_b200.build``.  The library lands in
``easy_as_b200/_lib/libeas_cuda.so`` so that it ships with the source tree
(no site-packages install, no JIT cache).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libeas_cuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _flags(ptxas_verbose: bool = False) -> list[str]:
    return [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
            *(["-Xptxas", "-v"] if ptxas_verbose else [])]


def source_hash() -> str:
    """sha256 over every source and header the library is built from, and the nvcc flags."""
    import hashlib

    h = hashlib.sha256()
    deps = sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "eas_cuda.h"]
    for p in deps:
        if p.exists():
            h.update(p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    h.update(" ".join(_flags()).encode())
    return h.hexdigest()


STAMP = LIB.with_name(LIB.name + ".sha256")


def needs_build() -> bool:
    """Rebuild unless the library exists and its stamp (written beside it by the build that made it)
    matches the current sources and flags; file times play no part."""
    if not LIB.exists() or not STAMP.exists():
        return True
    return STAMP.read_text().strip() != source_hash()


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    digest = source_hash()
    cmd = [nvcc(), *_flags(ptxas_verbose), "-I", str(PKG.parent / "include"), "-I", str(CSRC),
           *map(str, sources()), "-o", str(tmp), "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    STAMP.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    print(build(verbose=True, force="--force" in args, ptxas_verbose="-v" in args))
