"""Build ``lib/libth_b200.so`` (all CUDA kernels + the C ABI) for sm_100a.

    python torch-helion_b200/build.py [--force] [--verbose]

The library is compiled in-tree with nvcc from ``csrc/th_b200.cu`` (a unity
translation unit) so it travels with the repository snapshot.  Beside it,
``libth_b200.so.sha256`` records a SHA-256 digest of every source under
``csrc/`` and ``include/`` plus the nvcc flags it was built from.  It is
rebuilt whenever that digest differs from the current sources' (file
contents, not modification times), and the loader refuses a library whose
digest does not match, so a binary in the tree is provably built from the
sources beside it.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "lib" / "libth_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
    "-shared", "-Xcompiler", "-fPIC",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


SHA = LIB.with_name(LIB.name + ".sha256")


def source_digest() -> str:
    """SHA-256 over the sources (path and contents, sorted) and the nvcc flags."""
    h = hashlib.sha256()
    srcs = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))
    for f in srcs:
        h.update(f.name.encode() + b"\0" + f.read_bytes() + b"\0")
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def built_digest() -> str | None:
    return SHA.read_text().strip() if SHA.exists() and LIB.exists() else None


def _stale() -> bool:
    return built_digest() != source_digest()


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *( ["-Xptxas", "-v"] if verbose else []), "-o", str(tmp), str(CSRC / "th_b200.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    if verbose:
        sys.stderr.write(res.stderr)
    tmp.replace(LIB)
    SHA.write_text(source_digest() + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
