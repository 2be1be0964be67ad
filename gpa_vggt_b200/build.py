"""Build the sm_100a shared library ``libgpa_b200.so`` in-tree with nvcc.

The library exposes the C ABI declared in ``include/gpa_b200.h``.  It is built
for ``sm_100a`` only (B200); nvcc cross-compiles it without a GPU present.

    python -m gpa_vggt_b200.build          # build if sources changed
    python -m gpa_vggt_b200.build --force  # rebuild
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libgpa_b200.so"
OBJ = PKG / "_build"
HEADER = ROOT / "include" / "gpa_b200.h"

SOURCES = ["merge.cu", "sim_argmax.cu", "attention.cu", "frame.cu", "norm.cu", "dpt.cu", "proj.cu",
           "exchange.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [HEADER]
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source (one nvcc per file, in parallel) and link
    them into one shared library (in-tree)."""
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    objs = [OBJ / (Path(s).stem + ".o") for s in SOURCES]
    jobs = [[nvcc, *NVCC_FLAGS, "-c", "-o", str(o), str(CSRC / s)] for s, o in zip(SOURCES, objs)]
    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
          *[str(o) for o in objs]], verbose)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
