"""Build ``lib/libbayes_ssm_b200.so`` from ``csrc/`` with nvcc for sm_100a.

Usage: ``python bayes-ssm_b200/bayes_ssm/_build.py [--verbose]``.  The library
is built in-tree so that it travels with the source tree; it is rebuilt only
when a source is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
CSRC = PKG_ROOT / "csrc"
INCLUDE = PKG_ROOT.parent / "include"
LIB_DIR = PKG_ROOT / "lib"
LIB = LIB_DIR / "libbayes_ssm_b200.so"
SOURCES = ["bssm_recurrence.cu", "bssm_staged.cu", "bssm_chain.cu", "bssm_assoc_scan.cu", "bssm_check.cu",
           "bssm_envelope.cu", "bssm_d64.cu", "bssm_rotation.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    objs = []
    obj_dir = PKG_ROOT / "_build"
    obj_dir.mkdir(exist_ok=True)
    procs = []
    for src in SOURCES:  # one nvcc per translation unit, in parallel
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
               "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd)))
        objs.append(str(obj))
    failed = [src for src, proc in procs if proc.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), "-shared", *ARCH, *objs, "-o", str(tmp)], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
