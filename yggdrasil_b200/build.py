"""Build libygg_b200.so in-tree with nvcc for sm_100a (the library travels with the tree; nothing is JIT-compiled).

    python -m yggdrasil_b200.build [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libygg_b200.so"
SOURCES = [CSRC / "ygg_load.cu", CSRC / "ygg_step.cu", CSRC / "ygg_coop.cu", CSRC / "ygg_grouped.cu",
           CSRC / "ygg_float.cu"]
HEADERS = [CSRC / "ygg_model.h", CSRC / "ygg_device.cuh", ROOT / "include" / "ygg_b200.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# no --use_fast_math and no FMA contraction: every f32 op of the step is single-rounded as in the reference
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC", "-cudart", "static",
         "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile the library if a source is newer than it; returns its path."""
    if not force and not stale():
        return LIB
    objs, procs = [], []
    tmp = PKG / "_build"
    tmp.mkdir(exist_ok=True)
    for src in SOURCES:   # the translation units compile in parallel
        obj = tmp / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
        objs.append(str(obj))
    for src, p in procs:
        out, err = p.communicate()
        if p.returncode:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{out}\n{err}")
        if verbose:
            print(err, file=sys.stderr)
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.force))
