"""Build libqik.so (the C-ABI CUDA library) in-tree for sm_100a.

    python qwen-image-kernel_b200/build.py [--force] [--verbose-ptxas]

Each .cu under csrc/ is compiled by nvcc to an object (in csrc/_build/) and linked
into qik/libqik.so with the CUDA runtime linked statically, so the library has no
dependency beyond the driver.  Objects are rebuilt when their source or any header
is newer.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = CSRC / "_build"
INCLUDE = HERE.parent / "include"
OUT = HERE / "qik" / "libqik.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas",
         "-warn-spills", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    objs = []
    changed = force or not OUT.exists()
    for src in sorted(CSRC.glob("*.cu")):
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
                and obj.stat().st_mtime >= newest_header):
            continue
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd[1:1] = ["-Xptxas", "-v"]
        print("[qik build]", " ".join(cmd[-4:]), flush=True)
        subprocess.run(cmd, check=True)
        changed = True
    if changed:
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(OUT), *map(str, objs)]
        print("[qik build] link", OUT.name, flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose_ptxas))
    sys.exit(0)
