#!/usr/bin/env python3
"""Build libg4b200.so (the C ABI of include/g4.h) for sm_100a, in-tree.

    python furiosa-opt-gemma4-12b_b200/build.py [--verbose-ptxas]

Each csrc/*.cu is compiled with nvcc (-gencode arch=compute_100a,code=sm_100a) into
_build/, then linked into g4b200/libg4b200.so next to the Python bindings.  Objects
are rebuilt only when a source or header is newer.  No GPU is needed to build.
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
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
OUT = PKG / "g4b200" / "libg4b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise SystemExit("nvcc not found")


def build(verbose_ptxas: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
            return obj
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0 or verbose_ptxas:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode != 0:
            raise SystemExit(f"nvcc failed on {src.name}")
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest_obj:
        # -Bsymbolic: calls inside the library bind to its own definitions, so another
        # library exporting the same names cannot interpose on them
        cmd = [cc, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-ldl", "-Xlinker", "-z,defs",
               "-Xlinker", "-Bsymbolic"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise SystemExit("link failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
