"""Builds libkvp.so in-tree for B200 (sm_100a).

    python cuda-kv-persistence_b200/build.py [--force] [--verbose]

Every csrc/*.cu and csrc/*.cpp is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into _build/, then
linked (static cudart) into kvp/_native/libkvp.so.  Host code is built with
-ffp-contract=off so the policies' float/double arithmetic matches the
reference's host build bit for bit.
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
BUILD = HERE / "_build"
OUT = HERE / "kvp" / "_native" / "libkvp.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    return shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def _flags(src: Path) -> list[str]:
    base = ["-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler",
            "-fPIC,-fvisibility=hidden,-ffp-contract=off", "-I", str(CSRC)]
    if src.suffix == ".cu":
        base += ["--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("KVP_PTXAS_V") else "-O3"]
    return base


def _deps_newer(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    if src.stat().st_mtime > t:
        return True
    headers = (list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) +
               list((HERE.parent / "include").rglob("*.h")))
    return any(h.stat().st_mtime > t for h in headers)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    OUT.parent.mkdir(parents=True, exist_ok=True)
    srcs = sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))
    objs = []
    relink = force or not OUT.exists()
    for src in srcs:
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or _deps_newer(obj, src):
            cmd = [nvcc(), "-c", str(src), "-o", str(obj), *_flags(src)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed on {src.name}")
            if verbose and r.stderr:
                sys.stderr.write(r.stderr)
            relink = True
    if relink:
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), "-shared", *ARCH, "-o", str(tmp), *map(str, objs), "-cudart", "static",
               "-Xcompiler", "-fPIC"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
