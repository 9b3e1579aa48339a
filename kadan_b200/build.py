"""Build libkadan_b200.so in-tree for sm_100a with nvcc.

The library holds every CUDA kernel and the C ABI declared in
include/kadan_b200.h. It is built next to this file so it travels with the
repository snapshot to the GPU machine.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
LIB = HERE / "libkadan_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-diag-suppress",
    "177",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the kadan_b200 CUDA library cannot be built")
    return path


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + sorted((ROOT / "include").rglob("*.h*"))


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources() + headers())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    objdir = ROOT / "_build" / "kadan_b200"
    objdir.mkdir(parents=True, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = objdir / (src.name + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if src.suffix == ".cpp":
            cmd = [nvcc(), *FLAGS, "-x", "cu", *ARCH, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    errors = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode:
            errors.append(f"{src.name}:\n{out.decode(errors='replace')}")
        elif verbose and out:
            print(out.decode(errors="replace"), file=sys.stderr)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart", "-lcuda"]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
