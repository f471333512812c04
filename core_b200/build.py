"""Build the CUDA library ``core_b200/libcore_b200.so`` for sm_100a with nvcc.

Usage:  python -m core_b200.build   (or core_b200.build.build())
Sources: core_b200/csrc/*.cu; public header: include/core_b200.h.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SRC = PKG / "csrc"
OUT = PKG / "libcore_b200.so"
BUILD = ROOT / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-diag-suppress", "177",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build core_b200")
    return cand


def sources():
    return sorted(SRC.glob("*.cu"))


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every .cu file and link the shared library; returns its path."""
    srcs = sources()
    deps = srcs + list(SRC.glob("*.cuh")) + list(SRC.glob("*.h")) + [ROOT / "include" / "core_b200.h"]
    if OUT.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if OUT.stat().st_mtime >= newest:
            return OUT
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    procs = []
    for s in srcs:
        obj = BUILD / (s.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(s), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for s, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((s, out.decode(errors="replace")))
        elif verbose and out:
            print(out.decode(errors="replace"))
    if failed:
        msg = "\n".join(f"--- {s.name}\n{o}" for s, o in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp),
           *map(str, objs), "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
