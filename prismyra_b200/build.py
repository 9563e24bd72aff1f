"""Build the sm_100a shared library ``prismyra_b200/libprismyra_moe.so`` from ``prismyra_b200/csrc/*.cu``.

Plain nvcc, no torch extension machinery: the library exports only the C ABI of ``include/prismyra_moe.h``.
``python -m prismyra_b200.build`` (or ``__graft_entry__.build()``) compiles it in-tree so it travels with the
checkout to the GPU host.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libprismyra_moe.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build prismyra_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [PKG.parent / "include" / "prismyra_moe.h"]
    return any(p.stat().st_mtime > t for p in deps if p.is_file())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not stale():
        return LIB
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
        "-I", str(PKG.parent / "include"), "-o", str(LIB) + ".tmp",
        *[str(s) for s in sources()],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building prismyra_b200")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force=True))
