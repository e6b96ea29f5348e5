"""Build libvqmoe.so in-tree with nvcc for sm_100a (B200).

    python -m knurlogic_b200.build [-v]

The library is plain CUDA C++ with a C ABI (include/vqmoe.h); it links only
the CUDA runtime, so the same .so serves ctypes, cgo or any other FFI.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libvqmoe.so"
SOURCES = ("router.cu", "expert.cu", "expert_prefill.cu", "expert_ref.cu", "dense_prefill.cu", "block.cu",
           "layout.cu", "noalloc.cu", "tp_reduce.cu", "decoder.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"),
              "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [
        ROOT / "include" / "vqmoe.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(ROOT / "include"),
           "-o", str(LIB), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
    if r.returncode:
        raise RuntimeError(f"nvcc failed ({r.returncode}) building {LIB.name}")
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(LIB)
