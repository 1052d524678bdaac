"""Build recipe for the sm_100a shared library ``hillserve_b200/_lib/libhsb.so``.

Plain ``nvcc`` (no PyTorch extension machinery): the library exposes only the
C ABI of ``include/hsb.h`` and links nothing but the CUDA runtime, so C, C++
and Python (ctypes) callers can all load it.  Objects are rebuilt only when a
source or header is newer than the library.

    python -m hillserve_b200.build [--force] [--verbose]
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
LIBDIR = PKG / "_lib"
OBJDIR = PKG / "_build"
LIB = LIBDIR / "libhsb.so"
COMPAT = PKG / "compat"
COMPAT_LIB = LIBDIR / "libhsb_compat.so"
CUDA_LIB = "/usr/local/cuda/lib64"
SOURCES = ["score.cu", "select.cu", "pack.cu", "attention.cu", "rehearsal.cu", "capi.cu", "noalloc.cu", "h2o.cu", "records.cu", "history.cu", "executor.cu", "synth.cu", "exchange.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libhsb.so")


def _flags() -> list[str]:
    return [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "--expt-relaxed-constexpr",
        "-Xcompiler",
        "-fPIC,-O2",
        f"-I{ROOT / 'include'}",
        f"-I{CSRC}",
    ]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    LIBDIR.mkdir(exist_ok=True)
    OBJDIR.mkdir(exist_ok=True)
    headers = [ROOT / "include" / "hsb.h", *CSRC.glob("*.cuh"), *CSRC.glob("*.h")]
    objs = []
    for src in SOURCES:
        s = CSRC / src
        if not s.exists():
            continue
        o = OBJDIR / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers]):
            cmd = [nvcc, *_flags(), "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    # The shared CUDA runtime: one runtime instance per process (PyTorch's when
    # it is loaded), so the current device and streams are the caller's.
    link = ["--cudart", "shared", f"-Xlinker=-rpath,{CUDA_LIB}"]
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", *link, "-o", str(LIB), *map(str, objs)]
        subprocess.run(cmd, check=True)
    # C++ drop-in layer over the C ABI (reference header names and classes).
    csrc = COMPAT / "compat.cpp"
    deps = [csrc, LIB, *COMPAT.rglob("*.hpp"), ROOT / "include" / "hsb.h"]
    if force or _stale(COMPAT_LIB, deps):
        cmd = [nvcc, "-std=c++17", "-O2", "-Xcompiler", "-fPIC", "-shared", "-x", "cu", *ARCH,
               f"-I{ROOT / 'include'}", f"-I{COMPAT}", str(csrc), "-o", str(COMPAT_LIB), f"-L{LIBDIR}", "-lhsb",
               *link, "-Xlinker=-rpath,$ORIGIN"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
