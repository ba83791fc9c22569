"""Build recipe of libqasr_b200.so (sm_100a) — in-tree, so the .so travels with the repo.

    python qwen3-asr-wgpu_b200/build.py [--force]

nvcc compiles the CUDA runtime + kernels for `-gencode arch=compute_100a,code=sm_100a`
only (no PTX fallback, no other architecture); g++ compiles the host helpers with
OpenMP.  The CUDA runtime is linked statically and the driver is reached through
cudaGetDriverEntryPoint, so the library loads on a machine without a GPU driver.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_build"
LIB = PKG / "libqasr_b200.so"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-march=x86-64-v3", "-fopenmp", "-Wall"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
           "-ccbin", CXX, "-Xptxas", "-v"] + ARCH

CUDA_SOURCES = ["runtime.cu", "audio.cu"]
CXX_SOURCES = ["synth.cpp", "host_helpers.cpp", "checkpoint.cpp", "batch_decode.cpp", "session.cpp"]


def _sources_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(NVFLAGS + CXXFLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    stamp = OUT_DIR / "digest"
    digest = _sources_digest()
    if LIB.exists() and stamp.exists() and stamp.read_text() == digest and not force:
        return LIB
    objs = []
    inc = ["-I", str(INCLUDE), "-I", str(CSRC)]
    for src in CXX_SOURCES:
        obj = OUT_DIR / (src + ".o")
        cmd = [CXX, *CXXFLAGS, *inc, "-c", str(CSRC / src), "-o", str(obj)]
        _run(cmd, verbose)
        objs.append(obj)
    for src in CUDA_SOURCES:
        obj = OUT_DIR / (src + ".o")
        cmd = [NVCC, *NVFLAGS, *inc, "-c", str(CSRC / src), "-o", str(obj)]
        log = _run(cmd, verbose)
        (OUT_DIR / (src + ".ptxas.txt")).write_text(log)
        objs.append(obj)
    tmp = OUT_DIR / "libqasr_b200.so.tmp"
    cmd = [NVCC, *ARCH, "-shared", "-ccbin", CXX, "-Xcompiler", "-fopenmp", "-o", str(tmp),
           *map(str, objs), "-cudart", "static", "-lgomp"]
    _run(cmd, verbose)
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    return r.stdout


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
