"""Builds libplamo_cuda.so (sm_100a) in-tree: plamo3-0.8b-runtime_b200/lib/libplamo_cuda.so.

nvcc cross-compiles without a GPU, so this runs on the CPU build host; the built library travels
with the source tree to the GPU machine. Object files are cached under _build/ and rebuilt when
their source or any header changed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libplamo_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no implicit multiply-add contraction; every fused multiply-add in the kernels is an
# explicit fmaf, so the CPU restatement can reproduce the arithmetic bit for bit.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]
SOURCES = ["kernels.cu", "gemm.cu", "gemm_tc.cu", "attn_tc.cu", "attn_mma.cu", "sampler.cu", "decode_mega.cu", "runtime.cu", "kernel_api.cu", "loader.cpp", "packer.cpp"]


def nvcc() -> str:
    for cand in [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")]:
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler_flags():
    # nvcc picks the first g++ on PATH; /usr/bin/g++ is the system toolchain with full libstdc++.
    gxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else shutil.which("g++")
    return ["-ccbin", gxx] if gxx else []


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, extra_flags=None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    cc = nvcc()
    host = _host_compiler_flags()
    flags = NVCC_FLAGS + (extra_flags or [])
    objs, changed = [], False
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if _stale(obj, src):
            changed = True
            lang = ["-x", "cu"] if name.endswith(".cu") else []
            cmd = [cc, *host, *ARCH, *flags, *lang, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if changed or not LIB.exists():
        cmd = [cc, *host, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB), "-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
