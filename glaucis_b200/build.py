"""Builds libglaucis_b200.so in-tree with nvcc for sm_100a (B200).

The library is a plain C-ABI shared object (see include/glaucis_b200.h); it
links the CUDA runtime statically and reaches the driver's tensor-map encoder
through cudaGetDriverEntryPoint, so it needs no -lcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libglaucis_b200.so"

SOURCES = ["capi.cu", "quant.cu", "gmm_fp8.cu", "chunk_gla.cu", "chunk_gla_bwd.cu",
           "gla_intermediates.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _deps() -> list[Path]:
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every .cu for sm_100a and links the shared library."""
    if not force and up_to_date():
        return LIB
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)

    def compile_one(src: str):
        obj = BUILD / (Path(src).stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, obj, r

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    logs = []
    for src, _, r in results:
        logs.append(f"== {src}\n{r.stdout}{r.stderr}")
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}{r.stderr}")
    (BUILD / "ptxas.log").write_text("\n".join(logs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *[str(o) for _, o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print("\n".join(logs))
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
