"""Build libpagedkv.so in-tree (next to this file) from csrc/*.cu for sm_100a.

The library is a plain C-ABI shared object (include/pagedkv.h): nvcc compiles
each translation unit for `-gencode arch=compute_100a,code=sm_100a`, links
against the shared CUDA runtime (so it shares the current-device state of the
PyTorch process that loads it) and needs no GPU to build.

    python pagedkv_build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libpagedkv.so"
BUILD_DIR = HERE / "_build"
SOURCES = ["capi.cu", "append.cu", "decode.cu", "prefill_tc.cu", "fused.cu", "linear_tc.cu",
           "sample.cu", "layers.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _nvcc() -> str:
    return os.environ.get("NVCC", str(CUDA_HOME / "bin" / "nvcc"))


def _flags(verbose: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "-I", str(INCLUDE), "--expt-relaxed-constexpr"]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _deps() -> list[Path]:
    return [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        list(INCLUDE.glob("*.h")) + [Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of libpagedkv.so."""
    if not force and up_to_date():
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = _nvcc()

    def compile_one(src: str) -> tuple[str, str]:
        obj = BUILD_DIR / (Path(src).stem + ".o")
        cmd = [nvcc, *_flags(verbose), "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        return str(obj), r.stdout + r.stderr

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", str(tmp), *[o for o, _ in results],
           "-Xlinker", f"-rpath,{CUDA_HOME / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
