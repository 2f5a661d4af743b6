"""Build the sm_100a shared library ``popkv_b200/lib/libpopkv_b200.so``.

The library is plain CUDA C++ behind the C ABI in ``include/popkv_b200.h``: no
torch headers, no JIT.  It is compiled with ``-fmad=false`` so that every fp32
multiply and add is rounded separately unless the source asks for a fused
multiply-add explicitly (the popcount score is specified bit for bit).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PACKAGE / "lib"
LIB_PATH = LIB_DIR / "libpopkv_b200.so"
SOURCES = ("abi.cu", "pack.cu", "score.cu", "score_mma.cu", "topk.cu", "attention.cu", "attention_static.cu",
           "peer.cu", "retrieve.cu", "decoder.cu", "gemv.cu")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source and link the shared library (incremental objects)."""
    if not force and not _stale():
        return LIB_PATH
    obj_dir = PACKAGE / "build"
    obj_dir.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    compiler = nvcc()
    objects, commands = [], []
    for source in SOURCES:
        src = CSRC / source
        obj = obj_dir / (src.stem + ".o")
        deps = [src] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
        if force or not obj.exists() or any(d.stat().st_mtime > obj.stat().st_mtime for d in deps):
            commands.append([compiler, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src),
                             "-o", str(obj)])
        objects.append(str(obj))
    # Translation units are independent: compile them in parallel.
    workers = max(1, min(len(commands), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        for cmd in commands:
            if verbose:
                print(" ".join(cmd), flush=True)
        for result in pool.map(lambda c: subprocess.run(c, capture_output=True, text=True), commands):
            if result.stdout:
                print(result.stdout, end="", flush=True)
            if result.stderr:
                print(result.stderr, end="", file=sys.stderr, flush=True)
            if result.returncode != 0:
                raise subprocess.CalledProcessError(result.returncode, result.args)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [compiler, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objects,
           "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
