"""Build the reference's own CUDA extension as a checker: ``oracle/_ref/popkv_ext_ref*.so``.

Test infrastructure, not product.  The reference binds its kernels through a
torch extension compiled at first use from two files (``csrc/popkv_ext.cpp``
and ``csrc/popkv_ext.cu``, loaded by ``popkv_cuda._extension``,
popkv_cuda.py:14-25, with ``-O3`` for the host code and ``-O3
--use_fast_math`` for the device code).  This recipe compiles those two files
where they lie in a reference checkout, with those flags plus torch's standard
extension flags, for sm_100a, and links them against the torch libraries of
this image.  Nothing of the reference is copied: the sources are read in
place and only the built module goes to ``oracle/_ref/`` (git-ignored; it
travels to a GPU box like the package's own library).

On the GPU box the module is imported by path (``load_reference_extension``)
by the parity tests and by ``bench.py --impl reference`` to time the
reference's own kernels beside ours.  Its functions are the reference's:
``pack_dim``, ``pack_into_dim``, ``query_encode_out``, ``score_encoded``,
``score_dim`` and the rest of ``csrc/popkv_ext.cpp:39-52``.

Usage: ``python oracle/build_ref.py [REFERENCE_CHECKOUT]`` (default: the
``POPKV_REFERENCE`` environment variable).
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "popkv_ext_ref"


def module_path() -> Path:
    return OUT_DIR / (MODULE + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build(reference: str | os.PathLike | None = None, verbose: bool = False) -> Path:
    """Compile the reference's extension; returns the module path (skips an up-to-date build)."""
    import pybind11
    import torch
    from torch.utils import cpp_extension as ext

    root = Path(reference or os.environ.get("POPKV_REFERENCE", ""))
    cu, cpp = root / "csrc" / "popkv_ext.cu", root / "csrc" / "popkv_ext.cpp"
    if not cu.exists() or not cpp.exists():
        raise FileNotFoundError(f"reference sources not found under {root}/csrc")
    out = module_path()
    if out.exists() and out.stat().st_mtime > max(cu.stat().st_mtime, cpp.stat().st_mtime, Path(__file__).stat().st_mtime):
        return out
    OUT_DIR.mkdir(exist_ok=True)
    cuda_home = Path(ext.CUDA_HOME or "/usr/local/cuda")
    includes = [f"-I{p}" for p in ext.include_paths(device_type="cuda")]
    includes += [f"-I{sysconfig.get_paths()['include']}", f"-I{pybind11.get_include()}"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    defines = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H", abi]
    cu_obj, cpp_obj = OUT_DIR / "popkv_ext.cu.o", OUT_DIR / "popkv_ext.cpp.o"
    commands = [
        [str(cuda_home / "bin" / "nvcc"), "-c", str(cu), "-o", str(cu_obj), *includes, *defines,
         *ext.COMMON_NVCC_FLAGS, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
         "-Xcompiler", "-fPIC", "-O3", "--use_fast_math"],
        ["g++", "-c", str(cpp), "-o", str(cpp_obj), *includes, *defines, "-std=c++17", "-fPIC", "-O3"],
    ]
    with ThreadPoolExecutor(max_workers=2) as pool:
        for cmd, res in zip(commands, pool.map(lambda c: subprocess.run(c, capture_output=True, text=True),
                                               commands)):
            if verbose:
                print(" ".join(cmd), flush=True)
            if res.returncode != 0:
                raise RuntimeError(f"reference extension build failed:\n{' '.join(cmd)}\n{res.stderr[-4000:]}")
    libs = [f"-L{p}" for p in ext.library_paths(device_type="cuda")]
    link = ["g++", "-shared", str(cpp_obj), str(cu_obj), "-o", str(out), *libs, "-lc10", "-lc10_cuda",
            "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"]
    if verbose:
        print(" ".join(link), flush=True)
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference extension link failed:\n{res.stderr[-4000:]}")
    for obj in (cu_obj, cpp_obj):  # only the module travels to the GPU host
        obj.unlink(missing_ok=True)
    return out


def load_reference_extension():
    """Import the built reference extension (torch must be importable); None if not built."""
    path = module_path()
    if not path.exists():
        return None
    import torch  # noqa: F401  (the module links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(MODULE, str(path))
    spec = importlib.util.spec_from_file_location(MODULE, str(path), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
