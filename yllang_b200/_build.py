"""In-tree build of the native parts of yllang_b200.

* libyl_kvpath.so — the C-ABI CUDA library (kernels + yl_* entry points),
  compiled by nvcc for sm_100a only; depends on the CUDA runtime, not torch.
* _C*.so — the C++17 libtorch front end (yllang::StoreKVCache, MHAKVCache,
  the batch index builder and page allocator) as a torch extension linked
  against libyl_kvpath.so.

Both land inside the package directory so that they travel with the source
tree and are the files a process loads.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libyl_kvpath.so")

CUDA_SOURCES = ["common.cu", "kv_store.cu", "index_build.cu"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> str:
    """nvcc-compile libyl_kvpath.so for sm_100a (no-op when up to date)."""
    srcs = [os.path.join(CSRC, s) for s in CUDA_SOURCES]
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(INCLUDE, "yl_kvpath.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), "-std=c++17", "-O3", *GENCODE, "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-shared", f"-I{INCLUDE}", *srcs, "-o", tmp]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def build_extension(force: bool = False, verbose: bool = False):
    """Build and import the libtorch front end (yllang_b200._C)."""
    from torch.utils import cpp_extension

    build_dir = os.path.join(PKG, "_build")
    os.makedirs(build_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "torch", "*.cpp")))
    mod = cpp_extension.load(
        name="yllang_b200_C",
        sources=srcs,
        extra_include_paths=[INCLUDE, os.path.join(CSRC, "torch")],
        extra_cflags=["-O2", "-std=c++17"],
        extra_ldflags=[f"-L{PKG}", "-lyl_kvpath", f"-Wl,-rpath,{PKG}"],
        build_directory=build_dir,
        verbose=verbose,
        with_cuda=True,
    )
    return mod


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_extension(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
