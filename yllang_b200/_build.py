"""In-tree build of the native parts of yllang_b200.

* libyl_kvpath.so — the C-ABI CUDA library (kernels + yl_* entry points),
  compiled by nvcc for sm_100a only; depends on the CUDA runtime, not torch.
* libyl_attention.so — flashinfer's paged decode / causal prefill kernels
  (third-party, compiled from the headers flashinfer ships) behind a
  torch-free interface, for the front end's Attention layer.
* _C*.so — the C++17 libtorch front end (yllang::StoreKVCache, MHAKVCache,
  the batch index builder, page allocator and Attention) as a Python
  extension linked against libtorch, libyl_kvpath.so and libyl_attention.so.

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

CUDA_SOURCES = ["common.cu", "kv_store.cu", "index_build.cu", "kv_step.cu", "gather.cu", "qkv_store.cu",
                "page_alloc.cu", "ranges.cu"]
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


ATTN_LIB = os.path.join(PKG, "libyl_attention.so")


def _flashinfer_data() -> str:
    """Source headers shipped inside the installed flashinfer package (its
    own include tree, and the CCCL / CUTLASS trees it vendors)."""
    import importlib.util
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or spec.origin is None:
        raise RuntimeError("flashinfer is not installed: the attention layer compiles its kernels from its headers")
    return os.path.join(os.path.dirname(spec.origin), "data")


def build_attention(force: bool = False, verbose: bool = False) -> str:
    """nvcc-compile libyl_attention.so: flashinfer's paged decode and causal
    paged prefill kernels for sm_100a behind csrc/torch/attention_fi.h (no
    torch dependency; used by the front end's Attention)."""
    src = os.path.join(CSRC, "torch", "attention_fi.cu")
    noalloc = os.path.join(CSRC, "torch", "attention_noalloc.cu")
    deps = [src, noalloc, os.path.join(CSRC, "torch", "attention_fi.h"), os.path.join(INCLUDE, "yl_attention.h")]
    if not force and not _stale(ATTN_LIB, deps):
        return ATTN_LIB
    fi = _flashinfer_data()
    tmp = ATTN_LIB + ".tmp"
    cmd = [_nvcc(), "-std=c++17", "-O3", *GENCODE, "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler",
           "-fPIC,-fvisibility=hidden", "-shared", f"-I{fi}/cccl/libcudacxx/include", f"-I{fi}/include",
           f"-I{fi}/cutlass/include", f"-I{fi}/spdlog/include", f"-I{INCLUDE}", "-diag-suppress=20012,177,550",
           src, noalloc, "-o", tmp]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, ATTN_LIB)
    return ATTN_LIB


def _ext_path() -> str:
    import sysconfig
    return os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_extension(force: bool = False, verbose: bool = False) -> str:
    """g++-compile the libtorch front end into yllang_b200/_C*.so, linked
    against libyl_kvpath.so (found next to it at run time via $ORIGIN)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    out = _ext_path()
    tdir = os.path.join(CSRC, "torch")
    srcs = sorted(glob.glob(os.path.join(tdir, "*.cpp")))
    deps = srcs + glob.glob(os.path.join(tdir, "*.h")) + [os.path.join(INCLUDE, "yl_kvpath.h")]
    attn = build_attention(force=force, verbose=verbose)
    if not force and not _stale(out, deps + [attn]):
        return out
    build_dir = os.path.join(PKG, "_build")
    os.makedirs(build_dir, exist_ok=True)
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = getattr(cpp_extension, "_get_pybind11_abi_build_flags", lambda: [])()
    cflags = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden",
              f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
              "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", *abi,
              f"-I{INCLUDE}", f"-I{tdir}", f"-I{sysconfig.get_paths()['include']}", f"-I{cuda_home}/include"]
    cflags += [f"-I{p}" for p in cpp_extension.include_paths()]
    objs, procs = [], []
    for src in srcs:
        obj = os.path.join(build_dir, os.path.basename(src) + ".o")
        objs.append(obj)
        procs.append(subprocess.Popen(["g++", *cflags, "-c", src, "-o", obj]))
    if any(p.wait() != 0 for p in procs):
        raise RuntimeError("compiling the libtorch front end failed")
    build_library()
    tmp = out + ".tmp"
    subprocess.run(["g++", "-shared", *objs, "-o", tmp, f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu",
                    "-ltorch_python", "-lc10_cuda", "-ltorch_cuda", f"-L{PKG}", "-lyl_kvpath", "-lyl_attention",
                    "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"], check=True)
    os.replace(tmp, out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_extension(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
