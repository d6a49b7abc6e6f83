"""Build the native library in-tree: blackflash_b200/lib/libblackflash_b200.so.

The library is plain CUDA C++ compiled by nvcc for sm_100a only (no torch
headers), so it builds in seconds and loads through ctypes from Python or
through the C ABI (include/blackflash_b200.h) from any other host language.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libblackflash_b200.so")
HARNESS_PATH = os.path.join(LIB_DIR, "flash_attn")
# The torch-extension module `blackflash_cuda`, built at the repository root so that
# `import blackflash_cuda` resolves as it does for the reference's installed extension.
EXT_SRC = os.path.join(CSRC, "torch_ext.cpp")

SOURCES = ["fa_fwd_sm100.cu", "capi.cu", "lse_merge.cu", "noalloc.cu", "ring_ipc.cu"]
HEADERS = ["sm100_ptx.cuh", "fa_fwd_sm100.h", "fa_fwd_sm100_d128.cuh", "fa_bwd_sm100.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", os.path.join(REPO_DIR, "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build blackflash_b200")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)


def build_lib(force: bool = False, verbose: bool = False) -> str:
    """Compile libblackflash_b200.so if any source is newer than it; return its path."""
    os.makedirs(LIB_DIR, exist_ok=True)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps += [os.path.join(REPO_DIR, "include", f) for f in ("blackflash_b200.h", "blackflash_b200_diag.h", "flash_attn.cuh")]
    if force or _stale(LIB_PATH, deps):
        tmp = LIB_PATH + ".tmp"
        cmd = [_nvcc(), *ARCH, *COMMON, "-shared", "-o", tmp, *[os.path.join(CSRC, f) for f in SOURCES]]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_harness(force: bool = False, verbose: bool = False) -> str:
    """Compile the standalone ref_data harness (csrc/harness.cu) against the library."""
    lib = build_lib(force=force, verbose=verbose)
    src = os.path.join(CSRC, "harness.cu")
    if force or _stale(HARNESS_PATH, [src, lib]):
        cmd = [_nvcc(), *ARCH, *COMMON, "-o", HARNESS_PATH, src, "-L", LIB_DIR, "-lblackflash_b200",
               f"-Xlinker=-rpath,{LIB_DIR}", "-Xlinker=-rpath,$ORIGIN"]
        _run(cmd, verbose)
    return HARNESS_PATH


def ext_path() -> str:
    import sysconfig
    return os.path.join(REPO_DIR, "blackflash_cuda" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile the `blackflash_cuda` torch extension (csrc/torch_ext.cpp, g++ against the
    installed torch headers) linked to libblackflash_b200.so; return its path."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension
    lib = build_lib(force=force, verbose=verbose)
    out = ext_path()
    deps = [EXT_SRC, lib, os.path.join(REPO_DIR, "include", "blackflash_b200.h")]
    if not (force or _stale(out, deps)):
        return out
    cuda_home = cpp_extension.CUDA_HOME or "/usr/local/cuda"
    incs = cpp_extension.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"],
                                                               os.path.join(cuda_home, "include")]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch.compiled_with_cxx11_abi())
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-DTORCH_EXTENSION_NAME=blackflash_cuda",
           *[f"-I{i}" for i in incs], EXT_SRC, "-o", out + ".tmp",
           f"-L{LIB_DIR}", "-lblackflash_b200", "-Wl,-rpath,$ORIGIN/blackflash_b200/lib",
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           ]
    _run(cmd, verbose)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build_lib(force="--force" in sys.argv, verbose=True))
    if os.path.exists(os.path.join(CSRC, "harness.cu")):
        print(build_harness(force="--force" in sys.argv, verbose=True))
    print(build_torch_ext(force="--force" in sys.argv, verbose=True))
