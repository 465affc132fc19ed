"""Build the in-tree C-ABI library ``libdrofell_w4a16.so`` for sm_100a with nvcc.

    python -m drofell_for_revision_b200.build [--verbose] [--ptxas-info]

Objects go to ``_build/`` at the repository root; the shared library is written
next to this file so it travels with the package.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_NAME = "libdrofell_w4a16.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = [
    "w4a16_capi.cu",
    "w4a16_dequant.cu",
    "w4a16_gemv.cu",
    "w4a16_gemv_mma.cu",
    "w4a16_gemm_sm100.cu",
    "w4a16_gemm_ns.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fvisibility=hidden"]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found")
    return found


def _compile(src: str, ptxas_info: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if ptxas_info or verbose:
        sys.stdout.write(res.stderr)
    return obj


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_mtime = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f != "w4a16_torch.cpp"]
    deps.append(os.path.join(ROOT, "include", "drofell_w4a16.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > lib_mtime for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link the shared library. Returns its path."""
    if not force and not ptxas_info and not _stale():
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, ptxas_info, verbose), SOURCES))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


TORCH_EXT = os.path.join(PKG_DIR, "_w4a16_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
TORCH_SRC = os.path.join(CSRC, "w4a16_torch.cpp")


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    """The torch fast path of the forward (csrc/w4a16_torch.cpp), compiled with g++
    against torch's headers and linked to libdrofell_w4a16.so next to it. Returns its path."""
    deps = [TORCH_SRC, os.path.join(ROOT, "include", "drofell_w4a16.h"), LIB_PATH]
    if not force and os.path.exists(TORCH_EXT) and all(os.path.getmtime(d) <= os.path.getmtime(TORCH_EXT)
                                                       for d in deps):
        return TORCH_EXT
    import torch
    from torch.utils import cpp_extension as ce
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = 1 if torch.compiled_with_cxx11_abi() else 0
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", TORCH_SRC, "-o", TORCH_EXT + ".tmp",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_w4a16_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{sysconfig.get_paths()['include']}",
           f"-I{os.path.join(cuda_home, 'include')}",
           *[f"-L{p}" for p in ce.library_paths()], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", f"-L{PKG_DIR}", "-ldrofell_w4a16", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"torch extension build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(TORCH_EXT + ".tmp", TORCH_EXT)
    return TORCH_EXT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    print(build_torch_ext(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
