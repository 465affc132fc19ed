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
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
