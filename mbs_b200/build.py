"""Build libmbs_gemm_kernel.so (the C-ABI kernel library) in-tree with nvcc.

    python -m mbs_b200.build [--force]

The library is compiled for sm_100a only and links the CUDA runtime
dynamically, so it shares the process's libcudart (and therefore the current
device and streams) with PyTorch when both are loaded.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
REPO = os.path.dirname(PKG_DIR)
LIB_NAME = "libmbs_gemm_kernel.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
# Debug variant with per-role cycle counters (-DMBS_TIMING=1, mbs_timing_read()).
TIMING_LIB_PATH = os.path.join(PKG_DIR, "libmbs_gemm_kernel_timing.so")
SOURCES = ["common.cu", "quant.cu", "gemm.cu", "probe.cu", "ipc.cu"]
HEADERS = ["common.h", "ptx.cuh", "mx_quant.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin/ on PATH")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(REPO, "include", "mbs_gemm_a4w4.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date(path: str = LIB_PATH) -> bool:
    if not os.path.exists(path):
        return False
    t = os.path.getmtime(path)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, timing: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    path = TIMING_LIB_PATH if timing else LIB_PATH
    if not force and up_to_date(path):
        return path
    cuda_home = os.path.dirname(os.path.dirname(_nvcc()))
    tmp = path + ".tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "shared",
           "-Xlinker", f"-rpath,{os.path.join(cuda_home, 'lib64')}",
           "-I", os.path.join(REPO, "include"),
           "-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    if timing:
        cmd.insert(1, "-DMBS_TIMING=1")
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, cwd=CSRC, capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stderr or "") + (res.stdout or "")
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{msg}")
    os.replace(tmp, path)
    return path


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                timing="--timing" in sys.argv))
