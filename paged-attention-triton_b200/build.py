"""Build the sm_100a shared library ``paged_attention/libpa_decode.so``.

The library is the C-ABI boundary declared in ``include/pa_decode.h`` (at the
repository root): plain ``extern "C"`` entry points over the CUDA kernels in
``csrc/``. It links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it loads on a machine without a GPU.

    python build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
INCLUDE = os.path.join(REPO, "include")
SOURCES = [os.path.join(HERE, "csrc", "pa_decode.cu")]
HEADERS = [os.path.join(INCLUDE, "pa_decode.h")]
OUTPUT = os.path.join(HERE, "paged_attention", "libpa_decode.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _stale() -> bool:
    if not os.path.exists(OUTPUT):
        return True
    out_t = os.path.getmtime(OUTPUT)
    return any(os.path.getmtime(s) > out_t for s in SOURCES + HEADERS + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if a source is newer than it; return its path."""
    if not force and not _stale():
        return OUTPUT
    cmd = [_nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", "-o", OUTPUT + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, flush=True)
    os.replace(OUTPUT + ".tmp", OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
