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
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
INCLUDE = os.path.join(REPO, "include")
SOURCES = [os.path.join(HERE, "csrc", "pa_decode.cu")]
HEADERS = [os.path.join(INCLUDE, "pa_decode.h"), os.path.join(HERE, "csrc", "fastdiv.h")]
OUTPUT = os.path.join(HERE, "paged_attention", "libpa_decode.so")
EXT_SOURCE = os.path.join(HERE, "csrc", "torch_ext.cpp")
EXT_OUTPUT = os.path.join(HERE, "paged_attention", "_pa_ext.so")
BUILD_DIR = os.path.join(HERE, "_build")
# pa_decode.cu compiles as parts in parallel: 0 = host API and small kernels,
# 1-4 = decode-kernel instantiations (see the PA_PART blocks in the source).
PARTS = (0, 1, 2, 3, 4)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMPILE_FLAGS = ARCH_FLAGS + [
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-diag-suppress", "177",          # constants unused by the host-only part
]
LINK_FLAGS = ARCH_FLAGS + ["-shared", "-cudart", "static"]


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


def _ext_stale() -> bool:
    if not os.path.exists(EXT_OUTPUT):
        return True
    t = os.path.getmtime(EXT_OUTPUT)
    return any(os.path.getmtime(x) > t for x in (EXT_SOURCE, HEADERS[0], OUTPUT, __file__))


def build_extension(force: bool = False, verbose: bool = False) -> str:
    """Compile the PyTorch binding ``paged_attention/_pa_ext.so`` (g++ against
    torch's headers, linked to libpa_decode.so found next to it at run time)."""
    if not force and not _ext_stale():
        return EXT_OUTPUT
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_pa_ext",
           "-DTORCH_API_INCLUDE_EXTENSION_H", f"-I{INCLUDE}", f"-I{cuda_home}/include",
           f"-I{sysconfig.get_paths()['include']}"]
    cmd += [f"-I{p}" for p in ce.include_paths()]
    cmd += [EXT_SOURCE, "-o", EXT_OUTPUT + ".tmp"]
    cmd += [f"-L{p}" for p in ce.library_paths()]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
            f"-L{os.path.dirname(OUTPUT)}", "-l:libpa_decode.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(EXT_OUTPUT + ".tmp", EXT_OUTPUT)
    return EXT_OUTPUT


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library (and the PyTorch binding) if a source is newer."""
    _build_library(force, verbose)
    build_extension(force, verbose)
    return OUTPUT


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, flush=True)


def _build_library(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUTPUT
    os.makedirs(BUILD_DIR, exist_ok=True)
    src = SOURCES[0]
    objs = [os.path.join(BUILD_DIR, f"pa_decode_part{k}.o") for k in PARTS]
    cmds = []
    for k, obj in zip(PARTS, objs):
        cmd = [_nvcc(), *COMPILE_FLAGS, f"-DPA_PART={k}", f"-I{INCLUDE}", "-c", "-o", obj, src]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        cmds.append(cmd)
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as pool:
        list(pool.map(lambda c: _run(c, verbose), cmds))
    _run([_nvcc(), *LINK_FLAGS, "-o", OUTPUT + ".tmp", *objs], verbose)
    os.replace(OUTPUT + ".tmp", OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
