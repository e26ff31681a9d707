"""Build libw8a8.so in-tree with nvcc for sm_100a.

    python -m imagine_b200.build          # incremental
    python -m imagine_b200.build --force  # rebuild everything

The library is a plain C-ABI shared object (include/w8a8.h) linked against the
static CUDA runtime, so it loads without PyTorch and without a JIT cache.
Objects go to imagine_b200/_build/ (git-ignored); the .so sits next to this
file so that it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libw8a8.so")

SOURCES = ["api.cu", "quantize.cu", "convrot.cu", "gemm_sm100.cu", "gemm_splitk_static.cu", "gemv.cu",
           "mxfp8.cu", "rope.cu", "sampler.cu"]
HEADERS = ["sm100_ptx.cuh", "epilogue.cuh", "quant_common.cuh", "w8a8_internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS] + \
        [os.path.join(ROOT, "include", "w8a8.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= _newest(deps):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-c",
           os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            if f.endswith(".o"):
                os.remove(os.path.join(BUILD, f))
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart=static", "-o", tmp, *objs,
               "-Xlinker", "--no-undefined", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


SHIM = os.path.join(PKG, "libimagine_kitchen_w8a8.so")


def build_shim(force: bool = False) -> str:
    """The imagine_kitchen_call front end (csrc/kitchen_shim.cpp): compiled with
    g++ against the LibTorch headers of the installed torch (the at::Tensor
    handles the reference's crate passes), linked to libw8a8.so by rpath."""
    import torch

    src = os.path.join(CSRC, "kitchen_shim.cpp")
    fwd = os.path.join(CSRC, "kitchen_forward.cpp")
    deps = [src, fwd, os.path.join(CSRC, "kitchen_forward.h"), os.path.join(ROOT, "include", "w8a8.h"),
            LIB]
    if not force and os.path.exists(SHIM) and os.path.getmtime(SHIM) >= _newest(deps):
        return SHIM
    tdir = os.path.dirname(torch.__file__)
    tinc = os.path.join(tdir, "include")
    tlib = os.path.join(tdir, "lib")
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = SHIM + ".tmp"
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-fvisibility=hidden",
           "-I", tinc, "-I", os.path.join(tinc, "torch", "csrc", "api", "include"), "-I", cuda_inc,
           src, fwd, "-o", tmp, "-L", PKG, "-l:libw8a8.so", "-L", tlib, "-lc10", "-lc10_cuda",
           "-ltorch_cpu", "-ldl",
           f"-Wl,-rpath,$ORIGIN:{tlib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"kitchen shim build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, SHIM)
    return SHIM


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_shim(force=a.force))
