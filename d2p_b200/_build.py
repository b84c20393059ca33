"""In-tree build of the two native libraries of d2p_b200.

* ``libd2p_b200.so`` -- the CUDA kernels and the C ABI (include/d2p_b200.h),
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
  It has no torch dependency and can be loaded with ctypes / cgo / JNI.
* ``_C.so`` -- the torch dispatcher registration (``torch.ops.d2p.*``), a thin
  C++ layer over the C ABI, compiled with g++ against the installed torch and
  linked to ``libd2p_b200.so`` through an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Rebuilds are
skipped when the outputs are newer than every source.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libd2p_b200.so")
EXT = os.path.join(PKG, "_C.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"

CU_SOURCES = ["sw_plane.cu", "sw_wavefront.cu", "sw_linear.cu", "sw_affine_fast.cu", "sw_tangent.cu",
              "sw_affine_tangent.cu", "sw_strip.cu", "sw_nw.cu", "sw_nw_wave_tan.cu", "sw_nw_affine.cu", "sw_nw_affine_wave.cu", "sw_dtw.cu", "sw_dtw_wave.cu", "sw_embed.cu", "sw_elementwise.cu", "sw_capi.cu", "sw_noalloc.cu", "sw_selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _newer(out: str, deps) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps)


def _run(cmd, verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def build_cuda_lib(verbose: bool = False, force: bool = False, extra_flags=None) -> str:
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        os.path.join(INCLUDE, "d2p_b200.h")
    ]
    if not force and _newer(LIB, deps):
        return LIB
    cmd = [NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v" if verbose else "-O3",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-I" + INCLUDE,
           *(extra_flags or []), *srcs, "-o", LIB]
    _run(cmd, verbose)
    return LIB


def build_torch_ext(verbose: bool = False, force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "torch_bindings.cpp")
    deps = [src, os.path.join(INCLUDE, "d2p_b200.h"), LIB]
    if not force and _newer(EXT, deps):
        return EXT
    tdir = os.path.dirname(torch.__file__)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = cpp_extension.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE]
    cmd = [CXX, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *["-I" + i for i in incs], src, "-o", EXT,
           "-L" + PKG, "-ld2p_b200", "-Wl,-rpath,$ORIGIN",
           "-L" + os.path.join(tdir, "lib"), "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-Wl,-rpath," + os.path.join(tdir, "lib")]
    _run(cmd, verbose)
    return EXT


def build(verbose: bool = False, force: bool = False) -> None:
    build_cuda_lib(verbose=verbose, force=force)
    build_torch_ext(verbose=verbose, force=force)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
