"""Build the native parts of mps_deform_conv in-tree.

1. ``mps_deform_conv/lib/libdcn_b200.so`` -- the CUDA kernels and the C ABI of
   ``include/dcn_b200.h``, compiled by nvcc for sm_100a only.
2. ``mps_deform_conv/lib/libdcn_b200_bounds.so`` -- the same sources with
   ``-DDCN_DEBUG_BOUNDS``: the gather and scatter index math is checked
   against each tensor's extent and violations are recorded
   (``dcn_debug_bounds_read``); for tests, not for production.
3. ``mps_deform_conv/_C*.so`` -- the thin PyTorch extension that mirrors the
   reference's pybind11 module ``_C`` and calls the C ABI.

Usage:  python mps-deform-conv_b200/build.py [--force] [--no-bounds]
Every step is incremental (skipped when outputs are newer than sources).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
import sysconfig

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
PKG = os.path.join(PKG_ROOT, "mps_deform_conv")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libdcn_b200.so")
BOUNDS_LIB = os.path.join(LIBDIR, "libdcn_b200_bounds.so")
BUILD = os.path.join(PKG_ROOT, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-v",
]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(home, "bin", "nvcc")


def _stale(out: str, deps) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False, bounds: bool = False) -> str:
    """Compile and link libdcn_b200.so, or with `bounds` libdcn_b200_bounds.so."""
    out = BOUNDS_LIB if bounds else LIB
    bdir = os.path.join(BUILD, "bounds") if bounds else BUILD
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    if not force and not _stale(out, deps):
        return out
    os.makedirs(bdir, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    objs = []
    logs = []
    for s in srcs:
        o = os.path.join(bdir, os.path.basename(s) + ".o")
        cmd = [_nvcc(), *NVCC_FLAGS, *(["-DDCN_DEBUG_BOUNDS"] if bounds else []), "-I", INCLUDE, "-I", CSRC,
               "-c", s, "-o", o]
        r = subprocess.run(cmd, capture_output=True, text=True)
        logs.append(r.stdout + r.stderr)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"nvcc failed on {s}")
        objs.append(o)
    with open(os.path.join(bdir, "ptxas.log"), "w") as f:
        f.write("\n".join(logs))
    if verbose:
        print("\n".join(logs))
    # Export only the extern "C" symbols (dcn_*); the CUDA runtime is linked statically.
    cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
           *objs, "-o", out, "-Xlinker", "--exclude-libs,ALL"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    return out


def build_ext(force: bool = False) -> str:
    """Build the torch extension _C (C++ only; links libdcn_b200.so)."""
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "ext_C.cpp")
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = os.path.join(PKG, "_C" + suffix)
    if not force and not _stale(out, [src, LIB, os.path.join(INCLUDE, "dcn_b200.h")]):
        return out
    import torch

    bdir = os.path.join(BUILD, "ext")
    os.makedirs(bdir, exist_ok=True)
    abi = int(torch.compiled_with_cxx11_abi())
    incs = [INCLUDE, sysconfig.get_paths()["include"], *ce.include_paths(device_type="cuda")]
    libs = ce.library_paths(device_type="cuda")
    tmp = os.path.join(bdir, "_C" + suffix)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", src, "-o", tmp,
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-fvisibility=hidden",
           *[f"-I{p}" for p in incs], *[f"-L{p}" for p in libs],
           f"-L{LIBDIR}", "-ldcn_b200", "-Wl,-rpath,$ORIGIN/lib",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("extension build failed")
    shutil.copy2(tmp, out)
    return out


def build_all(force: bool = False, verbose: bool = False, bounds: bool = True) -> None:
    build_lib(force=force, verbose=verbose)
    if bounds:
        build_lib(force=force, bounds=True)
    build_ext(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv, bounds="--no-bounds" not in sys.argv)
    print("built", LIB)
