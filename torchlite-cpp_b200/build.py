"""Builds the native libraries of the package in-tree.

  lib/libtl_cuda.so         CUDA kernels + the C ABI (include/tlc.h), sm_100a only
  lib/libtorchlite_b200.so  the C++ tl:: layer (host/) over the C ABI
  lib/tl_tests              C++ tests of the tl:: layer (host/tests)

Usage:  python torchlite-cpp_b200/build.py [--jobs N] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
LIB = os.path.join(PKG, "lib")
OBJ = os.path.join(PKG, "lib", "obj")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-Wall",
                     "--expt-relaxed-constexpr", "-I", os.path.join(REPO, "include")]
CXX_FLAGS = ["-std=c++17", "-O3", "-fPIC", "-Wall", "-I", os.path.join(REPO, "include"),
             "-I", os.path.join(PKG, "host", "include"), "-I", "/usr/local/cuda/include"]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(jobs: int = 8, verbose: bool = False, ptxas_info: bool = False) -> dict:
    os.makedirs(OBJ, exist_ok=True)
    cu = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cuh"))) + [os.path.join(REPO, "include", "tlc.h")]
    objs = []
    jobs_list = []
    for src in cu:
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if _stale(obj, [src] + hdrs) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs_list.append(([NVCC] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]))
    logs = {}
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        futs = {ex.submit(_run, c, verbose): c[-3] for c in jobs_list}
        for f in cf.as_completed(futs):
            logs[futs[f]] = f.result()
    so = os.path.join(LIB, "libtl_cuda.so")
    if _stale(so, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", so] + objs + ["-ldl"], verbose)

    # C++ tl:: layer over the C ABI.
    host_src = sorted(glob.glob(os.path.join(PKG, "host", "src", "*.cpp")))
    host_hdr = sorted(glob.glob(os.path.join(PKG, "host", "include", "tl", "*.h")))
    tl_so = os.path.join(LIB, "libtorchlite_b200.so")
    if host_src and _stale(tl_so, host_src + host_hdr + [so]):
        _run(["g++"] + CXX_FLAGS + ["-shared", "-o", tl_so] + host_src +
             ["-L", LIB, "-ltl_cuda", "-Wl,-rpath,$ORIGIN"], verbose)
    test_src = sorted(glob.glob(os.path.join(PKG, "host", "tests", "*.cpp")))
    test_bin = os.path.join(LIB, "tl_tests")
    if test_src and _stale(test_bin, test_src + host_hdr + [tl_so]):
        _run(["g++"] + CXX_FLAGS + ["-UNDEBUG", "-o", test_bin] + test_src +
             ["-L", LIB, "-ltorchlite_b200", "-ltl_cuda", "-Wl,-rpath,$ORIGIN"], verbose)
    # The reference callers' scenarios on the device tl:: layer
    # (tests/integration/device_callers_main.cpp, compared with the reference
    # by tests/test_reference_callers.py).
    dc_src = os.path.join(REPO, "tests", "integration", "device_callers_main.cpp")
    dc_bin = os.path.join(LIB, "tl_device_callers")
    if os.path.exists(dc_src) and _stale(dc_bin, [dc_src] + host_hdr + [tl_so]):
        _run(["g++"] + CXX_FLAGS + ["-o", dc_bin, dc_src, "-L", LIB, "-ltorchlite_b200", "-ltl_cuda",
              "-Wl,-rpath,$ORIGIN"], verbose)
    return logs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    logs = build(a.jobs, a.verbose, a.ptxas_info)
    if a.ptxas_info:
        for k, v in logs.items():
            print(f"== {k}\n{v}")
    print("built", os.path.join(LIB, "libtl_cuda.so"))


if __name__ == "__main__":
    sys.exit(main())
