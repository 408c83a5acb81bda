"""Build recipe for the native parts of torch_vulkan_b200.

Produces, in this package directory (both git-ignored, both shipped with the source tree):
  libb2rt.so   the C-ABI library (include/b2rt.h): runtime, slab allocator, every CUDA kernel,
               compiled with nvcc for sm_100a only (-gencode arch=compute_100a,code=sm_100a);
  _b2ops.so    the ATen operator shim (csrc/shim/ops.cpp), linked against libb2rt.so and libtorch.

Incremental: an object is rebuilt when its source or any header under csrc/ or include/ is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = os.path.join(HERE, "libb2rt.so")
OPS = os.path.join(HERE, "_b2ops.so")


def _headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build_lib(verbose=False, jobs=None):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "runtime", "*.cu")) + glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    hdrs = _headers()
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.relpath(s, CSRC).replace(os.sep, "_") + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                   "-Xptxas", "-v" if verbose else "-O3", "-I", os.path.join(ROOT, "include"), "-c", s, "-o", o]
            todo.append(cmd)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for out in ex.map(_run, todo):
                if verbose and out:
                    print(out)
    if _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xlinker", "--exclude-libs,ALL"])
    return LIB


def build_ops(verbose=False):
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "shim", "ops.cpp")
    if not _stale(OPS, [src, LIB] + _headers()):
        return OPS
    inc = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_b2ops"]
    for i in inc:
        cmd += ["-isystem", i]
    cmd += [src, "-o", OPS, f"-L{HERE}", "-lb2rt", "-Wl,-rpath,$ORIGIN"]
    for d in libdirs:
        if "torch" in d:
            cmd += [f"-L{d}", f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    _run(cmd)
    return OPS


def build_all(verbose=False):
    build_lib(verbose=verbose)
    build_ops(verbose=verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built", LIB, OPS)
