"""Build the native libraries in-tree (no JIT cache, no pip install).

  libcascade_b200.so  -- the C ABI (include/cascade_b200.h) and all sm_100a
                         kernels; nvcc, relocatable device code, static cudart.
  _C.so               -- the torch op registration (csrc/torch_ops.cpp),
                         linked against libcascade_b200.so.

Both land in cascade_kernel/lib/. Usage: python build.py [--force] [-j N]
"""

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "cascade_kernel", "lib")
OBJ_DIR = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["capi.cu", "paged_decode.cu", "prefix_tc.cu", "combine.cu", "lse_merge.cu", "gateup.cu", "noalloc.cu",
              "rms_norm.cu", "roofline_probe.cu"]
HEADERS = ["ptx.cuh", "kernels.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-rdc=true",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", INCLUDE, "-I", CSRC,
]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {os.path.basename(cmd[-1])}")
    return r


def build_capi(force=False, jobs=8, verbose=False):
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "cascade_b200.h")]
    objs, todo = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            todo.append([NVCC] + NVCC_FLAGS + ["-Xptxas", "-v"] * verbose + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for r in ex.map(_run, todo):
            if verbose:
                sys.stderr.write(r.stderr)
    lib = os.path.join(LIB_DIR, "libcascade_b200.so")
    if force or todo or _newer(lib, objs):
        _run([NVCC, "-shared", "-rdc=true", "-gencode", "arch=compute_100a,code=sm_100a",
              "-Xcompiler", "-fPIC", *objs, "-o", lib])
    return lib


def build_torch_ext(force=False):
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    lib = os.path.join(LIB_DIR, "libcascade_b200.so")
    out = os.path.join(LIB_DIR, "_C.so")
    if not force and not _newer(out, [src, lib, os.path.join(INCLUDE, "cascade_b200.h")]):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = []
    for p in ce.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE]:
        inc += ["-I", p]
    tlib = ce.library_paths()[0]
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", *inc, src, "-o", out,
           "-L", LIB_DIR, "-lcascade_b200", "-L", tlib, "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + tlib]
    _run(cmd)
    return out


def build(force=False, jobs=8, verbose=False):
    build_capi(force=force, jobs=jobs, verbose=verbose)
    build_torch_ext(force=force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    build(force=a.force, jobs=a.j, verbose=a.v)
    print("built", LIB_DIR)
