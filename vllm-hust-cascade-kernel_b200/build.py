"""Build the native libraries in-tree (no JIT cache, no pip install) through
the package's CMake project (CMakeLists.txt beside this file):

  libcascade_b200.so  -- the C ABI (include/cascade_b200.h) and all sm_100a
                         kernels; relocatable device code, static cudart.
  _C.so               -- the torch op registration (csrc/torch_ops.cpp),
                         linked against libcascade_b200.so.

Both land in cascade_kernel/lib/. Usage: python build.py [--force] [-j N] [-v]
(-v prints ptxas register / shared-memory / spill figures per kernel).
"""

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "cascade_kernel", "lib")
BUILD_DIR = os.path.join(HERE, "_build", "cmake")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")


def _run(cmd, verbose=False):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout[-8000:] + r.stderr[-8000:])
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])}")
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    return r


def build(force=False, jobs=8, verbose=False):
    import torch
    from torch.utils import cpp_extension as ce

    if force and os.path.isdir(BUILD_DIR):
        shutil.rmtree(BUILD_DIR)
    os.makedirs(BUILD_DIR, exist_ok=True)
    # the host compiler torch's extensions are built with (the system g++):
    # the torch op library throws c10 errors through libstdc++ code it shares
    # with torch, so both must use the same C++ runtime
    cxx = shutil.which("g++") or "g++"
    cfg = ["cmake", "-S", HERE, "-B", BUILD_DIR, "-G", "Ninja", "-DCMAKE_BUILD_TYPE=Release",
           f"-DCMAKE_CUDA_COMPILER={NVCC}", f"-DCMAKE_CXX_COMPILER={cxx}", f"-DCMAKE_CUDA_HOST_COMPILER={cxx}",
           "-DTORCH_INCLUDE_DIRS=" + ";".join(ce.include_paths()),
           "-DTORCH_LIB_DIR=" + ce.library_paths()[0],
           f"-DCXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    cfg.append("-DCMAKE_CUDA_FLAGS=" + ("-Xptxas=-v" if verbose else ""))
    _run(cfg)
    _run(["cmake", "--build", BUILD_DIR, "-j", str(jobs)] + (["--", "-v"] if verbose else []), verbose=verbose)
    for name in ("libcascade_b200.so", "_C.so"):
        if not os.path.exists(os.path.join(LIB_DIR, name)):
            raise RuntimeError(f"build did not produce {name}")
    return LIB_DIR


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    build(force=a.force, jobs=a.j, verbose=a.v)
    print("built", LIB_DIR)
