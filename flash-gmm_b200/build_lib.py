"""Build libflashgmm_sm100.so in-tree with nvcc for sm_100a.

    python flash-gmm_b200/build_lib.py          # build if sources changed
    python flash-gmm_b200/build_lib.py --force  # rebuild

The library is a plain C-ABI shared object (include/flashgmm.h); it links the
CUDA runtime statically and needs no torch headers.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_NAME = "libflashgmm_sm100.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def nvcc_path() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in sources() + headers())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if not force and not needs_build():
        return LIB_PATH
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    common = [nvcc_path(), *NVCC_ARCH, "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", os.path.join(ROOT, "include"),
              *extra]
    objs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = common + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    link = [nvcc_path(), *NVCC_ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    args = sys.argv[1:]
    extra = [a for a in args if a.startswith("-X") or a.startswith("--resource")]
    print(build(force="--force" in args, verbose="-v" in args, extra=extra))
