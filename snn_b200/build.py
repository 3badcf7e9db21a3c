"""Builds snn_b200/_lib/libsnn_b200.so (sm_100a) in-tree with nvcc.

    python -m snn_b200.build            # build if sources changed
    python -m snn_b200.build --force    # rebuild everything

cudart is linked statically (nvcc's default), so the library does not depend
on which libcudart the host process (e.g. PyTorch) already loaded. NCCL is the
one the installed PyTorch uses (the nvidia-nccl wheel), found through an
rpath, so a process that also runs torch.distributed loads a single NCCL.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libsnn_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: no FMA contraction anywhere (the reference's bit-parity rule,
# CMakeLists.txt:57-60); the kernels also use explicitly rounded intrinsics.
NVCC_FLAGS = ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC,-Wall",
              "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def nccl_dirs() -> tuple[str, str]:
    """Include and lib directory of the NCCL that PyTorch links."""
    cands = []
    for p in sys.path:
        cands.append(os.path.join(p, "nvidia", "nccl"))
    for d in cands:
        inc, lib = os.path.join(d, "include"), os.path.join(d, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and glob.glob(os.path.join(lib, "libnccl.so*")):
            return inc, lib
    if os.path.exists("/usr/include/nccl.h"):
        return "/usr/include", "/usr/lib/x86_64-linux-gnu"
    raise RuntimeError("nccl.h not found")


def _newer(src_files, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in src_files)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                     glob.glob(os.path.join(ROOT, "include", "*.h")))
    inc, lib = nccl_dirs()
    cc = nvcc()
    incs = ["-I", os.path.join(ROOT, "include"), "-I", CSRC, "-I", inc]

    def compile_one(src):
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        if force or _newer([src] + headers, obj):
            cmd = [cc, *ARCH, *NVCC_FLAGS, *incs, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if force or _newer(objs, LIB):
        nccl_so = sorted(glob.glob(os.path.join(lib, "libnccl.so*")))[0]
        cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs,
               "-L", lib, "-l:" + os.path.basename(nccl_so), "-Xlinker", "-rpath," + lib]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
