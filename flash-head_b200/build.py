"""Build the FlashHead CUDA library in-tree for sm_100a.

    python flash-head_b200/build.py [--verbose] [--ptxas-info]

Produces ``flash-head_b200/flash_head/libflashhead_b200.so`` from
``csrc/flashhead.cu`` with nvcc (static CUDA runtime, so the library loads
with or without torch in the process). Rebuilds only when a source is newer
than the library unless ``force`` is set.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG_ROOT), "include")
LIB_PATH = os.path.join(PKG_ROOT, "flash_head", "libflashhead_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build the library)")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo",
           "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3", "-shared", "-cudart", "static",
           "-I", INCLUDE, "-o", tmp, os.path.join(CSRC, "flashhead.cu"), "-lrt", "-ldl",
           "-lpthread"]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force or args.ptxas_info, verbose=args.verbose,
                ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
