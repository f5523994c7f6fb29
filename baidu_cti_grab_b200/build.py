"""Build the sm_100a CUDA library (librep_b200.so) in-tree with nvcc.

    python -m baidu_cti_grab_b200.build [--force] [--verbose]

The library is one translation unit (csrc/rep_b200_all.cu) compiled for
``-gencode arch=compute_100a,code=sm_100a``; nvcc cross-compiles it on a
machine without a GPU.  The result sits next to this file so that it travels
with the source tree.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_NAME = "librep_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
MAIN_SRC = os.path.join(HERE, "csrc", "rep_b200_all.cu")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def sources() -> list:
    srcs = glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh"))
    srcs.append(os.path.join(REPO, "include", "rep_b200.h"))
    return sorted(srcs)


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile librep_b200.so if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, MAIN_SRC]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stderr or "") + (res.stdout or "")
        raise RuntimeError(f"nvcc failed building {LIB_NAME}:\n{msg}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
