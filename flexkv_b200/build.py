"""In-tree build of libflexkv_b200.so (sm_100a) with nvcc.

    python -m flexkv_b200.build          # build if sources are newer
    python -m flexkv_b200.build --force  # always rebuild

The library lands in flexkv_b200/_lib/ so it travels with the source tree;
no JIT cache is involved.  `-Xptxas -v` output (registers, spills, shared
memory per kernel) is written next to it as ptxas.txt.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libflexkv_b200.so")
SOURCES = ["fkv_common.cpp", "transfer.cu", "tp_group.cpp", "xxh64.cu", "engine.cpp", "ipc.cpp", "ssd.cpp",
           "block_index.cu"]
HEADERS = [os.path.join(CSRC, "fkv_common.h"), os.path.join(REPO_DIR, "include", "flexkv_b200.h")]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, s) for s in SOURCES] + HEADERS + [os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [
        _nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-O3,-Wall", "-Xptxas", "-v", "-shared",
        "-I", os.path.join(REPO_DIR, "include"),
        "-o", tmp, *[os.path.join(CSRC, s) for s in SOURCES], "-lpthread",
    ]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(LIB_DIR, "ptxas.txt"), "w") as f:
        f.write(res.stdout)
        f.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
