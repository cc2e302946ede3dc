"""Build libmxfa_b200.so in-tree with nvcc for sm_100a.

    python -m mxflashattn_b200.build        # or __graft_entry__.build()

The library is a plain C-ABI shared object (static CUDA runtime, no torch
types), written next to this file so it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB_NAME = "libmxfa_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)
SOURCES = ["capi.cu"]
HEADERS = ["common.cuh", "decode.cuh", "prefill_sm100.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(REPO, "include", "mxfa_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    mtime = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= mtime for f in _inputs() if os.path.exists(f))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    extra = os.environ.get("MXFA_NVCC_EXTRA", "").split()
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra, "-o", tmp, *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose and proc.stderr:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
