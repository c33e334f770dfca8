"""Builds libfast_moss_b200.so (sm_100a) in-tree with nvcc.

Usage: python build.py [--force]

The library is written next to the Python package
(fast_moss_b200/libfast_moss_b200.so) so that it is found without any
installation step and travels with the source tree.
"""

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "fast_moss_b200", "libfast_moss_b200.so")
SOURCES = ["capi.cu", "layer_norm.cu", "rope.cu", "gated_act.cu", "lfq.cu", "rvq.cu",
           "rvq_tc.cu", "rvq_pair.cu", "rvq_noalloc.cu", "qkv_rope.cu", "history_attn.cu", "linear.cu",
           "lfq_rvq.cu"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-rdc=true",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build fast_moss_b200")


def inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES]
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    files += [os.path.join(INCLUDE, "fast_moss_b200.h"), os.path.abspath(__file__)]
    return files


def up_to_date():
    if not os.path.exists(LIB):
        return False
    built = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= built for f in inputs())


def build(force=False, verbose=False):
    """Compiles the CUDA sources into the shared library; returns its path."""
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    cmd += ["-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed to build libfast_moss_b200.so")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=True))
