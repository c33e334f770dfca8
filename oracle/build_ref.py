"""Builds oracle/_ref/libref_prepare.so from the reference's own kernel source.

TEST INFRASTRUCTURE.  The reference's LFQ preparation kernel is CUDA C++
held as the string SOURCE in fast_moss/quantizer_prepare.py:16-58.  This
recipe reads that string from the reference checkout (it is not copied into
this repository), prepends a small host shim (IEEE round-to-nearest
stand-ins for __fadd_rn / __fmul_rn / __fdiv_rn / __fsqrt_rn / __fmaf_rn and
a blockIdx/threadIdx launch loop) and compiles it with g++ -ffp-contract=off,
feeding the source through stdin.  The only output is the shared library in
oracle/_ref/ (git-ignored), used to pin oracle.lfq_prepare.

Usage: python oracle/build_ref.py [--reference /path/to/reference]
(default: $FAST_MOSS_REFERENCE, else `reference` beside the repository root)
"""

import argparse
import ast
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libref_prepare.so")
# The reference checkout: $FAST_MOSS_REFERENCE, else a directory named
# `reference` beside this repository's root.
DEFAULT_REFERENCE = os.environ.get(
    "FAST_MOSS_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

SHIM = r"""
#include <cmath>
#define __device__
#define __global__
#define __forceinline__ inline
struct moss_dim3 { int x; };
static moss_dim3 blockIdx, blockDim, threadIdx;
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __fdiv_rn(float a, float b) { return a / b; }
static inline float __fsqrt_rn(float a) { return std::sqrt(a); }
static inline float __fmaf_rn(float a, float b, float c) { return std::fma(a, b, c); }
"""

DRIVER = r"""
extern "C" __attribute__((visibility("default")))
void ref_prepare(const float* x, float* e, float* norm, float* twice, float* denom,
                 int batch, int time) {
  const int rows = batch * time;
  blockDim.x = 128;
  for (int blk = 0; blk * 128 < rows; ++blk) {
    for (int th = 0; th < 128; ++th) {
      blockIdx.x = blk;
      threadIdx.x = th;
      quantizer_prepare(x, e, norm, twice, denom, batch, time);
    }
  }
}
"""


def reference_source(reference):
    path = os.path.join(reference, "fast_moss", "quantizer_prepare.py")
    tree = ast.parse(open(path).read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id == "SOURCE" for t in node.targets
        ):
            return ast.literal_eval(node.value)
    raise RuntimeError(f"SOURCE not found in {path}")


def build(reference=DEFAULT_REFERENCE, force=False):
    """Compiles the reference kernel for the host; returns the .so path or
    None when the reference checkout is absent."""
    if not os.path.isdir(reference):
        return OUT if os.path.exists(OUT) else None
    src_file = os.path.join(reference, "fast_moss", "quantizer_prepare.py")
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(src_file):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    program = SHIM + reference_source(reference) + DRIVER
    tmp = OUT + f".{os.getpid()}.tmp"
    subprocess.run(
        ["g++", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-x", "c++",
         "-", "-o", tmp],
        input=program.encode(), check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default=DEFAULT_REFERENCE)
    args = parser.parse_args()
    out = build(args.reference, force=True)
    if out is None:
        sys.exit(f"reference not found at {args.reference}")
    print(out)
