// LFQ arithmetic shared by the LFQ kernels (lfq.cu) and the multi-stage
// LFQ quantizer (lfq_rvq.cu): the reference's prepare summation orders
// (fast_moss/quantizer_prepare.py:17-57) and the first-NaN / first-minimum
// selection state (fast_moss/quantizer.py:33-39).
#pragma once

#include "common.cuh"

#include <climits>

namespace moss {

// Sum of the 8 pre-rounded values v in the reference's two orders.
__device__ __forceinline__ float sum8(const float* v, bool transposed) {
  if (transposed) {
    const float a = __fadd_rn(v[0], v[4]), b = __fadd_rn(v[1], v[5]);
    const float c = __fadd_rn(v[2], v[6]), d = __fadd_rn(v[3], v[7]);
    return __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
  }
  return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                   __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
}

// Sum of squares of x: the transposed order folds channels 4..7 into the
// accumulators of 0..3 with an FMA before the serial combine.
__device__ __forceinline__ float sum_squares(const float* x, bool transposed) {
  float sq[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) sq[d] = __fmul_rn(x[d], x[d]);
  if (transposed) {
    const float a = __fmaf_rn(x[4], x[4], sq[0]);
    const float b = __fmaf_rn(x[5], x[5], sq[1]);
    const float c = __fmaf_rn(x[6], x[6], sq[2]);
    const float d = __fmaf_rn(x[7], x[7], sq[3]);
    return __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
  }
  return sum8(sq, false);
}

// Running selection state of one lane: first NaN index and first minimum.
struct Pick {
  float best;
  int64_t best_i;
  int64_t nan_i;
};

// Branch-free: a NaN distance never compares below best; selects instead of
// data-dependent branches keep the lanes of a warp converged.
__device__ __forceinline__ void pick_push(Pick& p, float dist, int64_t j) {
  const bool is_nan = dist != dist;
  const bool better = dist < p.best;
  p.nan_i = (is_nan && j < p.nan_i) ? j : p.nan_i;
  p.best_i = better ? j : p.best_i;
  p.best = better ? dist : p.best;
}

// Warp-wide reduction; every lane returns the selected index.
__device__ __forceinline__ int64_t pick_reduce(Pick p) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, p.best, m);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, p.best_i, m);
    const int64_t on = __shfl_xor_sync(0xffffffffu, p.nan_i, m);
    if (ob < p.best || (ob == p.best && oi < p.best_i)) {
      p.best = ob;
      p.best_i = oi;
    }
    if (on < p.nan_i) p.nan_i = on;
  }
  return p.nan_i != INT64_MAX ? p.nan_i : p.best_i;
}

struct Pick32 {
  float best;
  int best_i;
  int nan_i;
};

// pick_push with 32-bit indices.
__device__ __forceinline__ void pick32_push(Pick32& p, float dist, int j) {
  const bool is_nan = dist != dist;
  const bool better = dist < p.best;
  p.nan_i = (is_nan && j < p.nan_i) ? j : p.nan_i;
  p.best_i = better ? j : p.best_i;
  p.best = better ? dist : p.best;
}

__device__ __forceinline__ int pick32_reduce(Pick32 p) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, p.best, m);
    const int oi = __shfl_xor_sync(0xffffffffu, p.best_i, m);
    const int on = __shfl_xor_sync(0xffffffffu, p.nan_i, m);
    if (ob < p.best || (ob == p.best && oi < p.best_i)) {
      p.best = ob;
      p.best_i = oi;
    }
    if (on < p.nan_i) p.nan_i = on;
  }
  return p.nan_i != INT_MAX ? p.nan_i : p.best_i;
}

}  // namespace moss
