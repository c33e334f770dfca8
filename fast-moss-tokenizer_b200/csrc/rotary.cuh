// Rotary-embedding arithmetic shared by the RoPE kernels and the fused
// qkv projection: the position offset as float32, and one rotated pair with
// every product and sum rounded (fast_moss/v2_pointwise.py:8-47).
#pragma once

#include "common.cuh"

namespace moss {

__device__ __forceinline__ float offset_as_float(const void* p, int dtype, int64_t b) {
  if (dtype == 0) return static_cast<float>(static_cast<const int64_t*>(p)[b]);
  if (dtype == 1) return static_cast<float>(static_cast<const int32_t*>(p)[b]);
  return static_cast<const float*>(p)[b];
}

__device__ __forceinline__ void rotate_pair(float qr, float qj, float c, float s, float& o0,
                                            float& o1) {
  o0 = __fsub_rn(__fmul_rn(qr, c), __fmul_rn(qj, s));
  o1 = __fadd_rn(__fmul_rn(qr, s), __fmul_rn(qj, c));
}

}  // namespace moss
