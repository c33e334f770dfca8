// Shared helpers for the fast_moss_b200 kernels (sm_100a).
//
// Every floating-point operation whose rounding matters is written with an
// explicit round-to-nearest intrinsic (__fadd_rn, __fmul_rn, __fmaf_rn, ...).
// Those are never contracted into a multiply-add, so the arithmetic is fixed
// by the source and not by the compiler.  The library is built with nvcc's
// default --fmad=true so that calls to the CUDA math library (expf, cosf,
// sinf, rsqrtf) compile exactly as they do inside PyTorch's own kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/fast_moss_b200.h"

namespace moss {

// ---------------------------------------------------------------- host errors
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
// Converts the pending launch error (if any) into MOSS_ERR_CUDA.
int launch_status(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device-side error word: bounded waits and range checks record a code here
// instead of trapping, so that the context stays usable.
extern __device__ int g_device_error;

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// ---------------------------------------------------------------- dtypes
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) {
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

template <int DT>
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i) {
  if constexpr (DT == MOSS_F32) {
    return static_cast<const float*>(p)[i];
  } else {
    return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
  }
}

template <int DT>
__device__ __forceinline__ void store_from_f32(void* p, int64_t i, float v) {
  if constexpr (DT == MOSS_F32) {
    static_cast<float*>(p)[i] = v;
  } else {
    static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
  }
}

// Rounds a float32 value to the storage dtype and back (one torch op output).
template <int DT>
__device__ __forceinline__ float round_to(float v) {
  if constexpr (DT == MOSS_F32) {
    return v;
  } else {
    return bf16_bits_to_f32(f32_to_bf16_bits(v));
  }
}

// Unpacks 8 bf16 values held in a 16-byte vector.
__device__ __forceinline__ void unpack_bf16x8(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[i] = static_cast<uint32_t>(f32_to_bf16_bits(f[2 * i])) |
           (static_cast<uint32_t>(f32_to_bf16_bits(f[2 * i + 1])) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Multiprocessor count of the current device (cached per device).
int sm_count();

}  // namespace moss
