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

// ---------------------------------------------------------------- bounded waits
// Every spin in these kernels (on an mbarrier phase, a copy or an MMA) goes
// through bounded_wait: it polls until `poll()` is true, and after
// `limit_ns` of %globaltimer time gives up, records MOSS_ERR_TIMEOUT in the
// device error word and returns false.  The caller then stops issuing work,
// waits (bounded again) for its own copies in flight, frees what it holds
// and returns, so no kernel traps or hangs.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // ~2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

template <typename Poll>
__device__ __forceinline__ bool bounded_wait(Poll poll, uint64_t limit_ns = kWaitLimitNs) {
  if (poll()) return true;
  const uint64_t start = global_ns();
  while (!poll()) {
    if (global_ns() - start > limit_ns) {
      record_device_error(MOSS_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
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
// Two float32 values rounded (nearest even) to bf16 and packed, lo in the
// low half: the same rounding as one scalar conversion per value.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// Packed bf16 arithmetic, one correctly rounded (nearest even) result per
// half.  The sum of two bf16 values rounds to the same bf16 value as the
// float32 sum rounded to bf16 (the float32 sum is exact whenever the
// exponents differ by at most 15; otherwise both round to the larger
// operand).  The same holds for the product whenever its magnitude is at
// least 2^-125; below that the float32 product can be inexact, so callers
// recompute results whose exponent field is 0 or 1.
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// True when either half has a biased exponent of 0 or 1 (|v| < 2^-125).
__device__ __forceinline__ bool bf16x2_tiny(uint32_t v) {
  return (v & 0x7f00u) == 0u || (v & 0x7f000000u) == 0u;
}

// Division of numerators n < 2^31 by a run-time constant d >= 1 with one
// multiply-high and two shifts (Granlund & Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994): with
// l = ceil(log2 d) and m = ceil(2^(31+l) / d) < 2^32,
// floor(n / d) = floor(m n / 2^(31+l)) = umulhi(m, 2n) >> l.
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const unsigned long long m = ((1ull << (31 + l)) + d - 1) / d;
  return FastDiv{d, static_cast<uint32_t>(m), l};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return __umulhi(f.m, n << 1) >> f.l;
}

// Multiprocessor count of the current device (cached per device).
int sm_count();

// Raises the dynamic shared memory limit of `kernel` on the current device
// once; `done` is the caller's per-kernel flag array indexed by device.
constexpr int kMaxDevices = 64;
template <typename K>
inline void allow_dynamic_smem(K kernel, size_t bytes, bool* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  if (!done[dev]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(bytes));
    done[dev] = true;
  }
}

// Blocks of `threads` threads of `kernel` that are resident on the whole
// device at once (a persistent grid), capped at `work` and at least 1.
template <typename K>
inline int64_t persistent_grid(K kernel, int threads, size_t shmem, int64_t work) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, shmem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t grid = static_cast<int64_t>(sm_count()) * per_sm;
  if (grid > work) grid = work;
  return grid < 1 ? 1 : grid;
}

}  // namespace moss
