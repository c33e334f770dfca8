// Activation formulas shared by the gated-activation kernels and the
// Linear epilogue: the float32 arithmetic of torch's eager silu / gelu
// (erf) / gelu (tanh), so both produce the bits of the eager chain.
#pragma once

#include "common.cuh"

namespace moss {

// silu(v) = v / (1 + expf(-v)) when only its bf16 rounding is kept.
//
// Fast form: e^-v = 2^th * 2^tl with th = v * L rounded and tl the rest of
// v * -log2(e) (one FMA gives v * L - th exactly, a second adds v times the
// tail of the constant), so e = ex2.approx(th) * (1 + ln2 tl) carries the
// error of ex2.approx (taken as 2^-21.5) and one rounding, independent of
// |v|; q = v * rcp.approx(1 + e) adds two roundings and the 2^-23 of
// rcp.approx.  That is within 11 units in the last place of q; the float32
// value torch computes (expf within 2 ulp, two roundings) is within 6 of
// the exact quotient, so the two round to the same bf16 value unless the
// fast quotient's low 16 bits lie within 32 units of the rounding midpoint
// 0x8000.  Those cases, |v| > 64 (where 1 + e or its reciprocal could leave
// the normal range) and |v| < 2^-100 (zero, subnormal or NaN v) take the
// exact torch formula.  The input is itself a bf16 value, so the exhaustive
// test over all 65536 inputs checks the claim on the hardware.
__device__ __forceinline__ float silu_exact(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
}

__device__ __forceinline__ float silu_fast(float v, bool& risky) {
  const float kL = -1.44269502162933349609375f;   // -log2(e) rounded to float
  const float kLlo = -1.925963033500011e-08f;     // -log2(e) - kL
  const float kLn2 = 0.693147182464599609375f;
  const float th = __fmul_rn(v, kL);
  const float tl = __fmaf_rn(v, kLlo, __fmaf_rn(v, kL, -th));
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(th));
  e = __fmaf_rn(e, __fmul_rn(kLn2, tl), e);
  const float d = __fadd_rn(1.0f, e);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float q = __fmul_rn(v, r);
  const float av = fabsf(v);
  risky = ((__float_as_uint(q) + 32u) & 0xffc0u) == 0x8000u || !(av <= 64.0f) ||
          !(av >= 7.888609052e-31f);
  return q;
}

__device__ __forceinline__ float silu_for_bf16(float v) {
  bool risky;
  const float q = silu_fast(v, risky);
  return risky ? silu_exact(v) : q;
}

template <int ACT, int DT>
__device__ __forceinline__ float activation(float v) {
  if constexpr (ACT == MOSS_ACT_SILU) {
    if constexpr (DT == MOSS_BF16) {
      return silu_for_bf16(v);
    } else {
      return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    }
  } else if constexpr (ACT == MOSS_ACT_GELU_ERF) {
    const float k_alpha = 0.70710678118654752440f;
    return __fmul_rn(__fmul_rn(v, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(v, k_alpha))));
  } else {
    const float k_beta = 0.79788456080286535588f;
    const float k_kappa = 0.044715f;
    const float cube = __fmul_rn(__fmul_rn(v, v), v);
    const float inner = __fmul_rn(k_beta, __fmaf_rn(k_kappa, cube, v));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
  }
}

template <int ACT>
__device__ __forceinline__ float activation_exact(float v) {
  if constexpr (ACT == MOSS_ACT_SILU) {
    return silu_exact(v);
  } else {
    return activation<ACT, MOSS_BF16>(v);
  }
}

// The per-device tables of the three activations over all 65536 bf16
// inputs (gated_act.cu), and whether they are built on the current device
// (the first call outside a stream capture builds them and waits).
extern __device__ uint16_t g_act_lut[3 * 65536];
bool act_lut_ready(cudaStream_t s);

}  // namespace moss
