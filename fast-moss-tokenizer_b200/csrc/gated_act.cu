// Bias + (gated) activation, one pass over HBM.
//
// The reference has no kernel for the FFN activation (it lives in the
// upstream model code); this reproduces the eager PyTorch chain that runs
// there, with one rounding to the storage dtype per torch op:
//   h    = round(x + bias)
//   a    = round(act(h_gate))           act evaluated in float32:
//            silu(v)      = v / (1 + expf(-v))
//            gelu_erf(v)  = v * 0.5 * (1 + erff(v * sqrt(1/2)))
//            gelu_tanh(v) = 0.5 * v * (1 + tanhf(k_beta * fma(0.044715, v^3, v)))
//   y    = round(a * h_up)              (gated)   or   y = a (ungated)
// For bf16 with the gate width a multiple of 8, each thread produces 8
// outputs from 16-byte loads of the gate half, the up half and the bias.
#include "common.cuh"

namespace moss {

template <int ACT>
__device__ __forceinline__ float activation(float v) {
  if constexpr (ACT == MOSS_ACT_SILU) {
    return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
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

template <int DT, int ACT, bool GATED>
__device__ __forceinline__ float gate_value(float xg, float bg, float xu, float bu) {
  const float hg = round_to<DT>(__fadd_rn(xg, bg));
  const float a = round_to<DT>(activation<ACT>(hg));
  if constexpr (GATED) {
    const float hu = round_to<DT>(__fadd_rn(xu, bu));
    return __fmul_rn(a, hu);
  } else {
    return a;
  }
}

// Vector path (bf16, 8 outputs per item).  out_w = width of the output row.
template <int ACT, bool GATED>
__global__ void __launch_bounds__(256) gated_act_bf16x8_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ bias, uint16_t* __restrict__ y,
    int64_t rows, int64_t width, int64_t out_w) {
  const int64_t per_row = out_w / 8;
  const int64_t items = rows * per_row;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = it / per_row;
    const int64_t c = (it - r * per_row) * 8;
    float xg[8], bg[8], xu[8], bu[8], out[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(x + r * width + c), xg);
    if (bias) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(bias + c), bg);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) bg[i] = 0.0f;
    }
    if constexpr (GATED) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(x + r * width + out_w + c), xu);
      if (bias) {
        unpack_bf16x8(*reinterpret_cast<const uint4*>(bias + out_w + c), bu);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) bu[i] = 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      out[i] = gate_value<MOSS_BF16, ACT, GATED>(xg[i], bg[i], GATED ? xu[i] : 0.0f,
                                                 GATED ? bu[i] : 0.0f);
    }
    *reinterpret_cast<uint4*>(y + r * out_w + c) = pack_bf16x8(out);
  }
}

template <int DT, int ACT, bool GATED>
__global__ void __launch_bounds__(256) gated_act_scalar_kernel(const void* __restrict__ x,
                                                               const void* __restrict__ bias,
                                                               void* __restrict__ y, int64_t rows,
                                                               int64_t width, int64_t out_w) {
  const int64_t items = rows * out_w;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = it / out_w;
    const int64_t c = it - r * out_w;
    const float xg = load_as_f32<DT>(x, r * width + c);
    const float bg = bias ? load_as_f32<DT>(bias, c) : 0.0f;
    float xu = 0.0f, bu = 0.0f;
    if constexpr (GATED) {
      xu = load_as_f32<DT>(x, r * width + out_w + c);
      bu = bias ? load_as_f32<DT>(bias, out_w + c) : 0.0f;
    }
    store_from_f32<DT>(y, it, gate_value<DT, ACT, GATED>(xg, bg, xu, bu));
  }
}

template <int ACT, bool GATED>
static void launch_gated(const void* x, const void* bias, void* y, int dtype, int64_t rows,
                         int64_t width, int64_t out_w, bool vec, cudaStream_t s) {
  const int sms = sm_count();
  if (vec) {
    const int64_t items = rows * (out_w / 8);
    int64_t grid = (items + 255) / 256;
    if (grid > static_cast<int64_t>(sms) * 8) grid = static_cast<int64_t>(sms) * 8;
    gated_act_bf16x8_kernel<ACT, GATED><<<static_cast<unsigned>(grid), 256, 0, s>>>(
        static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(bias),
        static_cast<uint16_t*>(y), rows, width, out_w);
  } else {
    const int64_t items = rows * out_w;
    int64_t grid = (items + 255) / 256;
    if (grid > static_cast<int64_t>(sms) * 8) grid = static_cast<int64_t>(sms) * 8;
    if (dtype == MOSS_BF16) {
      gated_act_scalar_kernel<MOSS_BF16, ACT, GATED>
          <<<static_cast<unsigned>(grid), 256, 0, s>>>(x, bias, y, rows, width, out_w);
    } else {
      gated_act_scalar_kernel<MOSS_F32, ACT, GATED>
          <<<static_cast<unsigned>(grid), 256, 0, s>>>(x, bias, y, rows, width, out_w);
    }
  }
}

}  // namespace moss

using namespace moss;

extern "C" int moss_gated_act(const void* x, const void* bias, void* y, int dtype, int64_t rows,
                              int64_t width, int act, int gated, void* stream) {
  const char* name = "moss_gated_act";
  if (rows < 0 || width <= 0) return fail(MOSS_ERR_VALUE, "%s: rows >= 0 and width > 0 required", name);
  if (dtype != MOSS_F32 && dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: dtype must be float32 or bfloat16", name);
  if (act < MOSS_ACT_SILU || act > MOSS_ACT_GELU_TANH)
    return fail(MOSS_ERR_VALUE, "%s: unknown activation %d", name, act);
  if (gated && (width % 2)) return fail(MOSS_ERR_VALUE, "%s: gated width must be even", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !y) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  const int64_t out_w = gated ? width / 2 : width;
  const bool vec = dtype == MOSS_BF16 && (out_w % 8 == 0) && aligned16(x) && aligned16(y) &&
                   (bias == nullptr || aligned16(bias));
  cudaStream_t s = as_stream(stream);
#define MOSS_GA(A)                                                              \
  if (gated) launch_gated<A, true>(x, bias, y, dtype, rows, width, out_w, vec, s); \
  else launch_gated<A, false>(x, bias, y, dtype, rows, width, out_w, vec, s);
  if (act == MOSS_ACT_SILU) {
    MOSS_GA(MOSS_ACT_SILU)
  } else if (act == MOSS_ACT_GELU_ERF) {
    MOSS_GA(MOSS_ACT_GELU_ERF)
  } else {
    MOSS_GA(MOSS_ACT_GELU_TANH)
  }
#undef MOSS_GA
  return launch_status(name);
}
