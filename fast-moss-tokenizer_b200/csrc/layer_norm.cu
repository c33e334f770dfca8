// Residual scale-add and LayerNorm kernels.
//
// Residual (fast_moss/v2_pointwise.py:92-98): y = x + u*s, product and sum
// rounded separately.
//
// LayerNorm: the reference normalises with stock nn.LayerNorm on CUDA
// (fast_moss/v2_runtime.py:259).  For float32 rows whose width n is a
// multiple of 4 (and 16-byte aligned pointers) PyTorch runs its vectorised
// layer-norm forward, whose arithmetic is reproduced here operation for
// operation:
//   * a block of 128 threads (4 warps of 32) per row; thread j reads float4
//     vectors j, j+128, j+256, ... and pushes their elements, in order,
//     through a Welford update with a float count:
//       delta = v - mean; count += 1; mean = fma(delta, 1/count, mean);
//       m2 = fma(delta, v - mean, m2)
//   * a shuffle-down tree (offsets 16..1) inside each warp, then a two-level
//     tree across the warps (warp w merges warp w+2, then warp 0 merges 1),
//     each merge of (own B, other A) being
//       count = cA + cB; coef = 1/count; nA = cA*coef; nB = cB*coef;
//       mean = fma(nA, meanA, nB*meanB);
//       m2 = fma(delta*delta*cA, nB, m2A + m2B),  delta = meanB - meanA
//   * var = m2 / n; rstd = rsqrtf(var + eps);
//     y = fma(gamma, rstd * (x - mean), beta).
// The kernel uses the same 128-thread row blocks, so every thread holds at
// most four float4 vectors (n <= 2048) in ~40 registers and up to 16 rows
// are resident per SM, keeping enough loads in flight for HBM.  The
// reciprocals of the per-thread Welford counts (1..16) are compile-time
// constants (IEEE division evaluated by the compiler); the merges use the
// correctly rounded reciprocal instruction.
#include "common.cuh"

namespace moss {

struct Welford {
  float mean;
  float m2;
  float count;
};

// 1/c for c = 0..16, correctly rounded (c = 0 unused).
__device__ __constant__ float kRcpSmall[17] = {
    0.0f,        1.0f / 1.0f,  1.0f / 2.0f,  1.0f / 3.0f,  1.0f / 4.0f,  1.0f / 5.0f,
    1.0f / 6.0f, 1.0f / 7.0f,  1.0f / 8.0f,  1.0f / 9.0f,  1.0f / 10.0f, 1.0f / 11.0f,
    1.0f / 12.0f, 1.0f / 13.0f, 1.0f / 14.0f, 1.0f / 15.0f, 1.0f / 16.0f};

// Welford update to the new count c (1 <= c <= 16), whose reciprocal comes
// from the table (a constant-bank operand once the loops are unrolled).
__device__ __forceinline__ Welford welford_push(Welford w, float v, int c) {
  const float delta = __fsub_rn(v, w.mean);
  const float mean = __fmaf_rn(delta, kRcpSmall[c], w.mean);
  const float m2 = __fmaf_rn(delta, __fsub_rn(v, mean), w.m2);
  return {mean, m2, static_cast<float>(c)};
}

// Merge of the thread's own state b with a partner state a.
__device__ __forceinline__ Welford welford_merge(Welford b, Welford a) {
  const float delta = __fsub_rn(b.mean, a.mean);
  const float count = __fadd_rn(a.count, b.count);
  if (count > 0.0f) {
    const float coef = __frcp_rn(count);
    const float na = __fmul_rn(a.count, coef);
    const float nb = __fmul_rn(b.count, coef);
    const float mean = __fmaf_rn(na, a.mean, __fmul_rn(nb, b.mean));
    const float m2 =
        __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), a.count), nb, __fadd_rn(a.m2, b.m2));
    return {mean, m2, count};
  }
  return {0.0f, 0.0f, count};
}

// The merge of two states whose counts are compile-time constants: every
// thread of a row holds 4 * NVT values when the row width is a multiple of
// 512, so the counts of the whole reduction tree are known in advance, and
// the reciprocal and the two weights are the same correctly rounded values
// the general merge computes (IEEE float constant expressions).
template <int CA, int CB>
struct MergeWeights {
  static constexpr float count = static_cast<float>(CA + CB);
  static constexpr float coef = 1.0f / count;
  static constexpr float na = static_cast<float>(CA) * coef;
  static constexpr float nb = static_cast<float>(CB) * coef;
};

template <int CA, int CB>
__device__ __forceinline__ Welford welford_merge_const(Welford b, Welford a) {
  using W = MergeWeights<CA, CB>;
  const float delta = __fsub_rn(b.mean, a.mean);
  const float mean = __fmaf_rn(W::na, a.mean, __fmul_rn(W::nb, b.mean));
  const float m2 = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), static_cast<float>(CA)), W::nb,
                             __fadd_rn(a.m2, b.m2));
  return {mean, m2, W::count};
}

// Shuffle-down level with offset O of the full-row reduction (every lane's
// count is C before the level).
template <int C, int O>
__device__ __forceinline__ Welford shuffle_level_const(Welford w) {
  Welford o;
  o.mean = __shfl_down_sync(0xffffffffu, w.mean, O);
  o.m2 = __shfl_down_sync(0xffffffffu, w.m2, O);
  return welford_merge_const<C, C>(w, o);
}

template <int DT>
__device__ __forceinline__ float4 load4(const void* base, int64_t i4, bool vec_ok) {
  if constexpr (DT == MOSS_F32) {
    if (vec_ok) return reinterpret_cast<const float4*>(base)[i4];
    const float* p = static_cast<const float*>(base) + 4 * i4;
    return make_float4(p[0], p[1], p[2], p[3]);
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(base) + 4 * i4;
    if (vec_ok) {
      const uint2 v = reinterpret_cast<const uint2*>(base)[i4];
      return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                         __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
    }
    return make_float4(bf16_bits_to_f32(p[0]), bf16_bits_to_f32(p[1]), bf16_bits_to_f32(p[2]),
                       bf16_bits_to_f32(p[3]));
  }
}

__device__ __forceinline__ float scale_add1(float x, float u, float s) {
  return __fadd_rn(x, __fmul_rn(u, s));
}

// gamma * (rstd * (x - mean)) + beta with gamma and beta already loaded
// (the same operations as ln_out's first case).
__device__ __forceinline__ float4 ln_out_gb(float4 v, float mean, float rstd, float4 g, float4 b) {
  float4 o;
  o.x = __fmaf_rn(g.x, __fmul_rn(rstd, __fsub_rn(v.x, mean)), b.x);
  o.y = __fmaf_rn(g.y, __fmul_rn(rstd, __fsub_rn(v.y, mean)), b.y);
  o.z = __fmaf_rn(g.z, __fmul_rn(rstd, __fsub_rn(v.z, mean)), b.z);
  o.w = __fmaf_rn(g.w, __fmul_rn(rstd, __fsub_rn(v.w, mean)), b.w);
  return o;
}

__device__ __forceinline__ float4 ln_out(float4 v, float mean, float rstd, const float* gamma,
                                         const float* beta, int i) {
  float4 o;
  if (gamma && beta) {
    // gamma * (rstd * (x - mean)) + beta with the outer multiply-add fused
    const float4 g = reinterpret_cast<const float4*>(gamma)[i];
    const float4 b = reinterpret_cast<const float4*>(beta)[i];
    o.x = __fmaf_rn(g.x, __fmul_rn(rstd, __fsub_rn(v.x, mean)), b.x);
    o.y = __fmaf_rn(g.y, __fmul_rn(rstd, __fsub_rn(v.y, mean)), b.y);
    o.z = __fmaf_rn(g.z, __fmul_rn(rstd, __fsub_rn(v.z, mean)), b.z);
    o.w = __fmaf_rn(g.w, __fmul_rn(rstd, __fsub_rn(v.w, mean)), b.w);
  } else if (gamma) {
    const float4 g = reinterpret_cast<const float4*>(gamma)[i];
    o.x = __fmul_rn(g.x, __fmul_rn(rstd, __fsub_rn(v.x, mean)));
    o.y = __fmul_rn(g.y, __fmul_rn(rstd, __fsub_rn(v.y, mean)));
    o.z = __fmul_rn(g.z, __fmul_rn(rstd, __fsub_rn(v.z, mean)));
    o.w = __fmul_rn(g.w, __fmul_rn(rstd, __fsub_rn(v.w, mean)));
  } else if (beta) {
    // without gamma the product rstd * (x - mean) itself fuses with the add
    const float4 b = reinterpret_cast<const float4*>(beta)[i];
    o.x = __fmaf_rn(rstd, __fsub_rn(v.x, mean), b.x);
    o.y = __fmaf_rn(rstd, __fsub_rn(v.y, mean), b.y);
    o.z = __fmaf_rn(rstd, __fsub_rn(v.z, mean), b.z);
    o.w = __fmaf_rn(rstd, __fsub_rn(v.w, mean), b.w);
  } else {
    o.x = __fmul_rn(rstd, __fsub_rn(v.x, mean));
    o.y = __fmul_rn(rstd, __fsub_rn(v.y, mean));
    o.z = __fmul_rn(rstd, __fsub_rn(v.z, mean));
    o.w = __fmul_rn(rstd, __fsub_rn(v.w, mean));
  }
  return o;
}

// One 128-thread block per row.  NVT = float4 vectors per thread
// (n <= 512 * NVT).  HAS_U selects the fused residual form.
template <int NVT, int XDT, int UDT, bool HAS_U, bool FULL>
__global__ void __launch_bounds__(128) residual_ln_kernel(
    const void* __restrict__ x, const void* __restrict__ u, const float* __restrict__ scale,
    const float* __restrict__ gamma, const float* __restrict__ beta, float eps, int n,
    float* __restrict__ residual_out, void* __restrict__ normed_out,
    float* __restrict__ mean_out, float* __restrict__ rstd_out, bool x_vec, bool u_vec,
    bool out_bf16) {
  __shared__ float red[4][3];
  __shared__ float stats[2];
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const int nvec = n >> 2;
  const int64_t base4 = row * nvec;

  // Issue every load of the row, and of the affine parameters, before any
  // arithmetic.
  const bool gb = gamma != nullptr && beta != nullptr;
  float4 val[NVT], upd[NVT], sv[NVT], gv[NVT], bv[NVT];
#pragma unroll
  for (int m = 0; m < NVT; ++m) {
    const int i = tid + 128 * m;
    if (i < nvec) {
      val[m] = load4<XDT>(x, base4 + i, x_vec);
      if constexpr (HAS_U) {
        upd[m] = load4<UDT>(u, base4 + i, u_vec);
        sv[m] = reinterpret_cast<const float4*>(scale)[i];
      }
      if (gb) {
        gv[m] = reinterpret_cast<const float4*>(gamma)[i];
        bv[m] = reinterpret_cast<const float4*>(beta)[i];
      }
    }
  }
  Welford w = {0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int m = 0; m < NVT; ++m) {
    const int i = tid + 128 * m;
    if (i < nvec) {
      if constexpr (HAS_U) {
        const float4 s = sv[m];
        val[m].x = scale_add1(val[m].x, upd[m].x, s.x);
        val[m].y = scale_add1(val[m].y, upd[m].y, s.y);
        val[m].z = scale_add1(val[m].z, upd[m].z, s.z);
        val[m].w = scale_add1(val[m].w, upd[m].w, s.w);
        if (residual_out != nullptr) reinterpret_cast<float4*>(residual_out)[base4 + i] = val[m];
      }
      // counts 4m+1 .. 4m+4: a valid vector m implies vectors 0..m-1 were valid
      w = welford_push(w, val[m].x, 4 * m + 1);
      w = welford_push(w, val[m].y, 4 * m + 2);
      w = welford_push(w, val[m].z, 4 * m + 3);
      w = welford_push(w, val[m].w, 4 * m + 4);
    }
  }
  if constexpr (FULL) {
    constexpr int C = 4 * NVT;
    w = shuffle_level_const<C, 16>(w);
    w = shuffle_level_const<2 * C, 8>(w);
    w = shuffle_level_const<4 * C, 4>(w);
    w = shuffle_level_const<8 * C, 2>(w);
    w = shuffle_level_const<16 * C, 1>(w);
  } else {
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
      Welford o;
      o.mean = __shfl_down_sync(0xffffffffu, w.mean, offset);
      o.m2 = __shfl_down_sync(0xffffffffu, w.m2, offset);
      o.count = __shfl_down_sync(0xffffffffu, w.count, offset);
      w = welford_merge(w, o);
    }
  }
  if (lane == 0) {
    red[warp][0] = w.mean;
    red[warp][1] = w.m2;
    red[warp][2] = w.count;
  }
  __syncthreads();
  if (tid == 0) {
    const Welford w0 = {red[0][0], red[0][1], red[0][2]};
    const Welford w1 = {red[1][0], red[1][1], red[1][2]};
    const Welford w2 = {red[2][0], red[2][1], red[2][2]};
    const Welford w3 = {red[3][0], red[3][1], red[3][2]};
    Welford t;
    if constexpr (FULL) {
      constexpr int CW = 128 * NVT;  // values per warp
      t = welford_merge_const<2 * CW, 2 * CW>(welford_merge_const<CW, CW>(w0, w2),
                                              welford_merge_const<CW, CW>(w1, w3));
    } else {
      t = welford_merge(welford_merge(w0, w2), welford_merge(w1, w3));
    }
    const float var = __fdiv_rn(t.m2, static_cast<float>(n));
    const float rstd = rsqrtf(__fadd_rn(var, eps));
    stats[0] = t.mean;
    stats[1] = rstd;
    if (mean_out) mean_out[row] = t.mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
  __syncthreads();
  const float mean = stats[0], rstd = stats[1];
#pragma unroll
  for (int m = 0; m < NVT; ++m) {
    const int i = tid + 128 * m;
    if (i < nvec) {
      const float4 o = gb ? ln_out_gb(val[m], mean, rstd, gv[m], bv[m])
                          : ln_out(val[m], mean, rstd, gamma, beta, i);
      if (out_bf16) {
        // the consumer's cast: round to nearest even, as torch's .to(bfloat16)
        reinterpret_cast<uint2*>(normed_out)[base4 + i] = make_uint2(
            static_cast<uint32_t>(f32_to_bf16_bits(o.x)) |
                (static_cast<uint32_t>(f32_to_bf16_bits(o.y)) << 16),
            static_cast<uint32_t>(f32_to_bf16_bits(o.z)) |
                (static_cast<uint32_t>(f32_to_bf16_bits(o.w)) << 16));
      } else {
        reinterpret_cast<float4*>(normed_out)[base4 + i] = o;
      }
    }
  }
}

// Plain residual update y = x + u*s over n elements, channel count c.
template <int XDT, int UDT>
__global__ void __launch_bounds__(256) scale_add_vec_kernel(const void* __restrict__ x,
                                                            const void* __restrict__ u,
                                                            const float* __restrict__ scale,
                                                            float* __restrict__ y, int64_t n4,
                                                            int64_t c4) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 xv = load4<XDT>(x, i, true);
    const float4 uv = load4<UDT>(u, i, true);
    const float4 s = reinterpret_cast<const float4*>(scale)[i % c4];
    float4 o;
    o.x = scale_add1(xv.x, uv.x, s.x);
    o.y = scale_add1(xv.y, uv.y, s.y);
    o.z = scale_add1(xv.z, uv.z, s.z);
    o.w = scale_add1(xv.w, uv.w, s.w);
    reinterpret_cast<float4*>(y)[i] = o;
  }
}

template <int XDT, int UDT>
__global__ void __launch_bounds__(256) scale_add_scalar_kernel(const void* __restrict__ x,
                                                               const void* __restrict__ u,
                                                               const float* __restrict__ scale,
                                                               float* __restrict__ y, int64_t n,
                                                               int64_t c) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    y[i] = scale_add1(load_as_f32<XDT>(x, i), load_as_f32<UDT>(u, i), scale[i % c]);
  }
}

// ------------------------------------------------------------------ launchers
template <int NVT, int XDT, int UDT, bool HAS_U>
static void launch_ln(const void* x, const void* u, const float* scale, const float* gamma,
                      const float* beta, float eps, int64_t rows, int n, float* res,
                      void* normed, float* mean, float* rstd, bool xv, bool uv, bool ob,
                      cudaStream_t s) {
  if (n == 512 * NVT) {  // every thread holds 4 * NVT values: constant merge weights
    residual_ln_kernel<NVT, XDT, UDT, HAS_U, true><<<static_cast<unsigned>(rows), 128, 0, s>>>(
        x, u, scale, gamma, beta, eps, n, res, normed, mean, rstd, xv, uv, ob);
  } else {
    residual_ln_kernel<NVT, XDT, UDT, HAS_U, false><<<static_cast<unsigned>(rows), 128, 0, s>>>(
        x, u, scale, gamma, beta, eps, n, res, normed, mean, rstd, xv, uv, ob);
  }
}

template <int XDT, int UDT, bool HAS_U>
static int dispatch_nvt(int nvt, const void* x, const void* u, const float* scale,
                        const float* gamma, const float* beta, float eps, int64_t rows, int n,
                        float* res, void* normed, float* mean, float* rstd, bool xv, bool uv,
                        bool ob, cudaStream_t s) {
  switch (nvt) {
    case 1:
      launch_ln<1, XDT, UDT, HAS_U>(x, u, scale, gamma, beta, eps, rows, n, res, normed, mean,
                                    rstd, xv, uv, ob, s);
      return MOSS_OK;
    case 2:
      launch_ln<2, XDT, UDT, HAS_U>(x, u, scale, gamma, beta, eps, rows, n, res, normed, mean,
                                    rstd, xv, uv, ob, s);
      return MOSS_OK;
    case 3:
      launch_ln<3, XDT, UDT, HAS_U>(x, u, scale, gamma, beta, eps, rows, n, res, normed, mean,
                                    rstd, xv, uv, ob, s);
      return MOSS_OK;
    case 4:
      launch_ln<4, XDT, UDT, HAS_U>(x, u, scale, gamma, beta, eps, rows, n, res, normed, mean,
                                    rstd, xv, uv, ob, s);
      return MOSS_OK;
    default:
      return MOSS_ERR_UNSUPPORTED;
  }
}

static int ln_common(const char* name, const void* x, int x_dtype, const void* u, int u_dtype,
                     const float* scale, const float* gamma, const float* beta, float eps,
                     int64_t rows, int64_t n, float* residual_out, void* normed_out,
                     int normed_dtype, float* mean, float* rstd, void* stream) {
  if (rows < 0 || n <= 0) return fail(MOSS_ERR_VALUE, "%s: rows must be >= 0 and n > 0", name);
  if (x == nullptr || normed_out == nullptr)
    return fail(MOSS_ERR_VALUE, "%s: null input or output pointer", name);
  if (x_dtype != MOSS_F32 && x_dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: x dtype must be float32 or bfloat16", name);
  if (u != nullptr && u_dtype != MOSS_F32 && u_dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: update dtype must be float32 or bfloat16", name);
  if (u != nullptr && scale == nullptr)
    return fail(MOSS_ERR_VALUE, "%s: a residual update needs a channel scale", name);
  if (n % 4 != 0)
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: width %lld is not a multiple of 4 (PyTorch uses its non-vectorised "
                "layer norm there)",
                name, static_cast<long long>(n));
  if (normed_dtype != MOSS_F32 && normed_dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: normalised output dtype must be float32 or bfloat16", name);
  const bool ob = normed_dtype == MOSS_BF16;
  if ((gamma && !aligned16(gamma)) || (beta && !aligned16(beta)) ||
      (ob ? (reinterpret_cast<uintptr_t>(normed_out) & 7u) != 0 : !aligned16(normed_out)) ||
      (residual_out && !aligned16(residual_out)) || (scale && !aligned16(scale)))
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: gamma/beta/scale/outputs must be 16-byte aligned (PyTorch uses its "
                "non-vectorised layer norm otherwise)",
                name);
  if (u == nullptr && x_dtype != MOSS_F32)
    return fail(MOSS_ERR_VALUE, "%s: plain layer norm takes float32 input", name);
  if (u == nullptr && !aligned16(x))
    return fail(MOSS_ERR_UNSUPPORTED, "%s: x must be 16-byte aligned", name);
  const int nvt = static_cast<int>((n / 4 + 127) / 128);
  if (nvt > 4)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: width %lld above the 2048 supported", name,
                static_cast<long long>(n));
  if (rows > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows", name);
  if (rows == 0) return MOSS_OK;
  const bool xv = (x_dtype == MOSS_F32) ? aligned16(x) : ((reinterpret_cast<uintptr_t>(x) & 7u) == 0);
  const bool uv = u == nullptr ? true
                               : ((u_dtype == MOSS_F32) ? aligned16(u)
                                                        : ((reinterpret_cast<uintptr_t>(u) & 7u) == 0));
  cudaStream_t s = as_stream(stream);
  const int ni = static_cast<int>(n);
  int st;
  if (u == nullptr) {
    st = dispatch_nvt<MOSS_F32, MOSS_F32, false>(nvt, x, nullptr, nullptr, gamma, beta, eps, rows,
                                                 ni, nullptr, normed_out, mean, rstd, xv, uv, ob, s);
  } else if (x_dtype == MOSS_F32 && u_dtype == MOSS_F32) {
    st = dispatch_nvt<MOSS_F32, MOSS_F32, true>(nvt, x, u, scale, gamma, beta, eps, rows, ni,
                                                residual_out, normed_out, mean, rstd, xv, uv, ob, s);
  } else if (x_dtype == MOSS_F32 && u_dtype == MOSS_BF16) {
    st = dispatch_nvt<MOSS_F32, MOSS_BF16, true>(nvt, x, u, scale, gamma, beta, eps, rows, ni,
                                                 residual_out, normed_out, mean, rstd, xv, uv, ob, s);
  } else if (x_dtype == MOSS_BF16 && u_dtype == MOSS_F32) {
    st = dispatch_nvt<MOSS_BF16, MOSS_F32, true>(nvt, x, u, scale, gamma, beta, eps, rows, ni,
                                                 residual_out, normed_out, mean, rstd, xv, uv, ob, s);
  } else {
    st = dispatch_nvt<MOSS_BF16, MOSS_BF16, true>(nvt, x, u, scale, gamma, beta, eps, rows, ni,
                                                  residual_out, normed_out, mean, rstd, xv, uv, ob, s);
  }
  if (st != MOSS_OK) return fail(st, "%s: unsupported width", name);
  return launch_status(name);
}

}  // namespace moss

using namespace moss;

extern "C" int moss_layer_norm(const float* x, const float* gamma, const float* beta, float eps,
                               int64_t rows, int64_t n, float* y, float* mean, float* rstd,
                               void* stream) {
  return ln_common("moss_layer_norm", x, MOSS_F32, nullptr, MOSS_F32, nullptr, gamma, beta, eps,
                   rows, n, nullptr, y, MOSS_F32, mean, rstd, stream);
}

extern "C" int moss_residual_layer_norm(const void* x, int x_dtype, const void* u, int u_dtype,
                                        const float* scale, const float* gamma,
                                        const float* beta, float eps, int64_t rows, int64_t n,
                                        float* residual_out, float* normed_out, float* mean,
                                        float* rstd, void* stream) {
  if (u == nullptr) return fail(MOSS_ERR_VALUE, "moss_residual_layer_norm: update is null");
  return ln_common("moss_residual_layer_norm", x, x_dtype, u, u_dtype, scale, gamma, beta, eps,
                   rows, n, residual_out, normed_out, MOSS_F32, mean, rstd, stream);
}

extern "C" int moss_residual_layer_norm_out(const void* x, int x_dtype, const void* u,
                                            int u_dtype, const float* scale, const float* gamma,
                                            const float* beta, float eps, int64_t rows, int64_t n,
                                            float* residual_out, void* normed_out,
                                            int normed_dtype, float* mean, float* rstd,
                                            void* stream) {
  return ln_common("moss_residual_layer_norm_out", x, x_dtype, u, u_dtype, scale, gamma, beta,
                   eps, rows, n, residual_out, normed_out, normed_dtype, mean, rstd, stream);
}

extern "C" int moss_scale_add(const void* x, int x_dtype, const void* u, int u_dtype,
                              const float* scale, float* y, int64_t n, int64_t c, void* stream) {
  const char* name = "moss_scale_add";
  if (n < 0 || c <= 0) return fail(MOSS_ERR_VALUE, "%s: n must be >= 0 and c > 0", name);
  if (n % c != 0) return fail(MOSS_ERR_VALUE, "%s: n is not a multiple of the channel count", name);
  if ((x_dtype != MOSS_F32 && x_dtype != MOSS_BF16) || (u_dtype != MOSS_F32 && u_dtype != MOSS_BF16))
    return fail(MOSS_ERR_VALUE, "%s: dtypes must be float32 or bfloat16", name);
  if (n == 0) return MOSS_OK;
  if (!x || !u || !scale || !y) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  cudaStream_t s = as_stream(stream);
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x), ua = reinterpret_cast<uintptr_t>(u);
  const bool vec = (c % 4 == 0) && aligned16(scale) && aligned16(y) &&
                   ((x_dtype == MOSS_F32) ? (xa & 15u) == 0 : (xa & 7u) == 0) &&
                   ((u_dtype == MOSS_F32) ? (ua & 15u) == 0 : (ua & 7u) == 0);
  const int sms = sm_count();
  if (vec) {
    const int64_t n4 = n / 4;
    int64_t grid = (n4 + 255) / 256;
    if (grid > static_cast<int64_t>(sms) * 16) grid = static_cast<int64_t>(sms) * 16;
#define MOSS_SA(XD, UD) \
  scale_add_vec_kernel<XD, UD><<<static_cast<unsigned>(grid), 256, 0, s>>>(x, u, scale, y, n4, c / 4)
    if (x_dtype == MOSS_F32 && u_dtype == MOSS_F32) MOSS_SA(MOSS_F32, MOSS_F32);
    else if (x_dtype == MOSS_F32) MOSS_SA(MOSS_F32, MOSS_BF16);
    else if (u_dtype == MOSS_F32) MOSS_SA(MOSS_BF16, MOSS_F32);
    else MOSS_SA(MOSS_BF16, MOSS_BF16);
#undef MOSS_SA
  } else {
    int64_t grid = (n + 255) / 256;
    if (grid > static_cast<int64_t>(sms) * 16) grid = static_cast<int64_t>(sms) * 16;
#define MOSS_SA(XD, UD) \
  scale_add_scalar_kernel<XD, UD><<<static_cast<unsigned>(grid), 256, 0, s>>>(x, u, scale, y, n, c)
    if (x_dtype == MOSS_F32 && u_dtype == MOSS_F32) MOSS_SA(MOSS_F32, MOSS_F32);
    else if (x_dtype == MOSS_F32) MOSS_SA(MOSS_F32, MOSS_BF16);
    else if (u_dtype == MOSS_F32) MOSS_SA(MOSS_BF16, MOSS_F32);
    else MOSS_SA(MOSS_BF16, MOSS_BF16);
#undef MOSS_SA
  }
  return launch_status(name);
}
