// Rotary embedding of q and k (interleaved pairs).
//
// Rotation (fast_moss/v2_pointwise.py:8-47):
//   o[2p]   = q[2p]*c - q[2p+1]*s
//   o[2p+1] = q[2p]*s + q[2p+1]*c      float32, every product and sum rounded
// output contiguous [b,h,t,d] in the input dtype (round to nearest even).
//
// Phase (fast_moss/v2_runtime.py:209-222), used when the tables are not
// given: freq[j] = expf(j * coef), ts = float(offset[b]) + t,
// phase = freq[j] * ts, c = cosf(phase), s = sinf(phase).
//
// Work decomposition: a CTA owns one batch index and a tile of TT time steps
// for ALL heads.  In phase mode it first evaluates the TT x d/2 (c, s) pairs
// once into shared memory (the phase does not depend on the head), then the
// 256 threads stream q and k for every head of the tile with 16-byte vector
// loads when the innermost stride is 1 (a qkv projection output viewed as
// [b,h,t,d] qualifies), or with per-element strided loads otherwise.
#include "common.cuh"

namespace moss {

struct RopeArgs {
  const void* q;
  const void* k;
  const float* cos_t;
  const float* sin_t;
  const void* offset;
  int offset_dtype;
  float coef;
  void* oq;
  void* ok;
  int64_t b, h, t, d;
  int64_t qs[4];
  int64_t ks[4];
  int tt;  // time steps per CTA
};

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

// VW = elements per thread item (8 for bf16 vectors, 4 for f32 vectors, 2 for
// the generic strided pair).  TABLES selects caller tables vs phase mode.
template <int DT, int VW, bool TABLES>
__global__ void __launch_bounds__(256) rope_kernel(RopeArgs a) {
  extern __shared__ float smem[];  // [2][tt][d/2] in phase mode
  const int half = static_cast<int>(a.d >> 1);
  const int64_t ntiles = (a.t + a.tt - 1) / a.tt;
  const int64_t bi = blockIdx.x / ntiles;
  const int64_t t0 = (blockIdx.x % ntiles) * a.tt;
  const int tt = static_cast<int>(a.t - t0 < a.tt ? a.t - t0 : a.tt);
  float* sc = smem;
  float* ss = smem + a.tt * half;

  if constexpr (!TABLES) {
    const float off = offset_as_float(a.offset, a.offset_dtype, bi);
    for (int i = threadIdx.x; i < tt * half; i += blockDim.x) {
      const int tl = i / half;
      const int j = i - tl * half;
      const float freq = expf(__fmul_rn(static_cast<float>(j), a.coef));
      const float ts = __fadd_rn(off, static_cast<float>(t0 + tl));
      const float phase = __fmul_rn(freq, ts);
      sc[i] = cosf(phase);
      ss[i] = sinf(phase);
    }
    __syncthreads();
  }

  // h * tt * (d / VW) <= h * 256 * 512 is checked on the host to fit in int.
  const int nvec = static_cast<int>(a.d / VW);
  const int items = static_cast<int>(a.h) * tt * nvec;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int vec = it % nvec;
    const int rest = it / nvec;
    const int tl = rest % tt;
    const int64_t hi = rest / tt;
    const int64_t ti = t0 + tl;
    const int p0 = vec * (VW / 2);  // first pair of this item
    float c[VW / 2], s[VW / 2];
    if constexpr (TABLES) {
      const int64_t tb = (bi * a.t + ti) * half + p0;
#pragma unroll
      for (int j = 0; j < VW / 2; ++j) {
        c[j] = a.cos_t[tb + j];
        s[j] = a.sin_t[tb + j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < VW / 2; ++j) {
        c[j] = sc[tl * half + p0 + j];
        s[j] = ss[tl * half + p0 + j];
      }
    }
    const int64_t qrow = bi * a.qs[0] + hi * a.qs[1] + ti * a.qs[2];
    const int64_t krow = bi * a.ks[0] + hi * a.ks[1] + ti * a.ks[2];
    const int64_t orow = ((bi * a.h + hi) * a.t + ti) * a.d + static_cast<int64_t>(vec) * VW;
    float qv[VW], kv[VW];
    if constexpr (VW == 8 && DT == MOSS_BF16) {
      const uint4 qraw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.q) + qrow + vec * VW);
      const uint4 kraw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.k) + krow + vec * VW);
      unpack_bf16x8(qraw, qv);
      unpack_bf16x8(kraw, kv);
    } else if constexpr (VW == 4 && DT == MOSS_F32) {
      const float4 q4 = *reinterpret_cast<const float4*>(static_cast<const float*>(a.q) + qrow + vec * VW);
      const float4 k4 = *reinterpret_cast<const float4*>(static_cast<const float*>(a.k) + krow + vec * VW);
      qv[0] = q4.x; qv[1] = q4.y; qv[2] = q4.z; qv[3] = q4.w;
      kv[0] = k4.x; kv[1] = k4.y; kv[2] = k4.z; kv[3] = k4.w;
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const int64_t de = static_cast<int64_t>(vec) * VW + e;
        qv[e] = load_as_f32<DT>(a.q, qrow + de * a.qs[3]);
        kv[e] = load_as_f32<DT>(a.k, krow + de * a.ks[3]);
      }
    }
    float qo[VW], ko[VW];
#pragma unroll
    for (int j = 0; j < VW / 2; ++j) {
      rotate_pair(qv[2 * j], qv[2 * j + 1], c[j], s[j], qo[2 * j], qo[2 * j + 1]);
      rotate_pair(kv[2 * j], kv[2 * j + 1], c[j], s[j], ko[2 * j], ko[2 * j + 1]);
    }
    if constexpr (VW == 8 && DT == MOSS_BF16) {
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.oq) + orow) = pack_bf16x8(qo);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.ok) + orow) = pack_bf16x8(ko);
    } else if constexpr (VW == 4 && DT == MOSS_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(a.oq) + orow) = make_float4(qo[0], qo[1], qo[2], qo[3]);
      *reinterpret_cast<float4*>(static_cast<float*>(a.ok) + orow) = make_float4(ko[0], ko[1], ko[2], ko[3]);
    } else {
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        store_from_f32<DT>(a.oq, orow + e, qo[e]);
        store_from_f32<DT>(a.ok, orow + e, ko[e]);
      }
    }
  }
}

template <int DT, bool TABLES>
static void launch_rope(RopeArgs a, bool vec, cudaStream_t s) {
  const int half = static_cast<int>(a.d >> 1);
  const int64_t ntiles = (a.t + a.tt - 1) / a.tt;
  const int64_t grid = a.b * ntiles;
  const size_t shmem = TABLES ? 0 : sizeof(float) * 2 * a.tt * half;
  constexpr int kVec = DT == MOSS_BF16 ? 8 : 4;
  if (vec) {
    rope_kernel<DT, kVec, TABLES><<<static_cast<unsigned>(grid), 256, shmem, s>>>(a);
  } else {
    rope_kernel<DT, 2, TABLES><<<static_cast<unsigned>(grid), 256, shmem, s>>>(a);
  }
}

static int rope_common(const char* name, RopeArgs a, int dtype, bool tables, void* stream) {
  if (a.b < 0 || a.h < 0 || a.t < 0 || a.d < 2 || (a.d & 1))
    return fail(MOSS_ERR_VALUE, "%s: expected equal B,H,T,even-D rotary inputs", name);
  if (dtype != MOSS_F32 && dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: q/k dtype must be float32 or bfloat16", name);
  if (a.d > 1024) return fail(MOSS_ERR_UNSUPPORTED, "%s: head dim above 1024", name);
  const int64_t n = a.b * a.h * a.t;
  if (n == 0) return MOSS_OK;
  if (!a.q || !a.k || !a.oq || !a.ok) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (tables && (!a.cos_t || !a.sin_t)) return fail(MOSS_ERR_VALUE, "%s: null table", name);
  if (!tables && !a.offset) return fail(MOSS_ERR_VALUE, "%s: null offset", name);
  if (!tables && (a.offset_dtype < 0 || a.offset_dtype > 2))
    return fail(MOSS_ERR_VALUE, "%s: offset dtype must be int64, int32 or float32", name);
  const int half = static_cast<int>(a.d / 2);
  int tt = 256 / half;
  if (tt < 1) tt = 1;
  if (tt > a.t) tt = static_cast<int>(a.t);
  a.tt = tt;
  const int64_t ntiles = (a.t + tt - 1) / tt;
  if (a.b * ntiles > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: grid too large", name);
  if (a.h * tt * (a.d / 2) > 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too many heads for one CTA tile", name);
  const int esize = dtype == MOSS_F32 ? 4 : 2;
  const int vw = dtype == MOSS_F32 ? 4 : 8;
  bool vec = (a.d % vw == 0) && a.qs[3] == 1 && a.ks[3] == 1 && aligned16(a.q) && aligned16(a.k) &&
             aligned16(a.oq) && aligned16(a.ok);
  for (int i = 0; i < 3 && vec; ++i) {
    if ((a.qs[i] * esize) % 16 != 0 || (a.ks[i] * esize) % 16 != 0) vec = false;
  }
  cudaStream_t s = as_stream(stream);
  if (dtype == MOSS_BF16) {
    if (tables) launch_rope<MOSS_BF16, true>(a, vec, s);
    else launch_rope<MOSS_BF16, false>(a, vec, s);
  } else {
    if (tables) launch_rope<MOSS_F32, true>(a, vec, s);
    else launch_rope<MOSS_F32, false>(a, vec, s);
  }
  return launch_status(name);
}

}  // namespace moss

using namespace moss;

extern "C" int moss_rotate(const void* q, const void* k, int dtype, const float* cos_t,
                           const float* sin_t, void* oq, void* ok, int64_t b, int64_t h, int64_t t,
                           int64_t d, const int64_t* q_strides, const int64_t* k_strides,
                           void* stream) {
  if (!q_strides || !k_strides) return fail(MOSS_ERR_VALUE, "moss_rotate: null strides");
  RopeArgs a{};
  a.q = q; a.k = k; a.cos_t = cos_t; a.sin_t = sin_t; a.oq = oq; a.ok = ok;
  a.b = b; a.h = h; a.t = t; a.d = d;
  for (int i = 0; i < 4; ++i) { a.qs[i] = q_strides[i]; a.ks[i] = k_strides[i]; }
  return rope_common("moss_rotate", a, dtype, true, stream);
}

extern "C" int moss_rope(const void* q, const void* k, int dtype, const void* offset,
                         int offset_dtype, float freq_coef, void* oq, void* ok, int64_t b,
                         int64_t h, int64_t t, int64_t d, const int64_t* q_strides,
                         const int64_t* k_strides, void* stream) {
  if (!q_strides || !k_strides) return fail(MOSS_ERR_VALUE, "moss_rope: null strides");
  RopeArgs a{};
  a.q = q; a.k = k; a.offset = offset; a.offset_dtype = offset_dtype; a.coef = freq_coef;
  a.oq = oq; a.ok = ok;
  a.b = b; a.h = h; a.t = t; a.d = d;
  for (int i = 0; i < 4; ++i) { a.qs[i] = q_strides[i]; a.ks[i] = k_strides[i]; }
  return rope_common("moss_rope", a, dtype, false, stream);
}
