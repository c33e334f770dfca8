// LFQ (eight-channel, cosine-normalised codebook) quantizer kernels.
//
// prepare (fast_moss/quantizer_prepare.py:16-58): for each latent row x[8]
//   total = sum x^2 in one of two fixed orders (see sum_squares), denom =
//   sqrt(total) clamped below at 1e-12 with NaN passing through, e = x/denom,
//   twice = 2e, norm = sum e^2 (same order family), every op round-to-nearest.
//   The "transposed" order applies when b == 1 and t > 1: the reference then
//   follows PyTorch's strided reduction (four cyclic accumulators, FMA);
//   otherwise the adjacent pairwise tree of a contiguous row.
// select (fast_moss/quantizer.py:8-49): distance = (norm - dot) + code_norm,
//   first NaN wins, else first minimum; int64 index; raw codeword gathered.
// decode (fast_moss/v2_runtime.py:143-181): prepare + dots + select fused,
//   dots as a sequential FMA over the 8 channels.
#include "lfq.cuh"

#include <math_constants.h>

namespace moss {

struct Prepared {
  float e[8];
  float twice[8];
  float norm;
  float denom;
};

__device__ __forceinline__ Prepared prepare_row(const float* __restrict__ x, int64_t row,
                                                int64_t t, bool transposed) {
  float v[8];
  const int64_t bi = row / t, ti = row - bi * t;
#pragma unroll
  for (int d = 0; d < 8; ++d) v[d] = x[bi * 8 * t + d * t + ti];
  Prepared p;
  float denom = __fsqrt_rn(sum_squares(v, transposed));
  denom = denom < 1.0e-12f ? 1.0e-12f : denom;  // a NaN compares false and stays
  float esq[8];
#pragma unroll
  for (int d = 0; d < 8; ++d) {
    p.e[d] = __fdiv_rn(v[d], denom);
    p.twice[d] = __fmul_rn(2.0f, p.e[d]);
    esq[d] = __fmul_rn(p.e[d], p.e[d]);
  }
  p.norm = sum8(esq, transposed);
  p.denom = denom;
  return p;
}

__global__ void __launch_bounds__(128) lfq_prepare_kernel(const float* __restrict__ x, int64_t b,
                                                          int64_t t, float* __restrict__ e,
                                                          float* __restrict__ norm,
                                                          float* __restrict__ twice,
                                                          float* __restrict__ denom) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t rows = b * t;
  if (row >= rows) return;
  const bool transposed = (b == 1 && t > 1);
  const Prepared p = prepare_row(x, row, t, transposed);
#pragma unroll
  for (int d = 0; d < 8; ++d) {
    const int64_t o = transposed ? d * t + row : row * 8 + d;
    e[o] = p.e[d];
    twice[o] = p.twice[d];
  }
  norm[row] = p.norm;
  denom[row] = p.denom;
}

// One warp per row; lane L visits codes L, L+32, ...  The initial best index
// of a lane is its own first code, so a row whose distances are all +inf
// resolves to code 0 like the reference's first-minimum rule.
__global__ void __launch_bounds__(256) lfq_select_kernel(
    const float* __restrict__ dots, const float* __restrict__ row_norm,
    const float* __restrict__ code_norm, const float* __restrict__ book,
    const float* __restrict__ latents, int64_t ls0, int64_t ls1, int64_t ls2, int64_t b,
    int64_t dd, int64_t t, int64_t k, int ste, float* __restrict__ out,
    int64_t* __restrict__ indices) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= b * t) return;
  const float n = row_norm[row];
  Pick p{CUDART_INF_F, lane, INT64_MAX};
  const float* drow = dots + row * k;
  for (int64_t j = lane; j < k; j += 32) {
    pick_push(p, __fadd_rn(__fsub_rn(n, drow[j]), code_norm[j]), j);
  }
  const int64_t idx = pick_reduce(p);
  if (lane == 0) indices[row] = idx;
  const int64_t bi = row / t, ti = row - bi * t;
  for (int64_t d = lane; d < dd; d += 32) {
    const float value = book[idx * dd + d];
    if (ste) {
      const float latent = latents[bi * ls0 + d * ls1 + ti * ls2];
      out[bi * dd * t + d * t + ti] = __fadd_rn(latent, __fsub_rn(value, latent));
    } else {
      out[row * dd + d] = value;
    }
  }
}

// Fused decode: prepare + sequential-FMA dots + select + gather.
__global__ void __launch_bounds__(256) lfq_decode_kernel(
    const float* __restrict__ x, const float* __restrict__ book_normed,
    const float* __restrict__ code_norm, const float* __restrict__ weight, int64_t b, int64_t t,
    int64_t k, float* __restrict__ out, int64_t* __restrict__ indices) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= b * t) return;
  const Prepared p = prepare_row(x, row, t, b == 1 && t > 1);
  Pick pk{CUDART_INF_F, lane, INT64_MAX};
  for (int64_t j = lane; j < k; j += 32) {
    const float4 c0 = reinterpret_cast<const float4*>(book_normed + j * 8)[0];
    const float4 c1 = reinterpret_cast<const float4*>(book_normed + j * 8)[1];
    float dot = __fmul_rn(p.twice[0], c0.x);
    dot = __fmaf_rn(p.twice[1], c0.y, dot);
    dot = __fmaf_rn(p.twice[2], c0.z, dot);
    dot = __fmaf_rn(p.twice[3], c0.w, dot);
    dot = __fmaf_rn(p.twice[4], c1.x, dot);
    dot = __fmaf_rn(p.twice[5], c1.y, dot);
    dot = __fmaf_rn(p.twice[6], c1.z, dot);
    dot = __fmaf_rn(p.twice[7], c1.w, dot);
    pick_push(pk, __fadd_rn(__fsub_rn(p.norm, dot), code_norm[j]), j);
  }
  const int64_t idx = pick_reduce(pk);
  if (lane == 0) indices[row] = idx;
  if (lane < 8) out[row * 8 + lane] = weight[idx * 8 + lane];
}

// The same decode for many rows: the normalised codebook and its norms are
// staged in shared memory once per block of kDecWarps warps, each warp takes
// kDecRows rows against the whole codebook, and every codeword read serves
// all of its rows.  Per row and code the arithmetic is lfq_decode_kernel's
// (prepare_row, the sequential 8-channel dot, the distance rounding, the
// first-NaN / first-minimum pick), so the results are the same bits.  Rows
// past the end are computed on the last row and discarded, so that every
// warp reaches the block barrier.
//
// Measured on B200 at 8192 rows x 1024 / 4096 codes: 16 warps x 4 rows
// (64 rows per staged codebook) 10.3 / 31.5 us; 8 x 8 11.8 / 37.6 us,
// 16 x 8 17.0 / 55.3 us, 32 x 2 13.7 / 42.3 us; splitting a row group's
// codes across 2 or 4 warps with a shared-memory merge of the picks
// 12.1-13.0 / 47-66 us.
#ifndef MOSS_DEC_ROWS
#define MOSS_DEC_ROWS 4
#endif
#ifndef MOSS_DEC_WARPS
#define MOSS_DEC_WARPS 16
#endif
constexpr int kDecRows = MOSS_DEC_ROWS;
constexpr int kDecWarps = MOSS_DEC_WARPS;
constexpr int kDecRowsPerBlock = kDecRows * kDecWarps;
constexpr int kDecMaxCodes = 4096;  // 36 bytes per code of shared memory

__global__ void __launch_bounds__(kDecWarps * 32) lfq_decode_tile_kernel(
    const float* __restrict__ x, const float* __restrict__ book_normed,
    const float* __restrict__ code_norm, const float* __restrict__ weight, int64_t b, int64_t t,
    int k, float* __restrict__ out, int64_t* __restrict__ indices) {
  extern __shared__ float4 dec_smem[];
  float4* sbook = dec_smem;                                 // [k][2]
  float* scn = reinterpret_cast<float*>(dec_smem + 2 * k);  // [k]
  for (int i = threadIdx.x; i < 2 * k; i += blockDim.x)
    sbook[i] = reinterpret_cast<const float4*>(book_normed)[i];
  for (int i = threadIdx.x; i < k; i += blockDim.x) scn[i] = code_norm[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t rows = b * t;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * kDecWarps + warp) * kDecRows;
  const bool transposed = (b == 1 && t > 1);
  // lane r prepares row r of the warp's group (all lanes run one
  // preparation in parallel), then every lane receives the group's values
  float tw[kDecRows][8], nrm[kDecRows];
  {
    const int64_t mine = row0 + (lane % kDecRows);
    const Prepared p = prepare_row(x, mine < rows ? mine : rows - 1, t, transposed);
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) {
#pragma unroll
      for (int d = 0; d < 8; ++d) tw[r][d] = __shfl_sync(0xffffffffu, p.twice[d], r);
      nrm[r] = __shfl_sync(0xffffffffu, p.norm, r);
    }
  }
  __syncthreads();
  Pick32 pk[kDecRows];
#pragma unroll
  for (int r = 0; r < kDecRows; ++r) pk[r] = Pick32{CUDART_INF_F, lane, INT_MAX};
  for (int j = lane; j < k; j += 32) {
    const float4 c0 = sbook[2 * j], c1 = sbook[2 * j + 1];
    const float cn = scn[j];
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) {
      float dot = __fmul_rn(tw[r][0], c0.x);
      dot = __fmaf_rn(tw[r][1], c0.y, dot);
      dot = __fmaf_rn(tw[r][2], c0.z, dot);
      dot = __fmaf_rn(tw[r][3], c0.w, dot);
      dot = __fmaf_rn(tw[r][4], c1.x, dot);
      dot = __fmaf_rn(tw[r][5], c1.y, dot);
      dot = __fmaf_rn(tw[r][6], c1.z, dot);
      dot = __fmaf_rn(tw[r][7], c1.w, dot);
      pick32_push(pk[r], __fadd_rn(__fsub_rn(nrm[r], dot), cn), j);
    }
  }
  // every lane gets each row's index; lane r writes row r
  int mine = 0;
#pragma unroll
  for (int r = 0; r < kDecRows; ++r) {
    const int idx = pick32_reduce(pk[r]);
    mine = lane == r ? idx : mine;
  }
  const int64_t row = row0 + lane;
  if (lane < kDecRows && row < rows) {
    indices[row] = mine;
    const float4* src = reinterpret_cast<const float4*>(weight + static_cast<int64_t>(mine) * 8);
    float4* dst = reinterpret_cast<float4*>(out + row * 8);
    dst[0] = src[0];
    dst[1] = src[1];
  }
}

}  // namespace moss

using namespace moss;

extern "C" int moss_lfq_prepare(const float* x, int64_t b, int64_t t, float* e, float* norm,
                                float* twice, float* denom, void* stream) {
  const char* name = "moss_lfq_prepare";
  if (b < 1 || t < 1) return fail(MOSS_ERR_VALUE, "%s: expected nonempty B,8,T latents", name);
  if (b * 8 * t > 2147483647LL) return fail(MOSS_ERR_VALUE, "%s: more than 2^31-1 elements", name);
  if (!x || !e || !norm || !twice || !denom) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  const int64_t rows = b * t;
  lfq_prepare_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, as_stream(stream)>>>(
      x, b, t, e, norm, twice, denom);
  return launch_status(name);
}

extern "C" int moss_lfq_select(const float* dots, const float* row_norm, const float* code_norm,
                               const float* codebook, const float* latents,
                               const int64_t* latent_strides, int64_t b, int64_t d, int64_t t,
                               int64_t k, int straight_through, float* out, int64_t* indices,
                               void* stream) {
  const char* name = "moss_lfq_select";
  if (b < 0 || d < 1 || t < 0 || k < 1 || k > 65536)
    return fail(MOSS_ERR_VALUE, "%s: incompatible quantizer shapes or unsupported codebook size", name);
  if (b * t == 0) return MOSS_OK;
  if (!dots || !row_norm || !code_norm || !codebook || !out || !indices)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  int64_t ls[3] = {0, 0, 0};
  if (straight_through) {
    if (!latents || !latent_strides) return fail(MOSS_ERR_VALUE, "%s: STE needs latents", name);
    for (int i = 0; i < 3; ++i) ls[i] = latent_strides[i];
  }
  const int64_t rows = b * t;
  lfq_select_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, as_stream(stream)>>>(
      dots, row_norm, code_norm, codebook, latents, ls[0], ls[1], ls[2], b, d, t, k,
      straight_through, out, indices);
  return launch_status(name);
}

extern "C" int moss_lfq_decode(const float* x, const float* book_normed, const float* code_norm,
                               const float* weight, int64_t b, int64_t t, int64_t k, float* out,
                               int64_t* indices, void* stream) {
  const char* name = "moss_lfq_decode";
  if (b < 1 || t < 1 || k < 1 || k > 65536)
    return fail(MOSS_ERR_VALUE, "%s: expected nonempty B,8,T latents and 1..65536 codes", name);
  if (!x || !book_normed || !code_norm || !weight || !out || !indices)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(book_normed)) return fail(MOSS_ERR_VALUE, "%s: normalised book must be 16-byte aligned", name);
  const int64_t rows = b * t;
  if (rows >= 256 && k <= kDecMaxCodes && rows / kDecRowsPerBlock < 0x7fffffffLL &&
      aligned16(weight) && aligned16(out)) {
    // many rows: the codebook staged once per block of kDecRowsPerBlock rows
    const size_t smem = static_cast<size_t>(k) * 36;
    static bool configured[kMaxDevices] = {};
    allow_dynamic_smem(lfq_decode_tile_kernel, kDecMaxCodes * 36, configured);
    lfq_decode_tile_kernel<<<static_cast<unsigned>((rows + kDecRowsPerBlock - 1) / kDecRowsPerBlock),
                             kDecWarps * 32, smem, as_stream(stream)>>>(
        x, book_normed, code_norm, weight, b, t, static_cast<int>(k), out, indices);
    return launch_status(name);
  }
  lfq_decode_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, as_stream(stream)>>>(
      x, book_normed, code_norm, weight, b, t, k, out, indices);
  return launch_status(name);
}
