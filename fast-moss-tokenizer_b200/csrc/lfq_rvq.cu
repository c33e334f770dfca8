// Multi-stage LFQ quantizer of the real codec: all stages in one kernel,
// the residual kept in shared memory from the first stage to the last.
//
// The reference runs one stage of the upstream quantizer (called at
// fast_moss/v2_codec.py:45) as separate launches: the 8-wide input
// projection, `prepare` (fast_moss/quantizer_prepare.py:111-157), the FP32
// GEMM of the dot products and `select` (fast_moss/v2_runtime.py:143-181,
// fast_moss/quantizer.py:52-108), the output projection and the residual
// update -- about six launches per stage, 32 stages per frame.  The stage
// loop and the projections live in the upstream module, which is not
// available, so their summation order is defined here:
//   per frame (b, t), r[d] = x[b, d, t]; for every stage s:
//     z_j  = dot_lanes(w_in[s, j, :], r) + b_in[s, j]            (j = 0..7)
//            dot_lanes: 32 partial sums p_l = sequential FMA from +0 over
//            d = l, l + 32, ...; then for off = 16, 8, 4, 2, 1:
//            p_l = p_l + p_(l xor off); the result is p_0
//     LFQ decode of z as a [B, 8, T] latent (the reference's prepare order,
//            transposed when B == 1 and T > 1; dots = twice . book_k as a
//            product then 7 FMAs; distance = (norm - dot) + code_norm;
//            first NaN, else first minimum)
//     c    = weight[s, index, :]                                   (raw)
//     o_d  = (FMA chain over j = 0..7 of w_out[s, d, j] c_j from +0) + b_out[s, d]
//     r_d  = r_d - o_d ;  codes[s, b * T + t] = index
// A CTA takes F frames (F = 1, 4 or 16 by the number of frames) for all
// stages, 256 threads: each warp forms a block of the z_j x frames (4 x 4
// at 16 frames, so each residual read serves four outputs and each weight
// read four frames), each thread scores codes tid, tid + 256, ... for every
// frame (a block reduction picks the winner), each thread updates dims
// tid, tid + 256, ... of every frame.  The stage weights are read through
// L1/L2 (about 120 KB per stage at D = 1280, K = 1024).
#include "lfq.cuh"

#include <math_constants.h>

namespace moss {
namespace lrvq {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxDim = 2048;
constexpr int kMaxCodes = 65536;
constexpr int kGroup = 4;  // codes per thread held in registers at a time
constexpr int kOutGroup = 8;  // output dims per thread held in registers at a time
constexpr int kInBlock = 10;  // input-projection dims per lane loaded ahead

struct Args {
  const float* x;       // [B, D, T]
  const float* w_in;    // [S, 8, D]
  const float* b_in;    // [S, 8]
  const float* book;    // [S, K, 8] normalised codebooks
  const float* cnorm;   // [S, K]
  const float* weight;  // [S, K, 8] raw codebooks
  const float* w_out;   // [S, D, 8]
  const float* b_out;   // [S, D]
  int64_t* codes;       // [S, B * T]
  float* residual;      // [B, D, T] or null
  int64_t t, rows;
  int d, stages, k;
  int transposed;
};

__host__ __device__ inline size_t smem_bytes(int f, int d) {
  // r [F][D], tw [F][8], norm [F], z [F][8], chosen codeword [F][8],
  // per-warp picks [F][warps] x (best, index, nan index), selection [F]
  return static_cast<size_t>(f) * (d + 8 + 1 + 8 + 8 + 3 * kWarps + 1) * 4;
}

__device__ __forceinline__ Pick32 pick_shfl(const Pick32& p, int o) {
  return Pick32{__shfl_xor_sync(0xffffffffu, p.best, o), __shfl_xor_sync(0xffffffffu, p.best_i, o),
                __shfl_xor_sync(0xffffffffu, p.nan_i, o)};
}
__device__ __forceinline__ void pick_merge(Pick32& p, const Pick32& o) {
  if (o.best < p.best || (o.best == p.best && o.best_i < p.best_i)) {
    p.best = o.best;
    p.best_i = o.best_i;
  }
  if (o.nan_i < p.nan_i) p.nan_i = o.nan_i;
}
// picks [0, M) -> [0, M / 2): the lanes with bit O set keep the upper half.
template <int M, int O, int N>
__device__ __forceinline__ void pick_halve(Pick32 (&pk)[N], int lane) {
  const bool up = (lane & O) != 0;
#pragma unroll
  for (int i = 0; i < M / 2; ++i) {
    const Pick32 lo = pk[i], hi = pk[i + M / 2];
    Pick32 keep = up ? hi : lo;
    pick_merge(keep, pick_shfl(up ? lo : hi, O));
    pk[i] = keep;
  }
}

template <int F>
__global__ void __launch_bounds__(kThreads, 2) lfq_rvq_kernel(const Args a) {
  extern __shared__ float sm[];
  const int D = a.d;
  float* r = sm;                        // [F][D]
  float* tw = r + F * D;                // [F][8]
  float* nrm = tw + F * 8;              // [F]
  float* z = nrm + F;                   // [F][8]
  float* cw = z + F * 8;                // [F][8]
  float* pbest = cw + F * 8;            // [F][warps]
  int* pidx = reinterpret_cast<int*>(pbest + F * kWarps);
  int* pnan = pidx + F * kWarps;
  int* sel = pnan + F * kWarps;         // [F]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * F;
  const int nf = static_cast<int>(a.rows - row0 < F ? a.rows - row0 : F);
  for (int i = tid; i < F * D; i += kThreads) {
    const int f = i / D, dd = i - f * D;
    float v = 0.0f;
    if (f < nf) {
      const int64_t row = row0 + f, bi = row / a.t, ti = row - bi * a.t;
      v = a.x[(bi * D + dd) * a.t + ti];
    }
    r[i] = v;
  }
  // 2e, norms and codewords of frames past the CTA's rows stay zero: the
  // distance and output phases run over all F frames without a guard, and
  // those frames' results are never used
  for (int i = tid; i < F * 25; i += kThreads) tw[i] = 0.0f;  // tw, nrm, z, cw
  __syncthreads();
  for (int s = 0; s < a.stages; ++s) {
    // ---- input projection: warp -> JW outputs z_j of FW frames (16 frames:
    // a 4 x 4 block, so each residual value read from shared memory serves
    // four outputs and each weight four frames); per output the order is
    // the same for every blocking: lane partial sums over dims lane,
    // lane + 32, ... from +0, then added pairwise across the lanes
    {
      constexpr int JW = F == 16 ? 4 : 1;
      constexpr int FW = F == 16 ? 4 : F;
      static_assert((8 / JW) * (F / FW) == kWarps, "one block per warp");
      const int j0 = (warp % (8 / JW)) * JW, f0 = (warp / (8 / JW)) * FW;
      const float* wrow = a.w_in + (static_cast<int64_t>(s) * 8 + j0) * D;
      float acc[JW][FW];
#pragma unroll
      for (int jj = 0; jj < JW; ++jj)
#pragma unroll
        for (int ff = 0; ff < FW; ++ff) acc[jj][ff] = 0.0f;
      // blocks of kInBlock dims per lane: the block's weight loads are all
      // issued before its multiply-adds, one round trip per block
      for (int db = 0; db < D; db += 32 * kInBlock) {
        float wv[kInBlock][JW];
#pragma unroll
        for (int u = 0; u < kInBlock; ++u) {
          const int dd = db + lane + 32 * u;
#pragma unroll
          for (int jj = 0; jj < JW; ++jj) wv[u][jj] = dd < D ? __ldg(wrow + jj * D + dd) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kInBlock; ++u) {
          const int dd = db + lane + 32 * u;
          if (dd < D) {
#pragma unroll
            for (int ff = 0; ff < FW; ++ff) {
              const float rv = r[(f0 + ff) * D + dd];
#pragma unroll
              for (int jj = 0; jj < JW; ++jj) acc[jj][ff] = __fmaf_rn(wv[u][jj], rv, acc[jj][ff]);
            }
          }
        }
      }
#pragma unroll
      for (int jj = 0; jj < JW; ++jj) {
#pragma unroll
        for (int ff = 0; ff < FW; ++ff) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
            acc[jj][ff] = __fadd_rn(acc[jj][ff], __shfl_xor_sync(0xffffffffu, acc[jj][ff], off));
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int jj = 0; jj < JW; ++jj) {
          const float bj = a.b_in[s * 8 + j0 + jj];
#pragma unroll
          for (int ff = 0; ff < FW; ++ff) z[(f0 + ff) * 8 + j0 + jj] = __fadd_rn(acc[jj][ff], bj);
        }
      }
    }
    __syncthreads();
    // ---- prepare (the reference's orders): thread f prepares frame f
    if (tid < nf) {
      float v[8], esq[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = z[tid * 8 + q];
      float denom = __fsqrt_rn(sum_squares(v, a.transposed != 0));
      denom = denom < 1.0e-12f ? 1.0e-12f : denom;  // a NaN compares false and stays
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float e = __fdiv_rn(v[q], denom);
        tw[tid * 8 + q] = __fmul_rn(2.0f, e);
        esq[q] = __fmul_rn(e, e);
      }
      nrm[tid] = sum8(esq, a.transposed != 0);
    }
    __syncthreads();
    // ---- distances and the first-NaN / first-minimum pick per frame
    {
      Pick32 pk[F];
#pragma unroll
      for (int f = 0; f < F; ++f) {
        pk[f].best = CUDART_INF_F;
        pk[f].best_i = tid < a.k ? tid : INT_MAX;
        pk[f].nan_i = INT_MAX;
      }
      const float* book = a.book + static_cast<int64_t>(s) * a.k * 8;
      const float* cn = a.cnorm + static_cast<int64_t>(s) * a.k;
      // kGroup codes of this thread (tid, tid + 256, ...) in registers, then
      // every frame's 2e read once per group; each frame still sees its
      // codes in ascending order
      for (int j0 = tid; j0 < a.k; j0 += kGroup * kThreads) {
        float4 c0[kGroup], c1[kGroup];
        float cnj[kGroup];
#pragma unroll
        for (int m = 0; m < kGroup; ++m) {
          const int j = j0 + m * kThreads;
          const int jj = j < a.k ? j : j0;
          c0[m] = __ldg(reinterpret_cast<const float4*>(book + static_cast<int64_t>(jj) * 8));
          c1[m] = __ldg(reinterpret_cast<const float4*>(book + static_cast<int64_t>(jj) * 8 + 4));
          cnj[m] = __ldg(cn + jj);
        }
#pragma unroll
        for (int f = 0; f < F; ++f) {
          {
            float t8[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) t8[q] = tw[f * 8 + q];
            const float nf_ = nrm[f];
#pragma unroll
            for (int m = 0; m < kGroup; ++m) {
              const int j = j0 + m * kThreads;
              if (j < a.k) {
                float dot = __fmul_rn(t8[0], c0[m].x);
                dot = __fmaf_rn(t8[1], c0[m].y, dot);
                dot = __fmaf_rn(t8[2], c0[m].z, dot);
                dot = __fmaf_rn(t8[3], c0[m].w, dot);
                dot = __fmaf_rn(t8[4], c1[m].x, dot);
                dot = __fmaf_rn(t8[5], c1[m].y, dot);
                dot = __fmaf_rn(t8[6], c1[m].z, dot);
                dot = __fmaf_rn(t8[7], c1[m].w, dot);
                pick32_push(pk[f], __fadd_rn(__fsub_rn(nf_, dot), cnj[m]), j);
              }
            }
          }
        }
      }
      // Warp reduction of the F frames' picks, scattered over the lanes:
      // each halving step keeps half of the frames and merges in the other
      // lane's copy of them, until every lane holds one frame (16 frames:
      // lanes differing in bit 0 share one; 4 frames: bits 0-2), then a
      // plain butterfly over the remaining lane bits.  The merge (lexicographic
      // minimum of (best, index), minimum NaN index) is associative and
      // commutative, so the winner is the same as over any other tree.
      int frame = 0;
      if constexpr (F == 16) {
        pick_halve<16, 16>(pk, lane);
        pick_halve<8, 8>(pk, lane);
        pick_halve<4, 4>(pk, lane);
        pick_halve<2, 2>(pk, lane);
        pick_merge(pk[0], pick_shfl(pk[0], 1));
        frame = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                ((lane >> 1) & 1);
      } else if constexpr (F == 4) {
        pick_halve<4, 16>(pk, lane);
        pick_halve<2, 8>(pk, lane);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) pick_merge(pk[0], pick_shfl(pk[0], o));
        frame = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
      } else {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) pick_merge(pk[0], pick_shfl(pk[0], o));
      }
      constexpr int kShare = F == 16 ? 1 : (F == 4 ? 7 : 31);  // lanes holding one frame
      if ((lane & kShare) == 0) {
        pbest[frame * kWarps + warp] = pk[0].best;
        pidx[frame * kWarps + warp] = pk[0].best_i;
        pnan[frame * kWarps + warp] = pk[0].nan_i;
      }
    }
    __syncthreads();
    if (tid < nf) {
      float best = pbest[tid * kWarps];
      int bi = pidx[tid * kWarps], ni = pnan[tid * kWarps];
      for (int w = 1; w < kWarps; ++w) {
        const float ob = pbest[tid * kWarps + w];
        const int oi = pidx[tid * kWarps + w], on = pnan[tid * kWarps + w];
        if (ob < best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
        if (on < ni) ni = on;
      }
      const int idx = ni != INT_MAX ? ni : bi;
      sel[tid] = idx;
      a.codes[static_cast<int64_t>(s) * a.rows + row0 + tid] = idx;
      const float* c = a.weight + (static_cast<int64_t>(s) * a.k + idx) * 8;
#pragma unroll
      for (int q = 0; q < 8; ++q) cw[tid * 8 + q] = c[q];
    }
    __syncthreads();
    // ---- output projection and residual update: thread -> dims tid, tid + 256, ...
    // kOutGroup dims of this thread (tid, tid + 256, ...) with their weights in
    // registers, then every frame's codeword read once per group
    for (int d0 = tid; d0 < D; d0 += kOutGroup * kThreads) {
      float4 w0[kOutGroup], w1[kOutGroup];
      float bo[kOutGroup];
#pragma unroll
      for (int m = 0; m < kOutGroup; ++m) {
        const int dd = d0 + m * kThreads;
        const int de = dd < D ? dd : d0;
        const float* wo = a.w_out + (static_cast<int64_t>(s) * D + de) * 8;
        w0[m] = __ldg(reinterpret_cast<const float4*>(wo));
        w1[m] = __ldg(reinterpret_cast<const float4*>(wo + 4));
        bo[m] = __ldg(a.b_out + static_cast<int64_t>(s) * D + de);
      }
#pragma unroll
      for (int f = 0; f < F; ++f) {
        {
          float c[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) c[q] = cw[f * 8 + q];
#pragma unroll
          for (int m = 0; m < kOutGroup; ++m) {
            const int dd = d0 + m * kThreads;
            if (dd < D) {
              float o = __fmaf_rn(w0[m].x, c[0], 0.0f);
              o = __fmaf_rn(w0[m].y, c[1], o);
              o = __fmaf_rn(w0[m].z, c[2], o);
              o = __fmaf_rn(w0[m].w, c[3], o);
              o = __fmaf_rn(w1[m].x, c[4], o);
              o = __fmaf_rn(w1[m].y, c[5], o);
              o = __fmaf_rn(w1[m].z, c[6], o);
              o = __fmaf_rn(w1[m].w, c[7], o);
              r[f * D + dd] = __fsub_rn(r[f * D + dd], __fadd_rn(o, bo[m]));
            }
          }
        }
      }
    }
    __syncthreads();
  }
  if (a.residual) {
    for (int i = tid; i < nf * D; i += kThreads) {
      const int f = i / D, dd = i - f * D;
      const int64_t row = row0 + f, bi = row / a.t, ti = row - bi * a.t;
      a.residual[(bi * D + dd) * a.t + ti] = r[i];
    }
  }
}

}  // namespace lrvq
}  // namespace moss

using namespace moss;

extern "C" int moss_lfq_rvq_encode(const float* x, int64_t b, int64_t d, int64_t t, int64_t stages,
                                   int64_t k, const float* w_in, const float* b_in,
                                   const float* book_normed, const float* code_norm,
                                   const float* weight, const float* w_out, const float* b_out,
                                   int64_t* codes, float* residual_out, void* stream) {
  const char* name = "moss_lfq_rvq_encode";
  if (b < 0 || t < 0 || d < 1 || stages < 1 || k < 1)
    return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (d > lrvq::kMaxDim || k > lrvq::kMaxCodes)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: at most %d channels and %d codes", name,
                lrvq::kMaxDim, lrvq::kMaxCodes);
  const int64_t rows = b * t;
  if (rows == 0) return MOSS_OK;
  if (!x || !w_in || !b_in || !book_normed || !code_norm || !weight || !w_out || !b_out || !codes)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(book_normed) || !aligned16(w_out))
    return fail(MOSS_ERR_VALUE, "%s: the codebooks and output projections must be 16-byte "
                "aligned", name);
  const int f = rows >= static_cast<int64_t>(sm_count()) * 16 ? 16
                : (rows >= static_cast<int64_t>(sm_count()) * 4 ? 4 : 1);
  const int64_t grid = (rows + f - 1) / f;
  if (grid > 0x7fffffffLL || stages > 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too many frames", name);
  lrvq::Args a{x, w_in, b_in, book_normed, code_norm, weight, w_out, b_out, codes, residual_out,
               t, rows, static_cast<int>(d), static_cast<int>(stages), static_cast<int>(k),
               (b == 1 && t > 1) ? 1 : 0};
  const size_t smem = lrvq::smem_bytes(f, static_cast<int>(d));
  cudaStream_t st = as_stream(stream);
  static bool configured[3][kMaxDevices] = {};
  switch (f) {
    case 16:
      allow_dynamic_smem(lrvq::lfq_rvq_kernel<16>, lrvq::smem_bytes(16, lrvq::kMaxDim),
                         configured[0]);
      lrvq::lfq_rvq_kernel<16><<<static_cast<unsigned>(grid), lrvq::kThreads, smem, st>>>(a);
      break;
    case 4:
      allow_dynamic_smem(lrvq::lfq_rvq_kernel<4>, lrvq::smem_bytes(4, lrvq::kMaxDim),
                         configured[1]);
      lrvq::lfq_rvq_kernel<4><<<static_cast<unsigned>(grid), lrvq::kThreads, smem, st>>>(a);
      break;
    default:
      allow_dynamic_smem(lrvq::lfq_rvq_kernel<1>, lrvq::smem_bytes(1, lrvq::kMaxDim),
                         configured[2]);
      lrvq::lfq_rvq_kernel<1><<<static_cast<unsigned>(grid), lrvq::kThreads, smem, st>>>(a);
  }
  return launch_status(name);
}
