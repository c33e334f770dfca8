// Multi-stage residual vector quantizer (encode + decode in one kernel).
//
// For every row, stage s = 0..S-1 (the selection rule of
// fast_moss/quantizer.py:33-39 applied to a raw-L2 codebook):
//   norm   = sum_d r[d]^2                 sequential FMA, d ascending, from 0
//   dot_j  = sum_d (2 r[d]) * c_j[d]      sequential FMA, d ascending, from 0
//   dist_j = (norm - dot_j) + cnorm_j     cnorm_j = sum_d c_j[d]^2 (same order)
//   idx    = first j with NaN dist, else first j with minimal dist
//   r -= c_idx ; recon += c_idx           (recon starts at +0)
//
// B200 mapping (FP32 FFMA; every index bit-exact by construction):
//   * a CTA owns 56 rows for all S stages; their residual, reconstruction,
//     2r (k-major) and norms live in shared memory for the whole run;
//   * the codebook streams through two 66 KB shared buffers (256 codes x 64
//     dims k-major + their norms) filled by cp.async.bulk with an mbarrier,
//     one chunk ahead, across stage boundaries;
//   * 256 threads = 8 warps; a thread owns 7 rows x 8 codes of each chunk
//     (56 accumulators), fed by four conflict-free 16-byte shared loads per
//     k step for 56 FFMAs;
//   * the per-(row, code) epilogue keeps a running first-minimum in
//     registers; any NaN distance sends the row to an exact NaN-aware rescan
//     (rare: only non-finite or overflowing inputs produce NaN);
//   * 8192 rows -> 147 CTAs, i.e. one CTA per SM on a 148-SM B200.
#include "common.cuh"

#include <math_constants.h>

namespace moss {
namespace rvq {

constexpr int kDim = 64;
constexpr int kChunk = 256;
constexpr int kRows = 56;
constexpr int kRowsPerThread = 7;
constexpr int kThreads = 256;
constexpr int kTwCols = 64;   // 8 row groups x 8 slots (slot 7 unused)
constexpr int kRStride = 65;  // padded row stride of r / recon in shared memory

struct Smem {
  float chunk[2][kDim][kChunk];
  float cnorm[2][kChunk];
  float twice[kDim][kTwCols];
  float r[kRows][kRStride];
  float recon[kRows][kRStride];
  float norms[kRows];
  float md[4][kRows];
  int mi[4][kRows];
  int mnan[kRows];
  int sel[kRows];
  int slow_list[kRows];
  int slow_count;
  alignas(8) unsigned long long full[2];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the given phase; gives up after ~2 s and records a timeout.
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity) {
  return bounded_wait([&] { return mbar_try_wait(bar, parity); });
}

// Local column of a row in the k-major 2r array.
__device__ __forceinline__ int tw_col(int local_row) {
  return (local_row / kRowsPerThread) * 8 + (local_row % kRowsPerThread);
}

// Exact NaN-aware selection of one row by one warp over all k codes of a
// stage (raw [k][64] layout).  Same dot order as the fast path.
__device__ int exact_select(const Smem& sm, int local_row, float norm, const float* __restrict__ book,
                            const float* __restrict__ cnorm, int k, int lane) {
  const int col = tw_col(local_row);
  float best = CUDART_INF_F;
  int best_i = lane;
  int nan_i = INT_MAX;
  for (int j = lane; j < k; j += 32) {
    const float* c = book + static_cast<int64_t>(j) * kDim;
    float dot = 0.0f;
    for (int d = 0; d < kDim; ++d) dot = __fmaf_rn(sm.twice[d][col], c[d], dot);
    const float dist = __fadd_rn(__fsub_rn(norm, dot), cnorm[j]);
    if (dist != dist) {
      if (j < nan_i) nan_i = j;
    } else if (dist < best) {
      best = dist;
      best_i = j;
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, m);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, m);
    const int on = __shfl_xor_sync(0xffffffffu, nan_i, m);
    if (ob < best || (ob == best && oi < best_i)) {
      best = ob;
      best_i = oi;
    }
    nan_i = min(nan_i, on);
  }
  return nan_i != INT_MAX ? nan_i : best_i;
}

struct EncodeArgs {
  const float* x;
  const float* books;
  const float* packed;
  const float* code_norm;
  int32_t* codes;
  float* recon;
  float* residual_out;
  int64_t rows;
  int stages;
  int k;
  int kpad;
};

// Thread-per-row pass: norm (sequential FMA) and the k-major 2r column.
__device__ __forceinline__ void refresh_rows(Smem& sm, int tid) {
  if (tid < kRows) {
    const int col = tw_col(tid);
    float n = 0.0f;
#pragma unroll 8
    for (int d = 0; d < kDim; ++d) {
      const float v = sm.r[tid][d];
      n = __fmaf_rn(v, v, n);
      sm.twice[d][col] = __fmul_rn(2.0f, v);
    }
    sm.norms[tid] = n;
  }
}

__global__ void __launch_bounds__(kThreads, 1) rvq_encode_kernel(EncodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int wc = warp & 3;              // code quarter of each chunk
  const int g = (warp >> 2) * 4 + (lane >> 3);  // row group 0..7
  const int cgl = lane & 7;
  const int row0 = g * kRowsPerThread;
  const int cbase = wc * 64 + cgl * 4;  // codes cbase..+3 and cbase+32..+35
  const int64_t grow0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int nch = a.kpad / kChunk;
  const int total = a.stages * nch;
  constexpr uint32_t kChunkBytes = kDim * kChunk * sizeof(float);
  constexpr uint32_t kNormBytes = kChunk * sizeof(float);

  if (tid == 0) {
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.slow_count = 0;
  }
  __syncthreads();
  if (tid == 0) {
    for (int q = 0; q < 2 && q < total; ++q) {
      const int s = q / nch, j = q % nch;
      mbar_arrive_expect_tx(&sm.full[q], kChunkBytes + kNormBytes);
      bulk_copy_g2s(&sm.chunk[q][0][0], a.packed + (static_cast<int64_t>(s) * nch + j) * kDim * kChunk,
                    kChunkBytes, &sm.full[q]);
      bulk_copy_g2s(&sm.cnorm[q][0], a.code_norm + static_cast<int64_t>(s) * a.kpad + j * kChunk,
                    kNormBytes, &sm.full[q]);
    }
  }
  // Load the rows (warp per row, coalesced) and clear the reconstruction.
  for (int lr = warp; lr < kRows; lr += kThreads / 32) {
    const int64_t gr = grow0 + lr;
    for (int d = lane; d < kDim; d += 32) {
      sm.r[lr][d] = gr < a.rows ? a.x[gr * kDim + d] : 0.0f;
      sm.recon[lr][d] = 0.0f;
    }
  }
  if (tid < kRows) sm.mnan[tid] = 0;
  __syncthreads();
  refresh_rows(sm, tid);
  __syncthreads();

  for (int s = 0; s < a.stages; ++s) {
    float nrm[kRowsPerThread], best[kRowsPerThread];
    int bidx[kRowsPerThread];
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      nrm[i] = sm.norms[row0 + i];
      best[i] = CUDART_INF_F;
      bidx[i] = 0;
    }
    int anynan = 0;

    for (int j = 0; j < nch; ++j) {
      const int q = s * nch + j;
      const int buf = q & 1;
      // All threads agree before leaving, so no thread exits ahead of a barrier.
      const int timed_out = !mbar_wait_bounded(&sm.full[buf], (q >> 1) & 1);
      if (__syncthreads_or(timed_out)) return;
      float acc[kRowsPerThread][8];
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) acc[i][jj] = 0.0f;

      const float* A = &sm.twice[0][g * 8];
      const float* B = &sm.chunk[buf][0][cbase];
#pragma unroll 4
      for (int kk = 0; kk < kDim; ++kk) {
        const float4 a0 = *reinterpret_cast<const float4*>(A + kk * kTwCols);
        const float4 a1 = *reinterpret_cast<const float4*>(A + kk * kTwCols + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(B + kk * kChunk);
        const float4 b1 = *reinterpret_cast<const float4*>(B + kk * kChunk + 32);
        const float av[7] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i)
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) acc[i][jj] = __fmaf_rn(av[i], bv[jj], acc[i][jj]);
      }
      // Distances and the running first minimum, codes in ascending order.
      float cn[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) cn[jj] = sm.cnorm[buf][cbase + (jj < 4 ? jj : 28 + jj)];
      const int code0 = j * kChunk + cbase;
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float dist = __fadd_rn(__fsub_rn(nrm[i], acc[i][jj]), cn[jj]);
          if (dist < best[i]) {
            best[i] = dist;
            bidx[i] = code0 + (jj < 4 ? jj : 28 + jj);
          }
          anynan |= (dist != dist);
        }
      }
      __syncthreads();  // everyone is done with this buffer
      if (tid == 0 && q + 2 < total) {
        const int qn = q + 2, sn = qn / nch, jn = qn % nch;
        mbar_arrive_expect_tx(&sm.full[buf], kChunkBytes + kNormBytes);
        bulk_copy_g2s(&sm.chunk[buf][0][0],
                      a.packed + (static_cast<int64_t>(sn) * nch + jn) * kDim * kChunk, kChunkBytes,
                      &sm.full[buf]);
        bulk_copy_g2s(&sm.cnorm[buf][0], a.code_norm + static_cast<int64_t>(sn) * a.kpad + jn * kChunk,
                      kNormBytes, &sm.full[buf]);
      }
    }

    // (a) merge the 8 code lanes of each row group, then publish per quarter.
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) anynan |= __shfl_xor_sync(0xffffffffu, anynan, m);
#pragma unroll
    for (int i = 0; i < kRowsPerThread; ++i) {
      float d = best[i];
      int ix = bidx[i];
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        const float od = __shfl_xor_sync(0xffffffffu, d, m);
        const int oi = __shfl_xor_sync(0xffffffffu, ix, m);
        if (od < d || (od == d && oi < ix)) {
          d = od;
          ix = oi;
        }
      }
      if (cgl == 0) {
        sm.md[wc][row0 + i] = d;
        sm.mi[wc][row0 + i] = ix;
        if (anynan) atomicOr(&sm.mnan[row0 + i], 1);
      }
    }
    __syncthreads();
    // (b) final merge across the four code quarters; queue NaN rows.
    if (tid < kRows) {
      float d = sm.md[0][tid];
      int ix = sm.mi[0][tid];
#pragma unroll
      for (int w = 1; w < 4; ++w) {
        const float od = sm.md[w][tid];
        const int oi = sm.mi[w][tid];
        if (od < d || (od == d && oi < ix)) {
          d = od;
          ix = oi;
        }
      }
      sm.sel[tid] = ix;
      if (sm.mnan[tid]) {
        const int slot = atomicAdd(&sm.slow_count, 1);
        sm.slow_list[slot] = tid;
      }
      sm.mnan[tid] = 0;
    }
    __syncthreads();
    // (c) exact rescan of the rows that saw a NaN distance.
    const int slow = sm.slow_count;
    if (slow > 0) {
      const float* book = a.books + static_cast<int64_t>(s) * a.k * kDim;
      const float* cnorm = a.code_norm + static_cast<int64_t>(s) * a.kpad;
      for (int i = warp; i < slow; i += kThreads / 32) {
        const int lr = sm.slow_list[i];
        const int ix = exact_select(sm, lr, sm.norms[lr], book, cnorm, a.k, lane);
        if (lane == 0) sm.sel[lr] = ix;
      }
      __syncthreads();
    }
    // (d) residual update, reconstruction, codes.
    {
      const float* book = a.books + static_cast<int64_t>(s) * a.k * kDim;
      for (int lr = warp; lr < kRows; lr += kThreads / 32) {
        const int ix = sm.sel[lr];
        const float* c = book + static_cast<int64_t>(ix) * kDim;
        for (int d = lane; d < kDim; d += 32) {
          const float cv = c[d];
          sm.r[lr][d] = __fsub_rn(sm.r[lr][d], cv);
          sm.recon[lr][d] = __fadd_rn(sm.recon[lr][d], cv);
        }
        const int64_t gr = grow0 + lr;
        if (lane == 0 && gr < a.rows) a.codes[static_cast<int64_t>(s) * a.rows + gr] = ix;
      }
    }
    __syncthreads();
    if (tid == 0) sm.slow_count = 0;
    refresh_rows(sm, tid);
    __syncthreads();
  }

  for (int lr = warp; lr < kRows; lr += kThreads / 32) {
    const int64_t gr = grow0 + lr;
    if (gr >= a.rows) break;
    for (int d = lane; d < kDim; d += 32) {
      a.recon[gr * kDim + d] = sm.recon[lr][d];
      if (a.residual_out) a.residual_out[gr * kDim + d] = sm.r[lr][d];
    }
  }
}

// Tensor-core tile image of 256 codes (73728 bytes): the 64 dims in a K-major
// 128-byte-swizzled layout (16-byte chunk index XOR n % 8, 8-code groups 1024
// bytes apart, the two 32-dim halves 32 KB apart), then an 8-wide K block
// without swizzle (8-code x 16-byte core matrices, K halves 128 bytes apart,
// 8-code groups 256 bytes apart) holding {-cnorm, 0 x 7} per code.
constexpr int kTcMainBytes = kChunk * kDim * 4;
constexpr int kTcTileBytes = kTcMainBytes + kChunk * 8 * 4;

__device__ __forceinline__ uint32_t tc_image_offset(int n, int k) {
  const int kk = k & 31;
  return static_cast<uint32_t>(k >> 5) * 32768u + static_cast<uint32_t>(n >> 3) * 1024u +
         static_cast<uint32_t>(n & 7) * 128u +
         static_cast<uint32_t>(((kk >> 2) ^ (n & 7)) << 4) + static_cast<uint32_t>(kk & 3) * 4u;
}
__device__ __forceinline__ uint32_t tc_extra_offset(int n, int k) {
  return kTcMainBytes + static_cast<uint32_t>(n >> 3) * 256u + static_cast<uint32_t>(k >> 2) * 128u +
         static_cast<uint32_t>(n & 7) * 16u + static_cast<uint32_t>(k & 3) * 4u;
}

// Codebook preparation, one CTA per (256-code chunk, stage).  The chunk's
// codewords are staged in shared memory with coalesced 16-byte loads (row
// stride 65 floats, so both row-wise and column-wise reads are free of bank
// conflicts); every output is then written in its own linear order, so all
// global stores are coalesced: the code norms (sequential FMA, d ascending,
// from +0; +inf for padding codes), the k-major copy read by the FFMA
// kernel, and the 128-byte-swizzled tensor-core tile image with its extra
// K block {-cnorm, 0 x 7} (-inf for padding codes).
constexpr int kPrepStride = kDim + 1;
constexpr size_t kPrepSmem = (static_cast<size_t>(kChunk) * kPrepStride + kChunk) * sizeof(float);

__global__ void __launch_bounds__(256) rvq_prepare_kernel(const float* __restrict__ books, int k,
                                                          int kpad, int stages,
                                                          float* __restrict__ code_norm,
                                                          float* __restrict__ packed) {
  extern __shared__ float prep_smem[];
  float* rows = prep_smem;                         // [kChunk][kPrepStride]
  float* norms = prep_smem + kChunk * kPrepStride;  // [kChunk]
  const int ch = blockIdx.x, s = blockIdx.y;
  const int nch = kpad / kChunk;
  const int base = ch * kChunk;
  const int valid = min(kChunk, k - base);  // >= 1: kpad < k + kChunk
  const float* book = books + (static_cast<int64_t>(s) * k + base) * kDim;
  // stage: float4 loads when the chunk's rows are 16-byte aligned (always,
  // since kDim floats per row, when `books` itself is)
  if ((reinterpret_cast<uintptr_t>(books) & 15u) == 0) {
    for (int f = threadIdx.x; f < valid * (kDim / 4); f += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(book)[f];
      const int n = f / (kDim / 4), d = (f % (kDim / 4)) * 4;
      float* dst = rows + n * kPrepStride + d;
      dst[0] = v.x; dst[1] = v.y; dst[2] = v.z; dst[3] = v.w;
    }
  } else {
    for (int f = threadIdx.x; f < valid * kDim; f += blockDim.x)
      rows[(f / kDim) * kPrepStride + f % kDim] = book[f];
  }
  for (int f = threadIdx.x + valid * kDim; f < kChunk * kDim; f += blockDim.x)
    rows[(f / kDim) * kPrepStride + f % kDim] = 0.0f;
  __syncthreads();
  {
    const int n = threadIdx.x;  // blockDim.x == kChunk
    float nv = CUDART_INF_F;
    if (n < valid) {
      nv = 0.0f;
      for (int d = 0; d < kDim; ++d) {
        const float v = rows[n * kPrepStride + d];
        nv = __fmaf_rn(v, v, nv);
      }
    }
    norms[n] = nv;
    code_norm[static_cast<int64_t>(s) * kpad + base + n] = nv;
  }
  __syncthreads();
  // k-major copy [stage][chunk][d][kChunk]
  float* kmajor = packed + (static_cast<int64_t>(s) * nch + ch) * kDim * kChunk;
  for (int f = threadIdx.x; f < kDim * kChunk; f += blockDim.x)
    kmajor[f] = rows[(f % kChunk) * kPrepStride + f / kChunk];
  // tensor-core tile image, walked in its byte order (inverse of
  // tc_image_offset / tc_extra_offset)
  float* tile = packed + static_cast<int64_t>(stages) * kpad * kDim +
                (static_cast<int64_t>(s) * nch + ch) * (kTcTileBytes / 4);
  for (int f = threadIdx.x; f < kTcMainBytes / 4; f += blockDim.x) {
    const int o = f * 4;
    const int kb = o >> 15, ng = (o >> 10) & 31, nr = (o >> 7) & 7, c16 = (o >> 4) & 7,
              w = (o >> 2) & 3;
    const int n = ng * 8 + nr, kk = kb * 32 + (((c16 ^ nr) << 2) | w);
    tile[f] = rows[n * kPrepStride + kk];
  }
  for (int f = threadIdx.x; f < kChunk * 8; f += blockDim.x) {
    const int o = f * 4;
    const int ng = o >> 8, eb = (o >> 7) & 1, nr = (o >> 4) & 7, w = (o >> 2) & 3;
    const int n = ng * 8 + nr, e = eb * 4 + w;
    // padding codes screen at -inf, below every real (finite) code
    tile[kTcMainBytes / 4 + f] = e ? 0.0f : (n < valid ? -norms[n] : -CUDART_INF_F);
  }
}

// Per-stage stats from the code norms: {max finite norm (from 0), 1 if any
// real code's norm is non-finite -- which is the case exactly when one of
// its values is non-finite or its squares overflow -- , 0, 0}.
__global__ void __launch_bounds__(256) rvq_stats_kernel(const float* __restrict__ code_norm,
                                                        int k, int kpad,
                                                        float* __restrict__ stats) {
  __shared__ float red_max[256];
  __shared__ int red_bad[256];
  const int s = blockIdx.x;
  float mx = 0.0f;
  int bad = 0;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const float n = code_norm[static_cast<int64_t>(s) * kpad + j];
    if (!isfinite(n)) bad = 1;
    else mx = fmaxf(mx, n);
  }
  red_max[threadIdx.x] = mx;
  red_bad[threadIdx.x] = bad;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      red_max[threadIdx.x] = fmaxf(red_max[threadIdx.x], red_max[threadIdx.x + w]);
      red_bad[threadIdx.x] |= red_bad[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    stats[s * 4 + 0] = red_max[0];
    stats[s * 4 + 1] = red_bad[0] ? 1.0f : 0.0f;
    stats[s * 4 + 2] = 0.0f;
    stats[s * 4 + 3] = 0.0f;
  }
}

// recon[r][d] = sum_s book_s[codes[s][r]][d], stage order, from +0.
__global__ void __launch_bounds__(256) rvq_decode_kernel(const int32_t* __restrict__ codes,
                                                         int64_t rows, const float* __restrict__ books,
                                                         int stages, int k, int d,
                                                         float* __restrict__ recon) {
  const int64_t n = rows * d;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / d;
    const int64_t dd = i - r * d;
    float acc = 0.0f;
    for (int s = 0; s < stages; ++s) {
      const int32_t c = codes[static_cast<int64_t>(s) * rows + r];
      if (c < 0 || c >= k) {
        record_device_error(MOSS_ERR_VALUE);
        continue;
      }
      acc = __fadd_rn(acc, books[(static_cast<int64_t>(s) * k + c) * d + dd]);
    }
    recon[i] = acc;
  }
}

}  // namespace rvq
}  // namespace moss

using namespace moss;

extern "C" int64_t moss_rvq_packed_floats(int64_t stages, int64_t k, int64_t d) {
  if (stages < 1 || k < 1 || d < 1) return 0;
  const int64_t kpad = (k + rvq::kChunk - 1) / rvq::kChunk * rvq::kChunk;
  // FFMA k-major copy, then the tensor-core tile images
  return stages * kpad * d + stages * (kpad / rvq::kChunk) * (rvq::kTcTileBytes / 4);
}

extern "C" int moss_rvq_prepare_codebooks(const float* books, int64_t stages, int64_t k, int64_t d,
                                          float* code_norm, float* packed, float* stats,
                                          void* stream) {
  const char* name = "moss_rvq_prepare_codebooks";
  if (stages < 1 || k < 1) return fail(MOSS_ERR_VALUE, "%s: need >= 1 stage and >= 1 code", name);
  if (d != rvq::kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only 64-dim codewords are supported", name);
  if (k > 65536 || stages > 65535) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many codes or stages", name);
  if (!books || !code_norm || !packed || !stats) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  const int64_t kpad = (k + rvq::kChunk - 1) / rvq::kChunk * rvq::kChunk;
  static bool smem_set[kMaxDevices] = {false};
  allow_dynamic_smem(rvq::rvq_prepare_kernel, rvq::kPrepSmem, smem_set);
  const dim3 grid(static_cast<unsigned>(kpad / rvq::kChunk), static_cast<unsigned>(stages));
  rvq::rvq_prepare_kernel<<<grid, rvq::kChunk, rvq::kPrepSmem, as_stream(stream)>>>(
      books, static_cast<int>(k), static_cast<int>(kpad), static_cast<int>(stages), code_norm,
      packed);
  rvq::rvq_stats_kernel<<<static_cast<unsigned>(stages), 256, 0, as_stream(stream)>>>(
      code_norm, static_cast<int>(k), static_cast<int>(kpad), stats);
  return launch_status(name);
}

extern "C" int moss_rvq_encode_ffma(const float* x, int64_t rows, int64_t d, const float* books,
                                    const float* packed, const float* code_norm,
                                    const float* stats, int64_t stages, int64_t k, int32_t* codes,
                                    float* recon, float* residual_out, void* stream) {
  const char* name = "moss_rvq_encode_ffma";
  (void)stats;
  if (rows < 0 || stages < 1 || k < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (d != rvq::kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only 64-dim codewords are supported", name);
  if (k > 65536 || stages > 65535) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many codes or stages", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !books || !packed || !code_norm || !codes || !recon)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(packed) || !aligned16(code_norm))
    return fail(MOSS_ERR_VALUE, "%s: packed codebook and norms must be 16-byte aligned", name);
  const int64_t grid = (rows + rvq::kRows - 1) / rvq::kRows;
  if (grid > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows", name);
  const int kpad = static_cast<int>((k + rvq::kChunk - 1) / rvq::kChunk * rvq::kChunk);
  const size_t smem = sizeof(rvq::Smem);
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(rvq::rvq_encode_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return fail(MOSS_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  rvq::EncodeArgs a{x, books, packed, code_norm, codes, recon, residual_out, rows,
                    static_cast<int>(stages), static_cast<int>(k), kpad};
  rvq::rvq_encode_kernel<<<static_cast<unsigned>(grid), rvq::kThreads, smem, as_stream(stream)>>>(a);
  return launch_status(name);
}

extern "C" int moss_rvq_decode(const int32_t* codes, int64_t rows, const float* books,
                               int64_t stages, int64_t k, int64_t d, float* recon, void* stream) {
  const char* name = "moss_rvq_decode";
  if (rows < 0 || stages < 1 || k < 1 || d < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (rows == 0) return MOSS_OK;
  if (!codes || !books || !recon) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  const int64_t n = rows * d;
  int64_t grid = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (grid > cap) grid = cap;
  rvq::rvq_decode_kernel<<<static_cast<unsigned>(grid), 256, 0, as_stream(stream)>>>(
      codes, rows, books, static_cast<int>(stages), static_cast<int>(k), static_cast<int>(d), recon);
  return launch_status(name);
}
