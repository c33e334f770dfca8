// Multi-stage residual VQ with tensor-core screening (tcgen05, TF32) and an
// exact FP32 rerank.  Produces exactly the codes of the FFMA kernel in
// rvq.cu (same documented arithmetic), typically ~10x faster.
//
// Why the indices stay exact.  For row r and code j let
//   key_j   = cnorm_j - A_j,  A_j = TF32 tensor-core value of sum_d 2r_d c_jd
//   exact_j = dist_j - norm   (real-number difference; dist_j in the pinned
//                              FP32 order of rvq.cu)
// TF32 keeps 10 fraction bits (relative error < 2^-10 per operand), so
// |A_j - sum 2r_d c_jd| < 2^-9 sum|2r_d c_jd| (+ accumulation rounding), and
// the pinned FP32 dot and the two FP32 roundings of dist add < 2^-20 (norm +
// cnorm_max + |dot|).  With S = |2r| (Euclidean), C = max_j |c_j|:
//   |key_j - exact_j| <= M = 2^-8 S C + 2^-20 (norm + cnorm_max) + 2^-100
// (a 2x margin over the TF32 bound).  Every minimiser j* of dist then has
// key_j* <= min_i key_i + 2M, so the candidates {j : key_j <= min key + 2M}
// contain all of them; a single candidate is the answer, several are
// reranked with the exact pinned arithmetic (first minimum wins).  Rows
// whose preconditions fail (non-finite norm or codebook, S*C >= 2^120, more
// than kCap candidates) are resolved by an exact NaN-aware scan of all codes.
//
// Structure of one CTA (128 rows = the 128 TMEM lanes, all stages):
//   warps 0-3  epilogue: thread i owns row i (residual in registers), reads
//              its TMEM lane, screens, reranks, updates, writes the next
//              stage's A operand (2r, K-major, 128B swizzle) to shared memory;
//   warp 4     producer: cp.async.bulk of pre-swizzled 256-code codebook
//              tiles (64 KB) into a 2-slot ring;
//   warp 5     TMEM allocator + MMA issuer: per tile, 8 x tcgen05.mma
//              (M=128, N=256, K=8) into one of two 256-column accumulators.
// Every wait is bounded (~2 s) and records MOSS_ERR_TIMEOUT; all roles then
// meet at the final barrier where the TMEM is released.
#include "common.cuh"

#include <math_constants.h>

namespace moss {
namespace rvqtc {

constexpr int kDim = 64;
constexpr int kRows = 128;
constexpr int kTileCodes = 256;
constexpr int kSlots = 2;
constexpr int kCap = 8;
constexpr int kEpiThreads = 128;
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = kTileCodes * kDim * 4;  // 65536
constexpr uint32_t kTmemCols = 512;
constexpr int kRStride = 65;

struct __align__(1024) Smem {
  float btile[kSlots][kTileCodes * kDim];  // pre-swizzled B images (1024-aligned)
  float a[kRows * kDim];                   // 2r, K-major SW128 image
  float recon[kRows * kRStride];
  float cn[4096];                          // code norms of the current stage (<= 4096 codes)
  float cand_key[kCap][kRows];
  int cand_idx[kCap][kRows];
  float norms[kRows];
  int sel[kRows];
  int slow_list[kRows];
  int slow_count;
  int abort_flag;
  uint32_t tmem_base;
  alignas(8) unsigned long long b_full[kSlots];
  alignas(8) unsigned long long b_empty[kSlots];
  alignas(8) unsigned long long t_full[2];
  alignas(8) unsigned long long t_empty[2];
  alignas(8) unsigned long long a_full;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
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
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait (~2 s); false after recording a timeout.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - start > 2000000000ull) {
      record_device_error(MOSS_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void epi_bar() {
  __syncwarp();
  asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ int epi_bar_or(int pred) {
  int out;
  __syncwarp();
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, 128, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(pred)
      : "memory");
  return out;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: kind::tf32, D f32, A/B tf32 K-major, M=128, N=256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((256u >> 3) << 17) |
                            ((128u >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
  __syncwarp();  // .sync.aligned: the whole warp, converged
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// Waits for the outstanding TMEM loads; the registers are threaded through so
// that no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Byte offset of element (row, k) in a K-major SW128 image whose 8-row
// groups are 1024 bytes apart and whose two 32-element K halves are `half`
// bytes apart.
__device__ __forceinline__ uint32_t sw128_offset(int row, int k, uint32_t half) {
  const int kk = k & 31;
  return static_cast<uint32_t>(k >> 5) * half + static_cast<uint32_t>(row >> 3) * 1024u +
         static_cast<uint32_t>(row & 7) * 128u +
         static_cast<uint32_t>(((kk >> 2) ^ (row & 7)) << 4) + static_cast<uint32_t>(kk & 3) * 4u;
}

struct Args {
  const float* x;
  const float* books;      // raw [stages][k][64]
  const float* image;      // [stages][ntiles][64 KB swizzled]
  const float* code_norm;  // [stages][kpad]
  const float* stats;      // [stages][4]: max code norm, non-finite flag
  int32_t* codes;
  float* recon;
  float* residual_out;
  int64_t rows;
  int stages;
  int k;
  int kpad;
};

// Exact NaN-aware selection of one row by one warp (pinned arithmetic).
__device__ int exact_scan(const float* tw, float norm, const float* __restrict__ book,
                          const float* __restrict__ cnorm, int k, int lane) {
  float best = CUDART_INF_F;
  int best_i = lane;
  int nan_i = INT_MAX;
  for (int j = lane; j < k; j += 32) {
    const float* c = book + static_cast<int64_t>(j) * kDim;
    float dot = 0.0f;
    for (int d = 0; d < kDim; ++d) dot = __fmaf_rn(tw[d], c[d], dot);
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

__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}


// Keeps the candidates still inside the window; returns their count.
__device__ __noinline__ int compact_candidates(Smem& sm, int row, float thr) {
  int w = 0;
  for (int e = 0; e < kCap; ++e) {
    const float ek = sm.cand_key[e][row];
    if (ek <= thr) {
      sm.cand_key[w][row] = ek;
      sm.cand_idx[w][row] = sm.cand_idx[e][row];
      ++w;
    }
  }
  return w;
}

// Screens 32 accumulator columns (codes code0..code0+31) of this row:
// key = cnorm - TF32 dot; keeps the running minimum and appends every code
// within `window` of it to the row's candidate list (pruning entries that
// fell out of the window when the list is full).
__device__ __forceinline__ void screen_chunk(const uint32_t (&acc)[32], int code0, Smem& sm,
                                             int row, int s, const Args& a, bool slow,
                                             float window, float& mkey, float& thr, int& cnt,
                                             bool& overflow) {
  const float4* cn4 = reinterpret_cast<const float4*>(&sm.cn[code0]);
  float key[32];
  float cm = CUDART_INF_F;
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const float4 cv = cn4[j4];
    key[4 * j4 + 0] = __fsub_rn(cv.x, __uint_as_float(acc[4 * j4 + 0]));
    key[4 * j4 + 1] = __fsub_rn(cv.y, __uint_as_float(acc[4 * j4 + 1]));
    key[4 * j4 + 2] = __fsub_rn(cv.z, __uint_as_float(acc[4 * j4 + 2]));
    key[4 * j4 + 3] = __fsub_rn(cv.w, __uint_as_float(acc[4 * j4 + 3]));
    cm = fminf(cm, fminf(fminf(key[4 * j4], key[4 * j4 + 1]),
                         fminf(key[4 * j4 + 2], key[4 * j4 + 3])));
  }
  if (slow || !(cm <= thr)) return;
  mkey = fminf(mkey, cm);
  thr = mkey + window;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (key[j] <= thr) {
      if (cnt == kCap) cnt = compact_candidates(sm, row, thr);
      if (cnt == kCap) {
        overflow = true;
      } else {
        sm.cand_key[cnt][row] = key[j];
        sm.cand_idx[cnt][row] = code0 + j;
        ++cnt;
        const float* cw = a.books + (static_cast<int64_t>(s) * a.k + code0 + j) * kDim;
        prefetch_l1(cw);
        prefetch_l1(cw + 32);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) rvq_tc_kernel(Args a) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand images.
  Smem& sm = *reinterpret_cast<Smem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ntiles = a.kpad / kTileCodes;
  const int total_tiles = a.stages * ntiles;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kRows;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.b_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kEpiThreads);
    }
    mbar_init(&sm.a_full, kEpiThreads);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.abort_flag = 0;
    sm.slow_count = 0;
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int q = 0; q < total_tiles; ++q) {
        const int slot = q % kSlots;
        if (!mbar_wait(&sm.b_empty[slot], ((q / kSlots) & 1) ^ 1)) {
          sm.abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&sm.b_full[slot], kTileBytes);
        bulk_g2s(&sm.btile[slot][0], a.image + static_cast<int64_t>(q) * (kTileBytes / 4),
                 kTileBytes, &sm.b_full[slot]);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t a_base = smem_u32(sm.a);
      int q = 0;
      bool ok = true;
      for (int s = 0; s < a.stages && ok; ++s) {
        if (!mbar_wait(&sm.a_full, s & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t, ++q) {
          const int slot = q % kSlots;
          const int abuf = q & 1;
          if (!mbar_wait(&sm.b_full[slot], (q / kSlots) & 1) ||
              !mbar_wait(&sm.t_empty[abuf], ((q >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_base = smem_u32(&sm.btile[slot][0]);
          const uint32_t d_tmem = tmem + static_cast<uint32_t>(abuf * 256);
#pragma unroll
          for (int kk = 0; kk < kDim / 8; ++kk) {
            const uint32_t koff = static_cast<uint32_t>(kk >> 2) + 0u;
            const uint64_t ad =
                sw128_desc(a_base + koff * (kRows * 128u) + static_cast<uint32_t>(kk & 3) * 32u);
            const uint64_t bd = sw128_desc(b_base + koff * (kTileCodes * 128u) +
                                           static_cast<uint32_t>(kk & 3) * 32u);
            mma_tf32(d_tmem, ad, bd, kk > 0 ? 1u : 0u);
          }
          mma_commit(&sm.t_full[abuf]);
          mma_commit(&sm.b_empty[slot]);
        }
      }
      if (!ok) sm.abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int row = tid;  // TMEM lane == row (warps 0..3)
    const int64_t grow = row0 + row;
    const bool valid = grow < a.rows;
    float r[kDim];
    if (valid) {
      const float4* src = reinterpret_cast<const float4*>(a.x + grow * kDim);
#pragma unroll
      for (int i = 0; i < kDim / 4; ++i) {
        const float4 v = src[i];
        r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int d = 0; d < kDim; ++d) r[d] = 0.0f;
    }
    for (int d = 0; d < kDim; ++d) sm.recon[row * kRStride + d] = 0.0f;
    unsigned char* a_bytes = reinterpret_cast<unsigned char*>(sm.a);
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

    int q = 0;
    bool aborted = false;
    for (int s = 0; s < a.stages; ++s) {
      // norm and the A operand (2r) of this stage
      float norm = 0.0f;
#pragma unroll
      for (int d = 0; d < kDim; ++d) norm = __fmaf_rn(r[d], r[d], norm);
      sm.norms[row] = norm;
#pragma unroll
      for (int c = 0; c < kDim / 4; ++c) {
        float4 v = make_float4(__fmul_rn(2.0f, r[4 * c]), __fmul_rn(2.0f, r[4 * c + 1]),
                               __fmul_rn(2.0f, r[4 * c + 2]), __fmul_rn(2.0f, r[4 * c + 3]));
        *reinterpret_cast<float4*>(a_bytes + sw128_offset(row, 4 * c, kRows * 128u)) = v;
      }
      // stage code norms into shared memory
      const float* cn_g = a.code_norm + static_cast<int64_t>(s) * a.kpad;
      for (int i = row; i < a.kpad; i += kEpiThreads) sm.cn[i] = cn_g[i];
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      epi_bar();  // cn visible to all epilogue threads
      mbar_arrive(&sm.a_full);

      // screening margin and preconditions
      const float cn_max = a.stats[s * 4 + 0];
      const bool book_ok = a.stats[s * 4 + 1] == 0.0f;
      const float s2r = __fmul_rn(2.0f, sqrtf(norm));
      const float cmax = sqrtf(cn_max);
      const float sc = s2r * cmax;
      bool slow = !(isfinite(norm) && book_ok && sc < 1.0e36f);
      const float margin = fmaf(sc, 0.00390625f, (norm + cn_max) * 9.5367431640625e-07f) + 1e-30f;
      const float window = 2.0f * margin * 1.0001f;
      float mkey = CUDART_INF_F;
      float thr = CUDART_INF_F;
      int cnt = 0;
      bool overflow = false;

      for (int t = 0; t < ntiles; ++t, ++q) {
        const int abuf = q & 1;
        const int timed_out = mbar_wait(&sm.t_full[abuf], (q >> 1) & 1) ? 0 : 1;
        if (epi_bar_or(timed_out)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t tcol = tmem + lane_base + static_cast<uint32_t>(abuf * 256);
        uint32_t va[32], vb[32];
        tmem_load32(tcol, va);
        tmem_wait_ld(va);
#pragma unroll 1
        for (int c = 0; c < kTileCodes / 32; c += 2) {
          tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
          screen_chunk(va, t * kTileCodes + c * 32, sm, row, s, a, slow, window, mkey, thr, cnt,
                       overflow);
          tmem_wait_ld(vb);
          if (c + 2 < kTileCodes / 32) tmem_load32(tcol + static_cast<uint32_t>((c + 2) * 32), va);
          screen_chunk(vb, t * kTileCodes + (c + 1) * 32, sm, row, s, a, slow, window, mkey, thr,
                       cnt, overflow);
          if (c + 2 < kTileCodes / 32) tmem_wait_ld(va);
        }
        tc_fence_before();
        mbar_arrive(&sm.t_empty[abuf]);
      }
      if (aborted) break;

      // ---- resolve the stage: candidates -> exact winner
      int winner = -1;
      if (!slow && !overflow) {
        int best_i = -1;
        float best_d = 0.0f;
        int live = 0;
        for (int e = 0; e < cnt; ++e) {
          if (sm.cand_key[e][row] <= thr) {
            ++live;
            best_i = sm.cand_idx[e][row];
          }
        }
        if (live == 1) {
          winner = best_i;
        } else if (live > 1) {
          best_i = -1;
          for (int e = 0; e < cnt; ++e) {
            if (sm.cand_key[e][row] > thr) continue;
            const int j = sm.cand_idx[e][row];
            const float4* cw =
                reinterpret_cast<const float4*>(a.books + (static_cast<int64_t>(s) * a.k + j) * kDim);
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < kDim / 4; ++i) {
              const float4 v = cw[i];
              dot = __fmaf_rn(__fmul_rn(2.0f, r[4 * i]), v.x, dot);
              dot = __fmaf_rn(__fmul_rn(2.0f, r[4 * i + 1]), v.y, dot);
              dot = __fmaf_rn(__fmul_rn(2.0f, r[4 * i + 2]), v.z, dot);
              dot = __fmaf_rn(__fmul_rn(2.0f, r[4 * i + 3]), v.w, dot);
            }
            const float dist = __fadd_rn(__fsub_rn(norm, dot), sm.cn[j]);
            if (best_i < 0 || dist < best_d) {
              best_d = dist;
              best_i = j;
            }
          }
          winner = best_i;
        }
      }
      if (winner < 0) {
        const int slot = atomicAdd(&sm.slow_count, 1);
        sm.slow_list[slot] = row;
      }
      epi_bar();
      const int nslow = sm.slow_count;
      if (nslow > 0) {
        // exact scan, one warp per row; 2r is read back from the A image
        const float* book = a.books + static_cast<int64_t>(s) * a.k * kDim;
        for (int i = warp; i < nslow; i += 4) {
          const int sr = sm.slow_list[i];
          float tw[kDim];
          for (int d = 0; d < kDim; ++d)
            tw[d] = *reinterpret_cast<const float*>(a_bytes + sw128_offset(sr, d, kRows * 128u));
          const int ix = exact_scan(tw, sm.norms[sr], book,
                                    a.code_norm + static_cast<int64_t>(s) * a.kpad, a.k, lane);
          if (lane == 0) sm.sel[sr] = ix;
        }
        epi_bar();
        if (winner < 0) winner = sm.sel[row];
        epi_bar();
        if (row == 0) sm.slow_count = 0;
      }
      // ---- update the residual and the reconstruction
      const float4* cw =
          reinterpret_cast<const float4*>(a.books + (static_cast<int64_t>(s) * a.k + winner) * kDim);
      float* rc = &sm.recon[row * kRStride];
#pragma unroll
      for (int i = 0; i < kDim / 4; ++i) {
        const float4 v = cw[i];
        r[4 * i] = __fsub_rn(r[4 * i], v.x);
        r[4 * i + 1] = __fsub_rn(r[4 * i + 1], v.y);
        r[4 * i + 2] = __fsub_rn(r[4 * i + 2], v.z);
        r[4 * i + 3] = __fsub_rn(r[4 * i + 3], v.w);
        rc[4 * i] = __fadd_rn(rc[4 * i], v.x);
        rc[4 * i + 1] = __fadd_rn(rc[4 * i + 1], v.y);
        rc[4 * i + 2] = __fadd_rn(rc[4 * i + 2], v.z);
        rc[4 * i + 3] = __fadd_rn(rc[4 * i + 3], v.w);
      }
      if (valid) a.codes[static_cast<int64_t>(s) * a.rows + grow] = winner;
      // the slow scan of other rows may still read the A image: write the
      // next stage's operand only after every epilogue thread is here
      epi_bar();
    }
    if (!aborted && valid) {
      float4* dst = reinterpret_cast<float4*>(a.recon + grow * kDim);
      const float* rc = &sm.recon[row * kRStride];
#pragma unroll
      for (int i = 0; i < kDim / 4; ++i)
        dst[i] = make_float4(rc[4 * i], rc[4 * i + 1], rc[4 * i + 2], rc[4 * i + 3]);
      if (a.residual_out) {
        float4* res = reinterpret_cast<float4*>(a.residual_out + grow * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i)
          res[i] = make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      }
    }
    if (aborted) sm.abort_flag = 1;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace rvqtc
}  // namespace moss

using namespace moss;

extern "C" int moss_rvq_encode(const float* x, int64_t rows, int64_t d, const float* books,
                               const float* packed, const float* code_norm, const float* stats,
                               int64_t stages, int64_t k, int32_t* codes, float* recon,
                               float* residual_out, void* stream) {
  const char* name = "moss_rvq_encode";
  if (rows < 0 || stages < 1 || k < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (d != rvqtc::kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only 64-dim codewords are supported", name);
  if (k > 4096 || stages > 65535)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: at most 4096 codes per stage (use moss_rvq_encode_ffma)", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !books || !packed || !code_norm || !stats || !codes || !recon)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(books) || !aligned16(packed) || !aligned16(code_norm) ||
      !aligned16(recon) || (residual_out && !aligned16(residual_out)))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t kpad = (k + rvqtc::kTileCodes - 1) / rvqtc::kTileCodes * rvqtc::kTileCodes;
  const int64_t grid = (rows + rvqtc::kRows - 1) / rvqtc::kRows;
  if (grid > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows", name);
  const size_t smem = sizeof(rvqtc::Smem) + 1024;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(rvqtc::rvq_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return fail(MOSS_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // The tensor-core image follows the FFMA layout in the packed buffer.
  const float* image = packed + stages * kpad * rvqtc::kDim;
  rvqtc::Args args{x, books, image, code_norm, stats, codes, recon, residual_out, rows,
                   static_cast<int>(stages), static_cast<int>(k), static_cast<int>(kpad)};
  rvqtc::rvq_tc_kernel<<<static_cast<unsigned>(grid), rvqtc::kThreads, smem, as_stream(stream)>>>(args);
  return launch_status(name);
}
