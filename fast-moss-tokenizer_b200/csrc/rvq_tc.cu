// Multi-stage residual VQ with tensor-core screening (tcgen05, TF32) and an
// exact FP32 resolution.  Produces exactly the codes of the FFMA kernel in
// rvq.cu (same documented arithmetic).
//
// Why the indices stay exact.  For row r and code j the tensor cores compute
//   acc_j = TF32 sum_d 2r_d c_jd  -  TF32(cnorm_j)      (9th K step: 1 x -cnorm)
// and key_j = -acc_j approximates exact_j = dist_j - norm (real-number
// difference; dist_j in the pinned FP32 order of rvq.cu).  TF32 keeps 10
// fraction bits (relative error < 2^-10 per operand), so the products are
// within 2^-9 sum|2r_d c_jd| <= 2^-9 S C (S = |2r|, C = max_j |c_j|) and the
// folded norm within 2^-10 cnorm_max; the pinned FP32 dot and the two FP32
// roundings of dist add less than 2^-20 (norm + cnorm_max + S C).  Hence
//   |key_j - exact_j| <= M = 2^-8 S C + 2^-9 cnorm_max + 2^-20 (norm + cnorm_max)
// (twice the TF32 bound).  Every minimiser j* of dist has key_j* <= min key
// + 2M, so the candidates {j : acc_j >= max acc - 2M} contain all of them.
// One candidate is the answer; several are resolved with the exact pinned
// arithmetic (first minimum wins).  Rows whose preconditions fail
// (non-finite norm or codebook, S C >= 1e36, candidate records overflow) are
// resolved by an exact NaN-aware scan of all codes.
//
// SIMT shape of the screening: per 32-code chunk a thread (one row) takes the
// chunk maximum, updates its running maximum, and forms a 32-bit mask of the
// codes inside the window -- all branch-free.  Only a non-empty mask costs a
// (rare, short) record of {chunk, mask, chunk max} in shared memory; the
// records are filtered against the final window at the end of the stage.
//
// A CTA owns `rows_per_cta` rows for all stages, 320 threads:
//   warps 0-7  epilogue (256 threads).  With at most 64 rows per CTA (the
//              default while the rows fit one CTA per SM: 8192 rows -> 147
//              CTAs of 56) every row is written into two TMEM lanes (lane i
//              and 64 + i), so four threads screen its 256 columns per tile
//              (two lane copies x two column halves); with 128 rows per CTA
//              each row has one lane and two threads.  The part-0 thread of
//              a row owns it: residual in registers, the exact resolve of
//              its warp's candidate queue, the residual update, and the next
//              stage's A operand (2r, K-major 128B-swizzled) in shared memory;
//   warp 8     producer: cp.async.bulk of pre-built 256-code codebook tile
//              images (64 KB swizzled dims + 8 KB norm column) into 2 slots;
//   warp 9     TMEM allocator + MMA issuer: per tile 9 x tcgen05.mma
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
constexpr int kRec = 8;       // screening records per row, column half and stage
constexpr int kQueue = 256;   // candidates resolved exactly per epilogue warp and stage
constexpr int kEpiThreads = 256;  // two threads per row (column halves)
constexpr int kThreads = kEpiThreads + 64;
constexpr int kProducerWarp = kEpiThreads / 32;
constexpr int kMmaWarp = kProducerWarp + 1;
constexpr uint32_t kMainBytes = kTileCodes * kDim * 4;   // 65536: swizzled dims
constexpr uint32_t kExtraBytes = kTileCodes * 8 * 4;     // 8192: norm column block
constexpr uint32_t kTileBytes = kMainBytes + kExtraBytes;  // 73728 per tile image
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxCodes = 4096;

struct __align__(1024) Smem {
  float btile[kSlots][kTileBytes / 4];  // tile images (each 1024-aligned)
  float a[kRows * kDim];                // 2r, K-major SW128 image
  float a_extra[kRows * 8];             // [1, 0 x 7] per row, no-swizzle K block
  // Per screening slot (column part x local row, at most 256 slots):
  float cmax[4][2 * kRows];  // chunk maxima of the current tile
  float rec_max[kRec][2 * kRows];
  uint32_t rec_mask[kRec][2 * kRows];
  unsigned char rec_chunk[kRec][2 * kRows];
  float amax_h[2 * kRows];  // running screening maximum
  int nrec_h[2 * kRows];
  float window[kRows];
  int pre_slow[kRows];  // row fails the screening preconditions this stage
  int row_bad[kRows];   // row's candidates did not fit the resolve queue
  unsigned long long best[kRows];  // (orderable distance << 32) | code
  int queue[kEpiThreads / 32][kQueue];  // (row << 16) | code
  float norms[kRows];
  int sel[kRows];
  int slow_list[kRows];
  int slow_count;
  uint32_t tmem_base;
  alignas(8) unsigned long long b_full[kSlots];
  alignas(8) unsigned long long b_empty[kSlots];
  alignas(8) unsigned long long t_full[2];
  alignas(8) unsigned long long t_empty[2];
  alignas(8) unsigned long long a_full;
};
// The dynamic allocation adds 1024 bytes of alignment slack.
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory above the sm_100 per-block limit");

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
// The waiting thread is suspended (up to ~20 us per attempt) instead of
// spinning, so waiting roles leave the issue slots to the epilogue warps.
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Bounded wait (~2 s); false after recording a timeout.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
  return bounded_wait([&] { return mbar_try_wait(bar, parity); });
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
// Barrier of the epilogue warps (both column halves).
__device__ __forceinline__ void epi_bar() {
  __syncwarp();
  asm volatile("bar.sync 1, 256;" ::: "memory");
}
__device__ __forceinline__ int epi_bar_or(int pred) {
  int out;
  __syncwarp();
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, 256, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(pred)
      : "memory");
  return out;
}

// Shared-memory matrix descriptors (descriptor version 1).
//   K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (SBO).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
//   K-major, no swizzle: 8-row x 16-byte core matrices; the two K halves
//   128 bytes apart (LBO), 8-row groups 256 bytes apart (SBO).
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (8ull << 16) | (16ull << 32) |
         (1ull << 46);
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

// Byte offset of (row, k) in a K-major SW128 image: 8-row groups 1024 bytes
// apart, 16-byte chunk index XOR row % 8, the two 32-element K halves `half`
// bytes apart.  The tile images built by rvq.cu use the same formula.
__device__ __forceinline__ uint32_t sw128_offset(int row, int k, uint32_t half) {
  const int kk = k & 31;
  return static_cast<uint32_t>(k >> 5) * half + static_cast<uint32_t>(row >> 3) * 1024u +
         static_cast<uint32_t>(row & 7) * 128u +
         static_cast<uint32_t>(((kk >> 2) ^ (row & 7)) << 4) + static_cast<uint32_t>(kk & 3) * 4u;
}
// Byte offset of (row, k < 8) in the no-swizzle K block.
__device__ __forceinline__ uint32_t plain_offset(int row, int k) {
  return static_cast<uint32_t>(row >> 3) * 256u + static_cast<uint32_t>(k >> 2) * 128u +
         static_cast<uint32_t>(row & 7) * 16u + static_cast<uint32_t>(k & 3) * 4u;
}

struct Args {
  const float* x;
  const float* books;      // raw [stages][k][64]
  const float* image;      // [stages][ntiles][kTileBytes]
  const float* code_norm;  // [stages][kpad]
  const float* stats;      // [stages][4]: max code norm, non-finite flag
  int32_t* codes;
  float* recon;
  float* residual_out;
  int64_t rows;
  int stages;
  int k;
  int kpad;
  int rows_per_cta;  // 128, or 64 with every row in two TMEM lanes
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

// Shared-memory vector store at a 32-bit shared address.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, float x0, float x1, float x2,
                                             float x3) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x0), "f"(x1), "f"(x2),
               "f"(x3)
               : "memory");
}

// Keeps the records (of one column half) whose chunk maximum is still
// inside the window.
__device__ __noinline__ int compact_records(Smem& sm, int slot, float athr) {
  int w = 0;
  for (int e = 0; e < kRec; ++e) {
    if (sm.rec_max[e][slot] >= athr) {
      sm.rec_max[w][slot] = sm.rec_max[e][slot];
      sm.rec_mask[w][slot] = sm.rec_mask[e][slot];
      sm.rec_chunk[w][slot] = sm.rec_chunk[e][slot];
      ++w;
    }
  }
  return w;
}

// Screening record: stores {chunk max, mask, chunk} and returns the new
// record count (kRec + 1 once the records overflowed; compaction of records
// that left the window is the rare case).
__device__ __forceinline__ int add_record(Smem& sm, int slot, int chunk, uint32_t mask, float cmx,
                                          float athr, int nrec) {
  if (nrec >= kRec) {
    if (nrec > kRec) return nrec;
    nrec = compact_records(sm, slot, athr);
    if (nrec == kRec) return kRec + 1;
  }
  sm.rec_max[nrec][slot] = cmx;
  sm.rec_mask[nrec][slot] = mask;
  sm.rec_chunk[nrec][slot] = static_cast<unsigned char>(chunk);
  return nrec + 1;
}

// Float ordering as an unsigned key (finite values; -0 is mapped to +0 by
// the caller so that equal distances compare equal).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum of 32 accumulator values: a depth-4 tree of three-input maxima
// (16 instructions).
__device__ __forceinline__ float max32(const uint32_t (&acc)[32]) {
  float m[11];
#pragma unroll
  for (int j = 0; j < 10; ++j)
    m[j] = max3f(__uint_as_float(acc[3 * j]), __uint_as_float(acc[3 * j + 1]),
                 __uint_as_float(acc[3 * j + 2]));
  m[10] = fmaxf(__uint_as_float(acc[30]), __uint_as_float(acc[31]));
  const float a = max3f(m[0], m[1], m[2]), b = max3f(m[3], m[4], m[5]);
  const float c = max3f(m[6], m[7], m[8]), d = fmaxf(m[9], m[10]);
  return fmaxf(max3f(a, b, c), d);
}

// Bit j set iff acc[j] >= athr; four independent 8-bit partial masks.
__device__ __forceinline__ uint32_t mask32(const uint32_t (&acc)[32], float athr) {
  uint32_t part[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int p = 0; p < 4; ++p)
      part[p] |= (__uint_as_float(acc[8 * p + j]) >= athr) ? (1u << (8 * p + j)) : 0u;
  }
  return (part[0] | part[1]) | (part[2] | part[3]);
}

__global__ void __launch_bounds__(kThreads, 1) rvq_tc_kernel(Args a) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand images, by pointer
  // arithmetic on the shared array: the compiler then keeps the shared state
  // space for every access through `sm` (an integer round trip would turn
  // them into generic accesses).
  Smem& sm = *reinterpret_cast<Smem*>(
      smem_raw +
      ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ntiles = a.kpad / kTileCodes;
  const int total_tiles = a.stages * ntiles;
  const int rpc = a.rows_per_cta;
  // rows_per_cta <= 64: every row sits in two TMEM lanes, copy c of local
  // row i in lane c * 64 + i (lanes i >= rpc of each copy hold no row)
  const int copies = rpc <= kRows / 2 ? 2 : 1;
  const int span = kRows / copies;  // lanes per copy
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * rpc;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.b_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.t_full[i], 1);
      mbar_init(&sm.t_empty[i], kEpiThreads);
    }
    mbar_init(&sm.a_full, span);  // every owner thread writes its lane
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.slow_count = 0;
  }
  if (warp == kMmaWarp) {
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

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int q = 0; q < total_tiles; ++q) {
        const int slot = q % kSlots;
        if (!mbar_wait(&sm.b_empty[slot], ((q / kSlots) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&sm.b_full[slot], kTileBytes);
        bulk_g2s(&sm.btile[slot][0], a.image + static_cast<int64_t>(q) * (kTileBytes / 4),
                 kTileBytes, &sm.b_full[slot]);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t a_base = smem_u32(sm.a);
      const uint64_t a_extra = plain_desc(smem_u32(sm.a_extra));
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
            const uint32_t koff = static_cast<uint32_t>(kk >> 2);
            const uint64_t ad =
                sw128_desc(a_base + koff * (kRows * 128u) + static_cast<uint32_t>(kk & 3) * 32u);
            const uint64_t bd = sw128_desc(b_base + koff * (kTileCodes * 128u) +
                                           static_cast<uint32_t>(kk & 3) * 32u);
            mma_tf32(d_tmem, ad, bd, kk > 0 ? 1u : 0u);
          }
          // 9th K step: 1 x (-cnorm_j)
          mma_tf32(d_tmem, a_extra, plain_desc(b_base + kMainBytes), 1u);
          mma_commit(&sm.t_full[abuf]);
          mma_commit(&sm.b_empty[slot]);
        }
      }
      // Let the final commit arrivals land before the CTA can retire.
      for (int last = (q > kSlots ? q - kSlots : 0); ok && last < q; ++last) {
        ok = mbar_wait(&sm.b_empty[last % kSlots], (last / kSlots) & 1);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // The CTA's rpc rows sit in the 128 TMEM lanes `copies` times (lane L
    // holds local row L % span when that is below rpc).  Warp w reads the lanes of quarter w % 4, and
    // the 2 * copies warps that see a row split every tile's 256 columns
    // into equal parts.  The part-0 thread of a row owns it (residual in
    // registers): it writes the A operand, resolves and updates.
    const int quarter = warp & 3;
    const int qpr = 4 / copies;               // lane quarters per copy
    const int lr = (quarter % qpr) * 32 + lane;  // local row
    const int part = (quarter / qpr) * 2 + (warp >> 2);
    const int nparts = 2 * copies;
    const int cpp = 8 / nparts;               // 32-code chunks per part and tile
    const int slot = part * span + lr;
    const bool owner = part == 0;
    const int64_t grow = row0 + lr;
    const bool valid = lr < rpc && grow < a.rows;
    float r[kDim];
    if (owner && valid) {
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
    unsigned char* a_bytes = reinterpret_cast<unsigned char*>(sm.a);
    if (owner) {
      unsigned char* e = reinterpret_cast<unsigned char*>(sm.a_extra);
      for (int cp = 0; cp < copies; ++cp) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float*>(e + plain_offset(lr + cp * span, k)) = k == 0 ? 1.0f : 0.0f;
      }
    }
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    // The A operand (2r, in every copy) of the next stage is written as soon
    // as the residual is known, so that its MMA starts before the bookkeeping
    // of the stage boundary.
    auto write_a = [&]() {
      const uint32_t a_base = smem_u32(sm.a);
      if (copies == 2) {
#pragma unroll
        for (int c = 0; c < kDim / 4; ++c) {
          const float x0 = __fmul_rn(2.0f, r[4 * c]), x1 = __fmul_rn(2.0f, r[4 * c + 1]);
          const float x2 = __fmul_rn(2.0f, r[4 * c + 2]), x3 = __fmul_rn(2.0f, r[4 * c + 3]);
          st_shared_v4(a_base + sw128_offset(lr, 4 * c, kRows * 128u), x0, x1, x2, x3);
          st_shared_v4(a_base + sw128_offset(lr + span, 4 * c, kRows * 128u), x0, x1, x2, x3);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kDim / 4; ++c) {
          const float x0 = __fmul_rn(2.0f, r[4 * c]), x1 = __fmul_rn(2.0f, r[4 * c + 1]);
          const float x2 = __fmul_rn(2.0f, r[4 * c + 2]), x3 = __fmul_rn(2.0f, r[4 * c + 3]);
          st_shared_v4(a_base + sw128_offset(lr, 4 * c, kRows * 128u), x0, x1, x2, x3);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sm.a_full);
    };
    if (owner) write_a();

    int q = 0;
    bool aborted = false;
    // The stage's codebook statistics are loaded one stage ahead.
    float next_cn_max = a.stats[0], next_flag = a.stats[1];
    for (int s = 0; s < a.stages; ++s) {
      const float* book = a.books + static_cast<int64_t>(s) * a.k * kDim;
      const float* cnorm = a.code_norm + static_cast<int64_t>(s) * a.kpad;
      const float cn_max = next_cn_max;
      const bool book_ok = next_flag == 0.0f;
      if (s + 1 < a.stages) {
        next_cn_max = a.stats[(s + 1) * 4 + 0];
        next_flag = a.stats[(s + 1) * 4 + 1];
      }
      float norm = 0.0f;
      if (owner) {
#pragma unroll
        for (int d = 0; d < kDim; ++d) norm = __fmaf_rn(r[d], r[d], norm);
        sm.norms[lr] = norm;
        // screening window and preconditions
        const float sc = __fmul_rn(2.0f, sqrtf(norm)) * sqrtf(cn_max);
        const bool slow = !(isfinite(norm) && book_ok && sc < 1.0e36f);
        const float margin = sc * 0.00390625f + cn_max * 0.001953125f +
                             (norm + cn_max) * 9.5367431640625e-07f + 1e-30f;
        sm.window[lr] = 2.0f * margin * 1.0001f;
        sm.pre_slow[lr] = slow || !valid ? 1 : 0;
        sm.row_bad[lr] = 0;
        sm.best[lr] = ~0ull;
      }
      epi_bar();  // the window is visible to every part
      const float window = sm.window[lr];
      float amax = -CUDART_INF_F;
      int nrec = 0;
      // A timed-out wait is agreed on at the end of the stage (all threads
      // run the same tiles; after a timeout this thread stops waiting and
      // the stage's values are discarded).
      int timed_out = 0;
      for (int t = 0; t < ntiles; ++t, ++q) {
        const int abuf = q & 1;
        if (!timed_out && !mbar_wait(&sm.t_full[abuf], (q >> 1) & 1)) timed_out = 1;
        tc_fence_after();
        const uint32_t tcol =
            tmem + lane_base + static_cast<uint32_t>(abuf * 256 + part * cpp * 32);
        uint32_t va[32], vb[32];
        if (cpp == 2) {
          // 64 rows per CTA: the part's two chunks are loaded once and kept
          // in registers for the mask.
          tmem_load32(tcol, va);
          tmem_load32(tcol + 32u, vb);
          tmem_wait_ld(va);
          tmem_wait_ld(vb);
          // The accumulator is in registers: hand it back to the MMA warp
          // now, so that the tile after next is computed while this one is
          // screened.
          tc_fence_before();
          mbar_arrive(&sm.t_empty[abuf]);
          const float ca = max32(va), cb = max32(vb);
          amax = fmaxf(amax, fmaxf(ca, cb));
          const float athr = amax - window;
          const uint32_t ma = valid ? mask32(va, athr) : 0u;
          const uint32_t mb = valid ? mask32(vb, athr) : 0u;
          const int chunk = t * 8 + part * cpp;
          if (ma) nrec = add_record(sm, slot, chunk, ma, ca, athr, nrec);
          if (mb) nrec = add_record(sm, slot, chunk + 1, mb, cb, athr, nrec);
        } else {
          // Pass 1: the chunk maxima of this part of the tile, then one
          // threshold; pass 2: window masks of the chunks that reach it.
          float tmax = -CUDART_INF_F;
#pragma unroll 1
          for (int c = 0; c < cpp; c += 2) {
            tmem_load32(tcol + static_cast<uint32_t>(c * 32), va);
            tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
            tmem_wait_ld(va);
            tmem_wait_ld(vb);
            const float ca = max32(va), cb = max32(vb);
            sm.cmax[c][slot] = ca;
            sm.cmax[c + 1][slot] = cb;
            tmax = fmaxf(tmax, fmaxf(ca, cb));
          }
          amax = fmaxf(amax, tmax);
          const float athr = amax - window;
#pragma unroll 1
          for (int c = 0; c < cpp; c += 2) {
            tmem_load32(tcol + static_cast<uint32_t>(c * 32), va);
            tmem_load32(tcol + static_cast<uint32_t>((c + 1) * 32), vb);
            tmem_wait_ld(va);
            tmem_wait_ld(vb);
            const uint32_t ma = valid ? mask32(va, athr) : 0u;
            const uint32_t mb = valid ? mask32(vb, athr) : 0u;
            const int chunk = t * 8 + part * cpp + c;
            if (ma) nrec = add_record(sm, slot, chunk, ma, sm.cmax[c][slot], athr, nrec);
            if (mb) nrec = add_record(sm, slot, chunk + 1, mb, sm.cmax[c + 1][slot], athr, nrec);
          }
          tc_fence_before();
          mbar_arrive(&sm.t_empty[abuf]);
        }
      }
      sm.amax_h[slot] = amax;
      sm.nrec_h[slot] = nrec;
      if (epi_bar_or(timed_out)) {  // every part's records are complete
        aborted = true;
        break;
      }

      // ---- resolve the stage: every surviving candidate gets its exact
      // distance.  The lanes of a warp share the candidates of its 32 rows
      // (from the A image, 2r in shared memory); per row the smallest
      // (distance, code) key wins, i.e. the first minimum.
      bool fast = sm.pre_slow[lr] == 0;
      float gmax = -CUDART_INF_F;
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        if (p < nparts) {
          fast = fast && sm.nrec_h[p * span + lr] <= kRec;
          gmax = fmaxf(gmax, sm.amax_h[p * span + lr]);
        }
      }
      const float athr = gmax - window;
      // A row needs the exact scan when its preconditions failed or its
      // candidates overflow the queue; the flag rides on the next barrier.
      int slow_flag = (owner && valid && !fast) ? 1 : 0;
      // Count the surviving candidates, keeping the first four in registers
      // for the queue fill and sending their codewords on their way into L1
      // (the lane that resolves a candidate reads it from there).
      int cnt = 0;
      int c0 = 0, c1 = 0, c2 = 0, c3 = 0;
      if (fast) {
        // the records' fields are loaded together, then walked
        float rmax[kRec];
        uint32_t rmask[kRec];
#pragma unroll
        for (int e = 0; e < kRec; ++e) {
          rmax[e] = e < nrec ? sm.rec_max[e][slot] : -CUDART_INF_F;
          rmask[e] = e < nrec ? sm.rec_mask[e][slot] : 0u;
        }
#pragma unroll
        for (int e = 0; e < kRec; ++e) {
          if (rmax[e] < athr || rmask[e] == 0u) continue;
          const int base = sm.rec_chunk[e][slot] * 32;
          for (uint32_t m = rmask[e]; m; m &= m - 1) {
            const int j = base + (__ffs(m) - 1);
            if (cnt < 4) {
              const int jc = j < a.k ? j : 0;
              prefetch_l1(book + static_cast<int64_t>(jc) * kDim);
              prefetch_l1(book + static_cast<int64_t>(jc) * kDim + 32);
              c3 = cnt == 3 ? j : c3;
              c2 = cnt == 2 ? j : c2;
              c1 = cnt == 1 ? j : c1;
              c0 = cnt == 0 ? j : c0;
            }
            ++cnt;
          }
        }
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int total = __shfl_sync(0xffffffffu, incl, 31);
      int* queue = sm.queue[warp];
      if (incl > kQueue) {
        sm.row_bad[lr] = 1;  // does not fit: exact scan
        slow_flag = 1;
      } else if (cnt > 4) {  // rare: walk the records again
        int pos = incl - cnt;
        for (int e = 0; e < nrec; ++e) {
          if (sm.rec_max[e][slot] < athr) continue;
          const int base = sm.rec_chunk[e][slot] * 32;
          for (uint32_t m = sm.rec_mask[e][slot]; m; m &= m - 1)
            queue[pos++] = (lr << 16) | (base + (__ffs(m) - 1));
        }
      } else if (cnt > 0) {
        const int pos = incl - cnt;
        queue[pos] = (lr << 16) | c0;
        if (cnt > 1) queue[pos + 1] = (lr << 16) | c1;
        if (cnt > 2) queue[pos + 2] = (lr << 16) | c2;
        if (cnt > 3) queue[pos + 3] = (lr << 16) | c3;
      }
      // entries [0, nq) are written: the rows whose candidates all fit
      const int nq = total <= kQueue ? total : __reduce_max_sync(0xffffffffu, incl <= kQueue ? incl : 0);
      __syncwarp();
      for (int i = lane; i < nq; i += 32) {
        const int ent = queue[i];
        const int rr = ent >> 16, j = ent & 0xffff;
        if (j >= a.k) continue;  // padding columns never reach the window
        const float4* cw = reinterpret_cast<const float4*>(book + static_cast<int64_t>(j) * kDim);
        float4 w[kDim / 4];
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) w[i4] = cw[i4];
        const float nj = cnorm[j];
        float dot = 0.0f;
#pragma unroll
        for (int i4 = 0; i4 < kDim / 4; ++i4) {
          const float4 tw =
              *reinterpret_cast<const float4*>(a_bytes + sw128_offset(rr, 4 * i4, kRows * 128u));
          dot = __fmaf_rn(tw.x, w[i4].x, dot);
          dot = __fmaf_rn(tw.y, w[i4].y, dot);
          dot = __fmaf_rn(tw.z, w[i4].z, dot);
          dot = __fmaf_rn(tw.w, w[i4].w, dot);
        }
        const float dist = __fadd_rn(__fadd_rn(__fsub_rn(sm.norms[rr], dot), nj), 0.0f);
        atomicMin(&sm.best[rr],
                  (static_cast<unsigned long long>(order_key(dist)) << 32) | static_cast<uint32_t>(j));
      }
      // every candidate of every row is in; is any row flagged?
      const int any_slow = epi_bar_or(slow_flag);
      int winner = -1;
      if (owner && fast && sm.row_bad[lr] == 0 && sm.best[lr] != ~0ull)
        winner = static_cast<int>(sm.best[lr] & 0xffffffffu);
      int nslow = 0;
      if (any_slow) {
        if (owner && valid && winner < 0) {
          const int at = atomicAdd(&sm.slow_count, 1);
          sm.slow_list[at] = lr;
        }
        epi_bar();
        nslow = sm.slow_count;
      }
      if (nslow > 0) {
        // exact scan, one warp per row; 2r is read back from the A image
        for (int i = warp; i < nslow; i += kEpiThreads / 32) {
          const int sr = sm.slow_list[i];
          float tw[kDim];
          for (int d = 0; d < kDim; ++d)
            tw[d] = *reinterpret_cast<const float*>(a_bytes + sw128_offset(sr, d, kRows * 128u));
          const int ix = exact_scan(tw, sm.norms[sr], book, cnorm, a.k, lane);
          if (lane == 0) sm.sel[sr] = ix;
        }
        epi_bar();
        if (owner && valid && winner < 0) winner = sm.sel[lr];
        epi_bar();
        if (warp == 0 && lane == 0) sm.slow_count = 0;
      }
      if (owner && valid && winner < 0) {
        // Unreachable: on the fast path the screening maximum is a real code
        // (padding codes screen at -inf, real ones are finite), so every
        // unflagged row has a resolved candidate.  Kept in bounds, reported.
        record_device_error(MOSS_ERR_UNSUPPORTED);
        winner = 0;
      }
      if (owner && valid) {
        // ---- update the residual (the reconstruction is summed at the end)
        const float4* cw =
            reinterpret_cast<const float4*>(book + static_cast<int64_t>(winner) * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i) {
          const float4 v = cw[i];
          r[4 * i] = __fsub_rn(r[4 * i], v.x);
          r[4 * i + 1] = __fsub_rn(r[4 * i + 1], v.y);
          r[4 * i + 2] = __fsub_rn(r[4 * i + 2], v.z);
          r[4 * i + 3] = __fsub_rn(r[4 * i + 3], v.w);
        }
        a.codes[static_cast<int64_t>(s) * a.rows + grow] = winner;
      }
      // every reader of this stage's A image (MMA, exact distances, slow
      // scan) is done: the next stage's operand can go in
      if (owner && s + 1 < a.stages) write_a();
      // the slow scan read the A image and the resolve read the other parts'
      // records: both must be finished before the next stage rewrites them
      epi_bar();
    }
    if (owner && !aborted && valid) {
      // recon = sum of the chosen codewords in stage order from +0 (the same
      // float32 additions as an incremental sum)
      float acc[kDim];
#pragma unroll
      for (int d = 0; d < kDim; ++d) acc[d] = 0.0f;
#pragma unroll 4
      for (int s = 0; s < a.stages; ++s) {
        const int c = a.codes[static_cast<int64_t>(s) * a.rows + grow];
        const float4* cw = reinterpret_cast<const float4*>(
            a.books + (static_cast<int64_t>(s) * a.k + c) * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i) {
          const float4 v = cw[i];
          acc[4 * i] = __fadd_rn(acc[4 * i], v.x);
          acc[4 * i + 1] = __fadd_rn(acc[4 * i + 1], v.y);
          acc[4 * i + 2] = __fadd_rn(acc[4 * i + 2], v.z);
          acc[4 * i + 3] = __fadd_rn(acc[4 * i + 3], v.w);
        }
      }
      float4* dst = reinterpret_cast<float4*>(a.recon + grow * kDim);
#pragma unroll
      for (int i = 0; i < kDim / 4; ++i)
        dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
      if (a.residual_out) {
        float4* res = reinterpret_cast<float4*>(a.residual_out + grow * kDim);
#pragma unroll
        for (int i = 0; i < kDim / 4; ++i)
          res[i] = make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
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
  if (k > rvqtc::kMaxCodes || stages > 65535)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: at most 4096 codes per stage (use moss_rvq_encode_ffma)", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !books || !packed || !code_norm || !stats || !codes || !recon)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(books) || !aligned16(packed) || !aligned16(code_norm) ||
      !aligned16(recon) || (residual_out && !aligned16(residual_out)))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t kpad = (k + rvqtc::kTileCodes - 1) / rvqtc::kTileCodes * rvqtc::kTileCodes;
  // While the rows fit one CTA per SM at 64 rows per CTA, they are spread
  // evenly over all SMs (ceil(rows / SMs) rows per CTA, each row in two
  // TMEM lanes so four threads share its columns: 8192 rows -> 147 CTAs of
  // 56); above that a CTA takes 128 rows, one lane each.
  const int64_t sms = sm_count();
  const int rows_per_cta =
      rows <= sms * 64 ? static_cast<int>((rows + sms - 1) / sms) : rvqtc::kRows;
  const int64_t grid = (rows + rows_per_cta - 1) / rows_per_cta;
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
  // The tensor-core tile images follow the FFMA layout in the packed buffer.
  const float* image = packed + stages * kpad * rvqtc::kDim;
  rvqtc::Args args{x, books, image, code_norm, stats, codes, recon, residual_out, rows,
                   static_cast<int>(stages), static_cast<int>(k), static_cast<int>(kpad),
                   rows_per_cta};
  rvqtc::rvq_tc_kernel<<<static_cast<unsigned>(grid), rvqtc::kThreads, smem, as_stream(stream)>>>(args);
  return launch_status(name);
}
