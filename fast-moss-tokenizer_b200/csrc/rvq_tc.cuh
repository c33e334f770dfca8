// Device building blocks shared by the tensor-core quantizer kernels
// (rvq_tc.cu: one CTA per row block; rvq_pair.cu: a CTA pair per row block
// splitting the codebook): mbarriers, bulk copies, tcgen05 MMA and TMEM
// loads, the operand image layouts, the screening records and the exact
// NaN-aware selection.
#pragma once

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
// Bounded wait (~2 s unless given); false after recording a timeout.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  return bounded_wait([&] { return mbar_try_wait(bar, parity); }, limit_ns);
}
// The same without the suspend hint: for waits on the critical path whose
// waiters have nothing else to do (the epilogue waiting for an accumulator).
__device__ __forceinline__ bool mbar_try_wait_spin(unsigned long long* bar, uint32_t parity) {
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
__device__ __forceinline__ bool mbar_wait_spin(unsigned long long* bar, uint32_t parity,
                                               uint64_t limit_ns = kWaitLimitNs) {
  return bounded_wait([&] { return mbar_try_wait_spin(bar, parity); }, limit_ns);
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
  // rvq_tc_kernel: rows of one CTA (128, or at most 64 with every row in two
  // TMEM lanes); rvq_pair_kernel: rows of one CTA pair (at most 128)
  int rows_per_cta;
};

// Exact NaN-aware selection of one row by one warp (pinned arithmetic).
static __device__ int exact_scan(const float* tw, float norm, const float* __restrict__ book,
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
template <typename S>
__device__ __noinline__ int compact_records(S& sm, int slot, float athr) {
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
template <typename S>
__device__ __forceinline__ int add_record(S& sm, int slot, int chunk, uint32_t mask, float cmx,
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

}  // namespace rvqtc
}  // namespace moss
