// Attention of a chunk's queries over a streaming history ring (bf16 in and
// out, FP32 arithmetic).
//
// The reference's streaming layer calls the upstream attention module with
// SDPA (the only validated backend, fast_moss/v2_runtime.py:40-41) over a
// bounded history that its StreamingCodec keeps at stable addresses
// (fast_moss/streaming.py:68-79); the patched layer calls it at
// fast_moss/v2_runtime.py:254-262.  Per stream s, head h and query t of the
// chunk (absolute position pos[s] + t), the keys are the ring's slots j with
//   0 <= slot_pos[s, j] <= pos[s] + t   and   slot_pos[s, j] > pos[s] + t - context
// (the boolean mask the history builds), and
//   out[s, t, h, :] = sum_j softmax_j(scale * q[s, h, t, :] . k[s, h, j, :]) v[s, h, j, :]
// with the softmax over the attended keys.
//
// One CTA per (stream, head).  All threads issue 16-byte cp.async loads of
// the head's whole K and V blocks at once (contiguous in the [S, H, N, 64]
// ring), K first: K rows land XOR-swizzled by 16-byte chunk so that the
// per-key dot products read shared memory without bank conflicts.  Thread j
// scores key j for every query; the softmax is a block reduction in a fixed
// order; for P.V each warp takes a strided eighth of the keys with lane l
// holding dims 2l and 2l+1, and the eight partial sums are added in warp
// order.  Everything is FP32 (expf, IEEE division), rounded once to bf16.
// The weights and the partial sums reuse K's shared memory once the scores
// are formed, so that three CTAs fit on an SM (registers capped to match):
// one CTA's loads then overlap the others' arithmetic.
#include <cuda.h>
#include <math_constants.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "rotary.cuh"
#include "tcgen05.cuh"

namespace moss {
namespace hattn {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kDim = 64;
constexpr int kMaxQueries = 8;
constexpr int kMaxKeys = 512;
constexpr int kKeysPerThread = kMaxKeys / kThreads;
// Every slot index j = tid + m * kThreads (m < kKeysPerThread) that a thread
// holds must cover [0, kMaxKeys) exactly; the host rejects n > kMaxKeys
// before any launch, so the per-thread arrays are never indexed past it.
static_assert(kKeysPerThread * kThreads == kMaxKeys, "slots per thread must tile kMaxKeys");

struct Args {
  const uint16_t* q;         // [S, H, T, 64]
  const uint16_t* k;         // [S, H, N, 64]
  const uint16_t* v;         // [S, H, N, 64]
  const int64_t* slot_pos;   // [S, N]
  const int64_t* pos;        // [S]
  uint16_t* out;             // [S, T, H, 64]
  int64_t context;
  float scale;
  int h, t, n;
};

// Rows of the weight array are padded to 4 floats (16 bytes).
__host__ __device__ constexpr int padded_keys(int n) { return (n + 3) & ~3; }

// Shared memory: region A holds K while the scores are formed, then the
// weights [t][padded n] and the P.V partial sums [warps][t][64]; then V,
// q (float) and the reduction slots.
__host__ __device__ constexpr size_t region_a(int t, int n) {
  return static_cast<size_t>(n) * kDim * 2 >
                 static_cast<size_t>(t) * (padded_keys(n) + kWarps * kDim) * 4
             ? static_cast<size_t>(n) * kDim * 2
             : static_cast<size_t>(t) * (padded_keys(n) + kWarps * kDim) * 4;
}

__host__ __device__ constexpr size_t smem_bytes(int t, int n) {
  return region_a(t, n) + static_cast<size_t>(n) * kDim * 2 +
         static_cast<size_t>(t) * kDim * 4 + static_cast<size_t>(kWarps) * kMaxQueries * 4;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int T>
__global__ void __launch_bounds__(kThreads, 3) history_attn_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char sm[];
  const int n = a.n;
  const int np = padded_keys(n);
  unsigned char* ks = sm;                                        // [n][128 B], swizzled
  float* ps = reinterpret_cast<float*>(sm);                      // [T][np] (after the scores)
  float* part = ps + T * np;                                     // [warps][T][64]
  unsigned char* vs = sm + region_a(T, n);                       // [n][128 B]
  float* qs = reinterpret_cast<float*>(vs + static_cast<size_t>(n) * kDim * 2);  // [T][64]
  float* red = qs + T * kDim;                                    // [warps][kMaxQueries]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t sh = blockIdx.x;           // s * H + h
  const int64_t s = sh / a.h;
  const int hh = static_cast<int>(sh - s * a.h);
  const char* kg = reinterpret_cast<const char*>(a.k + sh * n * kDim);
  const char* vg = reinterpret_cast<const char*>(a.v + sh * n * kDim);
  const int chunks = n * (kDim * 2 / 16);  // 8 chunks of 16 bytes per row
  for (int c = tid; c < chunks; c += kThreads) {
    const int row = c >> 3, col = c & 7;
    cp_async16(smem_u32(ks + row * 128 + ((col ^ (row & 7)) << 4)), kg + static_cast<size_t>(c) * 16);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int c = tid; c < chunks; c += kThreads) cp_async16(smem_u32(vs + c * 16), vg + static_cast<size_t>(c) * 16);
  asm volatile("cp.async.commit_group;" ::: "memory");
  const uint16_t* qg = a.q + sh * T * kDim;
  for (int i = tid; i < T * kDim; i += kThreads) qs[i] = bf16_bits_to_f32(qg[i]);
  const int64_t p0 = a.pos[s];
  // the slot positions of this thread's keys, loaded while K is in flight
  int64_t held[kKeysPerThread];
#pragma unroll
  for (int m = 0; m < kKeysPerThread; ++m) {
    const int j = tid + m * kThreads;
    held[m] = j < n ? a.slot_pos[s * n + j] : -1;
  }
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();

  // ---- scores: thread tid takes keys tid and tid + 256
  float sc[kKeysPerThread][T];
#pragma unroll
  for (int m = 0; m < kKeysPerThread; ++m) {
    const int j = tid + m * kThreads;
#pragma unroll
    for (int t = 0; t < T; ++t) sc[m][t] = -CUDART_INF_F;
    if (j < n) {
      float acc[T];
#pragma unroll
      for (int t = 0; t < T; ++t) acc[t] = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(ks + j * 128 + ((c ^ (j & 7)) << 4));
        float kv[8];
        unpack_bf16x8(raw, kv);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + t * kDim + c * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qs + t * kDim + c * 8 + 4);
          acc[t] = __fmaf_rn(qa.x, kv[0], acc[t]);
          acc[t] = __fmaf_rn(qa.y, kv[1], acc[t]);
          acc[t] = __fmaf_rn(qa.z, kv[2], acc[t]);
          acc[t] = __fmaf_rn(qa.w, kv[3], acc[t]);
          acc[t] = __fmaf_rn(qb.x, kv[4], acc[t]);
          acc[t] = __fmaf_rn(qb.y, kv[5], acc[t]);
          acc[t] = __fmaf_rn(qb.z, kv[6], acc[t]);
          acc[t] = __fmaf_rn(qb.w, kv[7], acc[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int64_t qp = p0 + t;
        const bool on = held[m] >= 0 && held[m] <= qp && held[m] > qp - a.context;
        sc[m][t] = on ? __fmul_rn(acc[t], a.scale) : -CUDART_INF_F;
      }
    }
  }
  // ---- softmax: block maxima, then exponentials and block sums
  float mx[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    float v = sc[0][t];
#pragma unroll
    for (int m = 1; m < kKeysPerThread; ++m) v = fmaxf(v, sc[m][t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp * kMaxQueries + t] = v;
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < T; ++t) {
    float v = red[t];
    for (int w = 1; w < kWarps; ++w) v = fmaxf(v, red[w * kMaxQueries + t]);
    mx[t] = v;
  }
  // every thread has read the maxima before the sums reuse `red`, and every
  // read of K is done before the weights overwrite it
  __syncthreads();
  float l[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    float sum = 0.0f;
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m) {
      const int j = tid + m * kThreads;
      // a query with no attended key keeps weights 0 (its output is NaN, as SDPA's)
      const float e = (j < n && mx[t] != -CUDART_INF_F) ? expf(__fsub_rn(sc[m][t], mx[t])) : 0.0f;
      if (j < n) ps[t * np + j] = e;
      sum = __fadd_rn(sum, e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    if (lane == 0) red[warp * kMaxQueries + t] = sum;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();  // V, the weights and the partial sums are visible
#pragma unroll
  for (int t = 0; t < T; ++t) {
    float v = red[t];
    for (int w = 1; w < kWarps; ++w) v = __fadd_rn(v, red[w * kMaxQueries + t]);
    l[t] = v;
  }

  // ---- P.V: warp w takes keys w, w + 8, ...; lane l dims 2l, 2l + 1
  float o0[T], o1[T];
#pragma unroll
  for (int t = 0; t < T; ++t) o0[t] = o1[t] = 0.0f;
  for (int j = warp; j < n; j += kWarps) {
    const uint32_t raw = *reinterpret_cast<const uint32_t*>(vs + j * 128 + lane * 4);
    const float v0 = __uint_as_float(raw << 16), v1 = __uint_as_float(raw & 0xffff0000u);
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float p = ps[t * np + j];
      o0[t] = __fmaf_rn(p, v0, o0[t]);
      o1[t] = __fmaf_rn(p, v1, o1[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < T; ++t)
    *reinterpret_cast<float2*>(part + (warp * T + t) * kDim + 2 * lane) = make_float2(o0[t], o1[t]);
  __syncthreads();
  for (int i = tid; i < T * kDim; i += kThreads) {
    const int t = i / kDim, d = i - t * kDim;
    float acc = part[t * kDim + d];
    for (int w = 1; w < kWarps; ++w) acc = __fadd_rn(acc, part[(w * T + t) * kDim + d]);
    float lt = l[0];
#pragma unroll
    for (int u = 1; u < T; ++u) lt = t == u ? l[u] : lt;
    a.out[((s * T + t) * a.h + hh) * kDim + d] = f32_to_bf16_bits(__fdiv_rn(acc, lt));
  }
}

// ---------------------------------------------------------------------------
// Persistent variant for many (stream, head) items: a CTA loops over items
// blockIdx.x, blockIdx.x + gridDim.x, ... (two CTAs per SM).  The arithmetic
// is that of history_attn_kernel, value for value; what changes is how the
// bytes arrive.  One thread loads an item's K block with one TMA 2-D load
// (the ring viewed as [S * H * N, 64] bf16 rows; the 128-byte swizzle
// puts 16-byte chunk c of row j at chunk c ^ (j % 8), the layout the
// per-key dot products read without bank conflicts) and its V block with
// one bulk copy, each completing on its own mbarrier; the next item's K is
// requested as soon as the current scores are formed and its V as soon as
// the current P.V is done, so HBM streams the next item while this one
// computes.  The next item's queries, slot positions and position are
// loaded into registers while the current one computes.
//
// Scores on the tensor cores: K as it lands (128-byte-swizzled rows of 64
// bf16: the K-major operand layout) is the A operand, the item's queries
// (bf16, padded to 16 rows of zeros, same layout, 2 KB) the B operand, and
// one thread issues per 128-key tile four tcgen05.mma kind::f16 (M = 128
// keys, N = 16 queries, K = 16 dims each) into 16 TMEM columns; thread tid
// < 128 then reads the scores of keys tid and tid + 128 (its TMEM lane in
// the two tiles) with one tcgen05.ld each.  The products of bf16 values are
// exact in FP32 and the tensor cores sum them in FP32, so the scores differ
// from a sequential FMA chain only by FP32 rounding (well inside the
// kernel's bound against float64 attention); this replaces 512 FMAs and 80
// shared-memory loads per scoring thread and item.  n <= 256 (one
// TMA box).  Every wait is bounded (~2 s, MOSS_ERR_TIMEOUT).
constexpr int kStreamMaxKeys = 256;

struct StreamArgs {
  CUtensorMap k_map;  // k_cache as [S * H * N, 64] bf16, box {64, n}, 128-byte swizzle
  Args a;
  int64_t items;
  // With the rotary fused in (moss_history_attention_qkv): the qkv
  // projection's output [S * T, 3 * H * 64] bf16 (row s * T + t: q, k, v of
  // every head), the ring slot of every token [S, T], the rotary frequency
  // coefficient; k_cache and v_cache (a.k, a.v) receive the chunk's keys and
  // values.
  const uint16_t* qkv;
  const int64_t* slots;
  float coef;
};

constexpr int kScoreRows = 16;  // MMA N: the queries, padded with zero rows

__host__ __device__ constexpr size_t stream_smem(int t, int n) {
  // K (whole 1024-byte swizzle atoms) | the queries as the MMA's B operand
  // (16 rows x 128 bytes, swizzled) | V | weights [n][4 or 8] (key-major,
  // so P.V reads one key's weights of every query with one vector load) |
  // partial sums [warps][t][64] | reduction slots | 3 mbarriers and the TMEM
  // address
  return static_cast<size_t>((n + 7) / 8) * 1024 + kScoreRows * 128 +
         static_cast<size_t>(n) * kDim * 2 +
         static_cast<size_t>(n) * (t <= 4 ? 4 : 8) * 4 + static_cast<size_t>(kWarps) * t * kDim * 4 +
         static_cast<size_t>(kWarps) * kMaxQueries * 4 + 32 + 1024;
}

// K-major operand with the 128-byte swizzle (the TMA layout): 128-byte rows,
// 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// kind::f16, D f32, A and B bf16 K-major, M = 128, N = 16.
constexpr uint32_t kScoreIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((kScoreRows >> 3) << 17) | ((128u >> 4) << 24);
__device__ __forceinline__ void mma_score(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kScoreIdesc), "r"(acc)
      : "memory");
}
// 8 accumulator columns of this thread's TMEM lane (whole warp), then wait.
__device__ __forceinline__ void tmem_load8(uint32_t taddr, uint32_t (&r)[8]) {
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
}

__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap* map, int row,
                                              unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(pipe::smem_u32(bar))
      : "memory");
}

template <int T, bool FUSED>
__global__ void __launch_bounds__(kThreads, 2) history_attn_stream_kernel(
    const __grid_constant__ StreamArgs sa) {
  extern __shared__ unsigned char smem_raw[];
  const Args& a = sa.a;
  const int n = a.n;
  constexpr int TP = T <= 4 ? 4 : 8;  // weights per key row (queries, padded)
  unsigned char* ks = smem_raw + ((1024u - (static_cast<uint32_t>(
                                                 __cvta_generic_to_shared(smem_raw)) & 1023u)) &
                                  1023u);
  unsigned char* qimg = ks + static_cast<size_t>((n + 7) / 8) * 1024;  // [16][128 B], swizzled
  unsigned char* vs = qimg + kScoreRows * 128;
  float* ps = reinterpret_cast<float*>(vs + static_cast<size_t>(n) * kDim * 2);  // [n][TP]
  float* part = ps + n * TP;                                                     // [warps][T][64]
  float* red = part + kWarps * T * kDim;                                         // [warps][8]
  unsigned long long* kfull = reinterpret_cast<unsigned long long*>(red + kWarps * kMaxQueries);
  unsigned long long* vfull = kfull + 1;
  unsigned long long* sfull = kfull + 2;  // the scores are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kfull + 3);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t bytes = static_cast<uint32_t>(n) * kDim * 2;
  int64_t item = blockIdx.x;
  if (item >= sa.items) return;  // uniform over the CTA

  if (tid == 0) {
    pipe::mbar_init(kfull, 1);
    pipe::mbar_init(vfull, 1);
    pipe::mbar_init(sfull, 1);
    pipe::fence_mbar_init();
  }
  // the padding rows of the query operand stay zero
  for (int i = tid; i < kScoreRows * 128 / 16; i += kThreads)
    reinterpret_cast<uint4*>(qimg)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 0) tc::alloc(tmem_slot, 32);  // two 128-key tiles x 16 columns
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  auto issue_k = [&](int64_t it) {
    pipe::mbar_arrive_expect_tx(kfull, bytes);
    tma_load_rows(pipe::smem_u32(ks), &sa.k_map, static_cast<int>(it * n), kfull);
  };
  auto issue_v = [&](int64_t it) {
    pipe::mbar_arrive_expect_tx(vfull, bytes);
    pipe::bulk_g2s(vs, a.v + it * n * kDim, bytes, vfull);
  };
  if (tid == 0) {
    issue_k(item);
    issue_v(item);
  }
  // Keys: thread tid < 128 scores keys tid and tid + 128 (every query
  // value it loads serves two keys); the other threads score none.
  constexpr int kPair = kStreamMaxKeys / 2;
  static_assert(kKeysPerThread == 2 && 2 * kPair == kStreamMaxKeys,
                "128 threads x 2 keys must cover the ring");
  auto key_of = [&](int m) { return tid < kPair ? tid + m * kPair : kStreamMaxKeys; };
  // this item's queries, slot positions and position, in registers
  auto load_meta = [&](int64_t it, float (&qv)[(T * kDim + kThreads - 1) / kThreads],
                       int64_t (&held)[kKeysPerThread], int64_t& p0) {
    const int64_t s = it / a.h;
    const uint16_t* qg = a.q + it * T * kDim;
#pragma unroll
    for (int c = 0; c < (T * kDim + kThreads - 1) / kThreads; ++c) {
      const int i = tid + c * kThreads;
      qv[c] = i < T * kDim ? bf16_bits_to_f32(qg[i]) : 0.0f;
    }
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m) {
      const int j = key_of(m);
      held[m] = j < n ? a.slot_pos[s * n + j] : -1;
    }
    p0 = a.pos[s];
  };
  // the slot positions and the position only (the queries come from qkv)
  auto load_meta_keys = [&](int64_t it, int64_t (&held)[kKeysPerThread], int64_t& p0) {
    const int64_t s = it / a.h;
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m) {
      const int j = key_of(m);
      held[m] = j < n ? a.slot_pos[s * n + j] : -1;
    }
    p0 = a.pos[s];
  };
  // Fused rotary: thread tid < 32 T owns dims 2p, 2p + 1 (p = tid % 32) of
  // token tid / 32: it reads that pair of q, k and v from the projection's
  // output and the token's ring slot.
  constexpr int kPairThreads = 32 * T;
  auto load_pairs = [&](int64_t it, uint32_t (&raw)[3], int64_t& slot) {
    if (FUSED && tid < kPairThreads) {
      const int64_t s = it / a.h;
      const int hh = static_cast<int>(it - s * a.h);
      const int tq = tid >> 5, p = tid & 31;
      const uint32_t* row =
          reinterpret_cast<const uint32_t*>(sa.qkv + (s * T + tq) * (3 * a.h * kDim));
      raw[0] = row[hh * (kDim / 2) + p];
      raw[1] = row[(a.h + hh) * (kDim / 2) + p];
      raw[2] = row[(2 * a.h + hh) * (kDim / 2) + p];
      slot = sa.slots[s * T + tq];
    }
  };
  constexpr int QC = (T * kDim + kThreads - 1) / kThreads;
  float qv[QC];
  int64_t held[kKeysPerThread];
  int64_t p0;
  uint32_t raw[3] = {0u, 0u, 0u};
  int64_t slot = 0;
  if (!FUSED) load_meta(item, qv, held, p0);
  if (FUSED) {
    load_meta_keys(item, held, p0);
    load_pairs(item, raw, slot);
  }
  int issued_k = 1, issued_v = 1, done_k = 0, done_v = 0, issued_s = 0, done_s = 0;
  for (int i = 0;; ++i) {
    const int64_t s = item / a.h;
    const int hh = static_cast<int>(item - s * a.h);
    const int64_t next = item + gridDim.x;
    const bool more = next < sa.items;
    uint32_t kbits = 0u;  // fused: this thread's rotated key pair (bf16 x 2)
    if constexpr (FUSED) {
      if (tid < kPairThreads) {
        // moss_rope_kv's arithmetic: phase = exp(p * coef) * (pos + t),
        // each product and sum rounded, one bf16 rounding per output
        const int tq = tid >> 5, p = tid & 31;
        const float ts = __fadd_rn(static_cast<float>(p0), static_cast<float>(tq));
        const float phase = __fmul_rn(expf(__fmul_rn(static_cast<float>(p), sa.coef)), ts);
        const float c = cosf(phase), sn = sinf(phase);
        float o0, o1;
        rotate_pair(__uint_as_float(raw[0] << 16), __uint_as_float(raw[0] & 0xffff0000u), c, sn,
                    o0, o1);
        *reinterpret_cast<uint32_t*>(qimg + (tq & 7) * 128 + ((((2 * p) >> 3) ^ (tq & 7)) << 4) +
                                     ((2 * p) & 7) * 2) = pack_bf16x2(o0, o1);
        rotate_pair(__uint_as_float(raw[1] << 16), __uint_as_float(raw[1] & 0xffff0000u), c, sn,
                    o0, o1);
        kbits = pack_bf16x2(o0, o1);
      }
    } else {
#pragma unroll
      for (int c = 0; c < QC; ++c) {
        const int q = tid + c * kThreads;
        if (q < T * kDim) {
          // the MMA's B operand: row t, dim d (bf16, exact: qv holds bf16 values)
          const int tq = q / kDim, d = q - tq * kDim;
          *reinterpret_cast<uint16_t*>(qimg + (tq & 7) * 128 + ((((d >> 3) ^ (tq & 7)) << 4)) +
                                       (d & 7) * 2) = f32_to_bf16_bits(qv[c]);
        }
      }
    }
    tc::fence_async_shared();  // the query operand is visible to the tensor cores
    const int kok = pipe::mbar_wait(kfull, i & 1) ? 1 : 0;
    done_k = i + kok;  // loads this thread saw land
    if constexpr (FUSED) {
      // the chunk's rotated keys: into the ring for the chunks after this
      // one, and over the (stale) rows of their slots in the landed K tile
      if (kok && tid < kPairThreads) {
        const int p = tid & 31;
        if (slot >= 0 && slot < n) {
          *reinterpret_cast<uint32_t*>(ks + (slot >> 3) * 1024 + (slot & 7) * 128 +
                                       ((((2 * p) >> 3) ^ (static_cast<int>(slot) & 7)) << 4) +
                                       ((2 * p) & 7) * 2) = kbits;
          reinterpret_cast<uint32_t*>(const_cast<uint16_t*>(a.k))[(item * n + slot) * (kDim / 2) + p] =
              kbits;
        } else {
          record_device_error(MOSS_ERR_VALUE);
        }
      }
      tc::fence_async_shared();  // the patched rows are visible to the tensor cores
    }
    if (__syncthreads_or(!kok)) break;  // K and the queries are visible to all
    if (tid == 0) {
      // scores: per 128-key tile 4 MMAs of K = 16 dims into 16 columns
      tc::fence_after();
      const uint32_t kb = pipe::smem_u32(ks), qb = pipe::smem_u32(qimg);
      for (int tile = 0; tile * 128 < n; ++tile) {
#pragma unroll
        for (int kk = 0; kk < kDim / 16; ++kk)
          mma_score(tmem + static_cast<uint32_t>(tile * kScoreRows),
                    sw128_desc(kb + static_cast<uint32_t>(tile) * 16384u + kk * 32u),
                    sw128_desc(qb + kk * 32u), kk > 0 ? 1u : 0u);
      }
      tc::commit(sfull);
      ++issued_s;
    }
    const int sok = pipe::mbar_wait(sfull, i & 1) ? 1 : 0;
    done_s = i + sok;
    tc::fence_after();
    // ---- scores: thread tid < 128 takes keys tid and tid + 128; each key's
    // dot products are summed in the same order as history_attn_kernel's
    float sc[kKeysPerThread][T];
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m)
#pragma unroll
      for (int t = 0; t < T; ++t) sc[m][t] = -CUDART_INF_F;
    if (tid < kPair) {
      const int j0 = tid, j1 = tid + kPair;
      const bool v0 = j0 < n, v1 = j1 < n;  // rows past n are never read
      // this thread's TMEM lane holds key j0 in tile 0 and key j1 in tile 1
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      uint32_t r0[8], r1[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      tmem_load8(lane_addr, r0);
      if (n > kPair) tmem_load8(lane_addr + kScoreRows, r1);
      float acc0[T], acc1[T];
#pragma unroll
      for (int t = 0; t < T; ++t) {
        acc0[t] = __uint_as_float(r0[t]);
        acc1[t] = __uint_as_float(r1[t]);
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int64_t qp = p0 + t;
        const bool on0 = v0 && held[0] >= 0 && held[0] <= qp && held[0] > qp - a.context;
        const bool on1 = v1 && held[1] >= 0 && held[1] <= qp && held[1] > qp - a.context;
        sc[0][t] = on0 ? __fmul_rn(acc0[t], a.scale) : -CUDART_INF_F;
        sc[1][t] = on1 ? __fmul_rn(acc1[t], a.scale) : -CUDART_INF_F;
      }
    }
    float mx[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float v = sc[0][t];
#pragma unroll
      for (int m = 1; m < kKeysPerThread; ++m) v = fmaxf(v, sc[m][t]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) red[warp * kMaxQueries + t] = v;
    }
    tc::fence_before();
    if (__syncthreads_or(!sok)) break;  // every read of K and of the scores is done
    if (tid == 0 && more) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue_k(next);
      ++issued_k;
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float v = red[t];
      for (int w = 1; w < kWarps; ++w) v = fmaxf(v, red[w * kMaxQueries + t]);
      mx[t] = v;
    }
    __syncthreads();  // the maxima are read before `red` takes the sums
    float l[T];
    float sum[T];
#pragma unroll
    for (int t = 0; t < T; ++t) sum[t] = 0.0f;
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m) {
      const int j = key_of(m);
      float e[TP];
#pragma unroll
      for (int t = 0; t < TP; ++t) e[t] = 0.0f;
#pragma unroll
      for (int t = 0; t < T; ++t) {
        e[t] = (j < n && mx[t] != -CUDART_INF_F) ? expf(__fsub_rn(sc[m][t], mx[t])) : 0.0f;
        sum[t] = __fadd_rn(sum[t], e[t]);
      }
      if (j < n) {
#pragma unroll
        for (int c = 0; c < TP / 4; ++c)
          *reinterpret_cast<float4*>(ps + j * TP + 4 * c) =
              make_float4(e[4 * c], e[4 * c + 1], e[4 * c + 2], e[4 * c + 3]);
      }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float s_t = sum[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s_t = __fadd_rn(s_t, __shfl_xor_sync(0xffffffffu, s_t, o));
      if (lane == 0) red[warp * kMaxQueries + t] = s_t;
    }
    // the next item's metadata while V lands
    float qn[QC];
    int64_t heldn[kKeysPerThread];
    int64_t p0n = 0;
    uint32_t rawn[3] = {0u, 0u, 0u};
    int64_t slotn = 0;
    if (more) {
      if constexpr (FUSED) {
        load_meta_keys(next, heldn, p0n);
        load_pairs(next, rawn, slotn);
      } else {
        load_meta(next, qn, heldn, p0n);
      }
    }
    const int vok = pipe::mbar_wait(vfull, i & 1) ? 1 : 0;
    done_v = i + vok;
    if constexpr (FUSED) {
      // the chunk's values: into the ring and over their slots' rows of V
      if (vok && tid < kPairThreads && slot >= 0 && slot < n) {
        const int p = tid & 31;
        *reinterpret_cast<uint32_t*>(vs + slot * 128 + p * 4) = raw[2];
        reinterpret_cast<uint32_t*>(const_cast<uint16_t*>(a.v))[(item * n + slot) * (kDim / 2) + p] =
            raw[2];
      }
    }
    if (__syncthreads_or(!vok)) break;  // V, the weights and the sums are visible
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float v = red[t];
      for (int w = 1; w < kWarps; ++w) v = __fadd_rn(v, red[w * kMaxQueries + t]);
      l[t] = v;
    }
    // ---- P.V: warp w takes keys w, w + 8, ...; lane l dims 2l, 2l + 1
    float o0[T], o1[T];
#pragma unroll
    for (int t = 0; t < T; ++t) o0[t] = o1[t] = 0.0f;
    for (int j = warp; j < n; j += kWarps) {
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(vs + j * 128 + lane * 4);
      const float v0 = __uint_as_float(raw << 16), v1 = __uint_as_float(raw & 0xffff0000u);
      float p[TP];
#pragma unroll
      for (int c = 0; c < TP / 4; ++c) {
        const float4 p4 = *reinterpret_cast<const float4*>(ps + j * TP + 4 * c);
        p[4 * c] = p4.x; p[4 * c + 1] = p4.y; p[4 * c + 2] = p4.z; p[4 * c + 3] = p4.w;
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        o0[t] = __fmaf_rn(p[t], v0, o0[t]);
        o1[t] = __fmaf_rn(p[t], v1, o1[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < T; ++t)
      *reinterpret_cast<float2*>(part + (warp * T + t) * kDim + 2 * lane) = make_float2(o0[t], o1[t]);
    __syncthreads();  // every read of V is done: the next item's V may come in
    if (tid == 0 && more) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue_v(next);
      ++issued_v;
    }
    for (int e = tid; e < T * kDim; e += kThreads) {
      const int t = e / kDim, d = e - t * kDim;
      float acc = part[t * kDim + d];
      for (int w = 1; w < kWarps; ++w) acc = __fadd_rn(acc, part[(w * T + t) * kDim + d]);
      float lt = l[0];
#pragma unroll
      for (int u = 1; u < T; ++u) lt = t == u ? l[u] : lt;
      a.out[((s * T + t) * a.h + hh) * kDim + d] = f32_to_bf16_bits(__fdiv_rn(acc, lt));
    }
    if (!more) break;
    item = next;
    if constexpr (FUSED) {
#pragma unroll
      for (int e = 0; e < 3; ++e) raw[e] = rawn[e];
      slot = slotn;
    } else {
#pragma unroll
      for (int c = 0; c < QC; ++c) qv[c] = qn[c];
    }
#pragma unroll
    for (int m = 0; m < kKeysPerThread; ++m) held[m] = heldn[m];
    p0 = p0n;
    __syncthreads();  // `part` and `ps` are read before they are rewritten
  }
  // after a timeout: the copies still in flight land before the CTA retires
  if (tid == 0) {
    for (int i = done_k; i < issued_k; ++i) pipe::mbar_wait(kfull, i & 1);
    for (int i = done_v; i < issued_v; ++i) pipe::mbar_wait(vfull, i & 1);
    // and the score MMAs still in flight finish before the TMEM is freed
    for (int i = done_s; i < issued_s; ++i) pipe::mbar_wait(sfull, i & 1);
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 0) tc::dealloc(tmem, 32);
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The key ring as [rows, 64] bf16 with a box of n rows and the 128-byte swizzle.
bool encode_ring(CUtensorMap* map, const void* base, int64_t rows, int n) {
  static EncodeTiled fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiled>(f);
  }();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kDim) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kDim), static_cast<cuuint32_t>(n)};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Launches the persistent kernel over its one wave of CTAs (two per SM).
template <bool FUSED>
int launch_stream(const StreamArgs& sa, int t, int n, cudaStream_t st, const char* name) {
  const size_t sh = stream_smem(t, n);
  const size_t sh_max = stream_smem(kMaxQueries, kStreamMaxKeys);
  const int64_t sms = sm_count();
  const unsigned sgrid = static_cast<unsigned>(2 * sms < sa.items ? 2 * sms : sa.items);
#define MOSS_HATTN_STREAM(T)                                                            \
  case T: {                                                                             \
    static bool attr_done[kMaxDevices] = {};                                            \
    allow_dynamic_smem(history_attn_stream_kernel<T, FUSED>, sh_max, attr_done);        \
    history_attn_stream_kernel<T, FUSED><<<sgrid, kThreads, sh, st>>>(sa);              \
    break;                                                                              \
  }
  switch (t) {
    MOSS_HATTN_STREAM(1) MOSS_HATTN_STREAM(2) MOSS_HATTN_STREAM(3) MOSS_HATTN_STREAM(4)
    MOSS_HATTN_STREAM(5) MOSS_HATTN_STREAM(6) MOSS_HATTN_STREAM(7) MOSS_HATTN_STREAM(8)
    default: break;
  }
#undef MOSS_HATTN_STREAM
  return launch_status(name);
}

}  // namespace hattn
}  // namespace moss

using namespace moss;

extern "C" int moss_history_attention(const void* q, const void* k_cache, const void* v_cache,
                                      const int64_t* slot_pos, const int64_t* pos, int64_t s,
                                      int64_t h, int64_t t, int64_t n, int64_t d, int64_t context,
                                      float scale, void* out, void* stream) {
  using namespace hattn;
  const char* name = "moss_history_attention";
  if (s < 0 || h < 1 || t < 1 || n < 1 || context < 1)
    return fail(MOSS_ERR_VALUE, "%s: need streams >= 0, heads, queries, slots and context >= 1", name);
  if (d != kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only heads of 64 are supported", name);
  if (t > kMaxQueries) return fail(MOSS_ERR_UNSUPPORTED, "%s: at most %d queries per stream", name, kMaxQueries);
  if (n > kMaxKeys) return fail(MOSS_ERR_UNSUPPORTED, "%s: at most %d history slots", name, kMaxKeys);
  if (s * h > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many streams x heads", name);
  if (s == 0) return MOSS_OK;
  if (!q || !k_cache || !v_cache || !slot_pos || !pos || !out)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(MOSS_ERR_VALUE, "%s: the history rings must be 16-byte aligned", name);
  Args a{static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k_cache),
         static_cast<const uint16_t*>(v_cache), slot_pos, pos, static_cast<uint16_t*>(out),
         context, scale, static_cast<int>(h), static_cast<int>(t), static_cast<int>(n)};
  cudaStream_t st = as_stream(stream);
  // many items of at most 256 slots: the persistent kernel (two CTAs per SM
  // streaming the next item while computing this one)
  const int64_t items = s * h;
  const int64_t sms = sm_count();
  if (n <= kStreamMaxKeys && items >= 2 * sms && items * n < 0x7fffffffLL) {
    StreamArgs sa{};
    if (!encode_ring(&sa.k_map, k_cache, items * n, static_cast<int>(n)))
      return fail(MOSS_ERR_CUDA, "%s: tensor map encoding failed", name);
    sa.a = a;
    sa.items = items;
    return launch_stream<false>(sa, static_cast<int>(t), static_cast<int>(n), st, name);
  }
  const size_t shmem = smem_bytes(static_cast<int>(t), static_cast<int>(n));
  const unsigned grid = static_cast<unsigned>(s * h);
#define MOSS_HATTN(T)                                                                   \
  case T: {                                                                             \
    static bool attr_done[kMaxDevices] = {};                                            \
    allow_dynamic_smem(history_attn_kernel<T>, shmem_max, attr_done);                   \
    history_attn_kernel<T><<<grid, kThreads, shmem, st>>>(a);                           \
    break;                                                                              \
  }
  const size_t shmem_max = smem_bytes(kMaxQueries, kMaxKeys);
  switch (t) {
    MOSS_HATTN(1) MOSS_HATTN(2) MOSS_HATTN(3) MOSS_HATTN(4)
    MOSS_HATTN(5) MOSS_HATTN(6) MOSS_HATTN(7) MOSS_HATTN(8)
    default: break;
  }
#undef MOSS_HATTN
  return launch_status(name);
}

extern "C" int moss_history_attention_qkv(const void* qkv, const int64_t* slots, float freq_coef,
                                          void* k_cache, void* v_cache, const int64_t* slot_pos,
                                          const int64_t* pos, int64_t s, int64_t h, int64_t t,
                                          int64_t n, int64_t d, int64_t context, float scale,
                                          void* out, void* stream) {
  using namespace hattn;
  const char* name = "moss_history_attention_qkv";
  if (s < 0 || h < 1 || t < 1 || n < 1 || context < 1)
    return fail(MOSS_ERR_VALUE, "%s: need streams >= 0, heads, queries, slots and context >= 1", name);
  if (d != kDim) return fail(MOSS_ERR_UNSUPPORTED, "%s: only heads of 64 are supported", name);
  if (s == 0) return MOSS_OK;
  if (!qkv || !slots || !k_cache || !v_cache || !slot_pos || !pos || !out)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(MOSS_ERR_VALUE, "%s: qkv and the history rings must be 16-byte aligned", name);
  // the persistent kernel's range only: many (stream, head) items, rings of
  // at most 256 slots, at most 8 queries
  const int64_t items = s * h;
  const int64_t sms = sm_count();
  if (t > kMaxQueries || n > kStreamMaxKeys || items < 2 * sms || items * n >= 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: needs at most %d queries, at most %d slots and at least %lld (stream, head) "
                "items; use moss_rope_kv and moss_history_attention",
                name, kMaxQueries, kStreamMaxKeys, static_cast<long long>(2 * sms));
  StreamArgs sa{};
  if (!encode_ring(&sa.k_map, k_cache, items * n, static_cast<int>(n)))
    return fail(MOSS_ERR_CUDA, "%s: tensor map encoding failed", name);
  sa.a = Args{nullptr, static_cast<const uint16_t*>(k_cache), static_cast<const uint16_t*>(v_cache),
              slot_pos, pos, static_cast<uint16_t*>(out), context, scale, static_cast<int>(h),
              static_cast<int>(t), static_cast<int>(n)};
  sa.items = items;
  sa.qkv = static_cast<const uint16_t*>(qkv);
  sa.slots = slots;
  sa.coef = freq_coef;
  return launch_stream<true>(sa, static_cast<int>(t), static_cast<int>(n), as_stream(stream), name);
}
