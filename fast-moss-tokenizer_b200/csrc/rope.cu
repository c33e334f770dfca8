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
// Work decomposition: a tile is one batch index and TT time steps for ALL
// heads, so the phase table of a tile (TT x d/2 (c, s) pairs, evaluated once
// into shared memory -- the phase does not depend on the head) serves every
// head.  Three kernels share that decomposition:
//   * rope_stream_kernel, for q and k whose time rows are contiguous within
//     each head: bulk copies stage whole tiles in shared memory (one CTA
//     per SM, producer thread + consumer warps);
//   * rope_vec_kernel, for other layouts with 16-byte rows (innermost
//     stride 1, e.g. a qkv projection output viewed as [b,h,t,d]):
//     persistent blocks that issue the next tile's loads and phase table
//     before rotating the current one;
//   * rope_pair_kernel, one interleaved pair per item, for any strides.
#include "pipeline.cuh"

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

// Fills the (c, s) pairs of this CTA's tile: [tt][half] each.
__device__ __forceinline__ void fill_phase(const RopeArgs& a, int64_t bi, int64_t t0, int tt,
                                           int half, float* sc, float* ss) {
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
}

#ifndef MOSS_ROPE_ITEMS
#define MOSS_ROPE_ITEMS 1
#endif
constexpr int kRopeItems = MOSS_ROPE_ITEMS;  // 16-byte q/k items per thread and tile

// Vector path: VW elements (16 bytes) per item, KI items per thread and
// tile.  A thread's items sit at the same place in every tile, so their
// offsets are computed once; persistent blocks then walk the tiles with a
// grid stride, issuing the loads of the next tile and its phase table
// (double-buffered in shared memory) before the current tile is rotated.
template <int KI>
struct ItemSlots {
  int64_t q[KI], k[KI], o[KI];  // element offsets from the tile's base
  int tl[KI];                   // time step within the tile (large: no item)
  int toff[KI];                 // first (c, s) pair of the item in the tile table
};

template <int KI>
struct TileData {
  uint4 q[KI], k[KI];
  bool ok[KI];
  int64_t bi, t0;
};

template <int DT, int KI>
__device__ __forceinline__ void load_tile(const RopeArgs& a, uint32_t tile, uint32_t ntiles_t,
                                          const ItemSlots<KI>& sl, TileData<KI>& v) {
  constexpr int kEs = DT == MOSS_BF16 ? 2 : 4;
  const uint32_t bi = tile / ntiles_t;
  v.bi = bi;
  v.t0 = static_cast<int64_t>(tile - bi * ntiles_t) * a.tt;
  const int64_t qb = v.bi * a.qs[0] + v.t0 * a.qs[2];
  const int64_t kb = v.bi * a.ks[0] + v.t0 * a.ks[2];
  const char* q = static_cast<const char*>(a.q);
  const char* k = static_cast<const char*>(a.k);
#pragma unroll
  for (int j = 0; j < KI; ++j) {
    v.ok[j] = v.t0 + sl.tl[j] < a.t;
    if (v.ok[j]) {
      v.q[j] = *reinterpret_cast<const uint4*>(q + (qb + sl.q[j]) * kEs);
      v.k[j] = *reinterpret_cast<const uint4*>(k + (kb + sl.k[j]) * kEs);
    }
  }
}

// (c, s) pairs of one tile: [tt][half] each, from the per-dimension freq.
__device__ __forceinline__ void fill_tile_phase(const RopeArgs& a, int64_t bi, int64_t t0,
                                                int half, const float* freq, float* sc,
                                                float* ss) {
  const float off = offset_as_float(a.offset, a.offset_dtype, bi);
  const int tbl = a.tt * half;
  for (int i = threadIdx.x; i < tbl; i += blockDim.x) {
    const int tl = i / half;
    const int j = i - tl * half;
    const float ts = __fadd_rn(off, static_cast<float>(t0 + tl));
    const float phase = __fmul_rn(freq[j], ts);
    sc[i] = cosf(phase);
    ss[i] = sinf(phase);
  }
}

template <int DT, bool TABLES, int KI>
__device__ __forceinline__ void rotate_tile(const RopeArgs& a, int half, const ItemSlots<KI>& sl,
                                            const TileData<KI>& v, const float* sc,
                                            const float* ss) {
  constexpr int VW = DT == MOSS_BF16 ? 8 : 4;
  const int64_t ob = (v.bi * a.h * a.t + v.t0) * a.d;
  const int64_t tb = (v.bi * a.t + v.t0) * half;
#pragma unroll
  for (int j = 0; j < KI; ++j) {
    if (!v.ok[j]) continue;
    float c[VW / 2], s[VW / 2];
    if constexpr (TABLES) {
#pragma unroll
      for (int p = 0; p < VW / 2; ++p) {
        c[p] = a.cos_t[tb + sl.toff[j] + p];
        s[p] = a.sin_t[tb + sl.toff[j] + p];
      }
    } else {
#pragma unroll
      for (int p = 0; p < VW / 2; ++p) {
        c[p] = sc[sl.toff[j] + p];
        s[p] = ss[sl.toff[j] + p];
      }
    }
    float qv[VW], kv[VW], qo[VW], ko[VW];
    if constexpr (DT == MOSS_BF16) {
      unpack_bf16x8(v.q[j], qv);
      unpack_bf16x8(v.k[j], kv);
    } else {
      qv[0] = __uint_as_float(v.q[j].x); qv[1] = __uint_as_float(v.q[j].y);
      qv[2] = __uint_as_float(v.q[j].z); qv[3] = __uint_as_float(v.q[j].w);
      kv[0] = __uint_as_float(v.k[j].x); kv[1] = __uint_as_float(v.k[j].y);
      kv[2] = __uint_as_float(v.k[j].z); kv[3] = __uint_as_float(v.k[j].w);
    }
#pragma unroll
    for (int p = 0; p < VW / 2; ++p) {
      rotate_pair(qv[2 * p], qv[2 * p + 1], c[p], s[p], qo[2 * p], qo[2 * p + 1]);
      rotate_pair(kv[2 * p], kv[2 * p + 1], c[p], s[p], ko[2 * p], ko[2 * p + 1]);
    }
    const int64_t o = ob + sl.o[j];
    if constexpr (DT == MOSS_BF16) {
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.oq) + o) = pack_bf16x8(qo);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.ok) + o) = pack_bf16x8(ko);
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(a.oq) + o) = make_float4(qo[0], qo[1], qo[2], qo[3]);
      *reinterpret_cast<float4*>(static_cast<float*>(a.ok) + o) = make_float4(ko[0], ko[1], ko[2], ko[3]);
    }
  }
}

// Shared memory (phase mode): freq[d/2] padded to 4 floats, then two
// buffers of {cos, sin} x [tt][d/2].
template <int DT, bool TABLES, int KI>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeArgs a, uint32_t ntiles_total) {
  constexpr int VW = DT == MOSS_BF16 ? 8 : 4;
  extern __shared__ float smem[];
  uint32_t tile = blockIdx.x;
  if (tile >= ntiles_total) return;
  const int half = static_cast<int>(a.d >> 1);
  const int tbl = a.tt * half;
  const int nvec = static_cast<int>(a.d / VW);
  const int items = static_cast<int>(a.h) * a.tt * nvec;
  const uint32_t ntiles_t = static_cast<uint32_t>((a.t + a.tt - 1) / a.tt);
  ItemSlots<KI> sl;
#pragma unroll
  for (int j = 0; j < KI; ++j) {
    const int it = threadIdx.x + j * 256;
    sl.q[j] = sl.k[j] = sl.o[j] = 0;
    sl.toff[j] = 0;
    sl.tl[j] = 0x3fffffff;
    if (it < items) {
      const int vec = it % nvec;
      const int rest = it / nvec;
      const int tl = rest % a.tt;
      const int64_t hi = rest / a.tt;
      sl.q[j] = hi * a.qs[1] + tl * a.qs[2] + vec * VW;
      sl.k[j] = hi * a.ks[1] + tl * a.ks[2] + vec * VW;
      sl.o[j] = (hi * a.t + tl) * a.d + vec * VW;
      sl.tl[j] = tl;
      sl.toff[j] = tl * half + vec * (VW / 2);
    }
  }
  const int fpad = (half + 3) & ~3;
  float* freq = smem;
  float* tabs = smem + fpad;
  TileData<KI> cur, nxt;
  load_tile<DT, KI>(a, tile, ntiles_t, sl, cur);
  int buf = 0;
  if constexpr (!TABLES) {
    for (int j = threadIdx.x; j < half; j += blockDim.x)
      freq[j] = expf(__fmul_rn(static_cast<float>(j), a.coef));
    __syncthreads();
    fill_tile_phase(a, cur.bi, cur.t0, half, freq, tabs, tabs + tbl);
    __syncthreads();
  }
  while (true) {
    const uint32_t next = tile + gridDim.x;
    const bool has_next = next < ntiles_total;
    if (has_next) {
      load_tile<DT, KI>(a, next, ntiles_t, sl, nxt);
      if constexpr (!TABLES) {
        float* nb = tabs + (buf ^ 1) * 2 * tbl;
        fill_tile_phase(a, nxt.bi, nxt.t0, half, freq, nb, nb + tbl);
      }
    }
    const float* cb = tabs + buf * 2 * tbl;
    rotate_tile<DT, TABLES, KI>(a, half, sl, cur, cb, cb + tbl);
    if (!has_next) break;
    if constexpr (!TABLES) __syncthreads();
    cur = nxt;
    tile = next;
    buf ^= 1;
  }
}

// Generic path: one interleaved pair per item, arbitrary element strides.
template <int DT, bool TABLES>
__global__ void __launch_bounds__(256) rope_pair_kernel(RopeArgs a) {
  extern __shared__ float smem[];
  const int half = static_cast<int>(a.d >> 1);
  const int64_t ntiles = (a.t + a.tt - 1) / a.tt;
  const int64_t bi = blockIdx.x / ntiles;
  const int64_t t0 = (blockIdx.x % ntiles) * a.tt;
  const int tt = static_cast<int>(a.t - t0 < a.tt ? a.t - t0 : a.tt);
  float* sc = smem;
  float* ss = smem + a.tt * half;
  if constexpr (!TABLES) {
    fill_phase(a, bi, t0, tt, half, sc, ss);
    __syncthreads();
  }
  const int items = static_cast<int>(a.h) * tt * half;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int p = it % half;
    const int rest = it / half;
    const int tl = rest % tt;
    const int64_t hi = rest / tt;
    const int64_t ti = t0 + tl;
    float c, s;
    if constexpr (TABLES) {
      c = a.cos_t[(bi * a.t + ti) * half + p];
      s = a.sin_t[(bi * a.t + ti) * half + p];
    } else {
      c = sc[tl * half + p];
      s = ss[tl * half + p];
    }
    const int64_t qb = bi * a.qs[0] + hi * a.qs[1] + ti * a.qs[2] + 2 * p * a.qs[3];
    const int64_t kb = bi * a.ks[0] + hi * a.ks[1] + ti * a.ks[2] + 2 * p * a.ks[3];
    float q0, q1, k0, k1;
    rotate_pair(load_as_f32<DT>(a.q, qb), load_as_f32<DT>(a.q, qb + a.qs[3]), c, s, q0, q1);
    rotate_pair(load_as_f32<DT>(a.k, kb), load_as_f32<DT>(a.k, kb + a.ks[3]), c, s, k0, k1);
    const int64_t o = ((bi * a.h + hi) * a.t + ti) * a.d + 2 * p;
    store_from_f32<DT>(a.oq, o, q0);
    store_from_f32<DT>(a.oq, o + 1, q1);
    store_from_f32<DT>(a.ok, o, k0);
    store_from_f32<DT>(a.ok, o + 1, k1);
  }
}

// ------------------------------------------------------------------ rope + history
// RoPE whose rotated keys (and the values) go straight into an attention
// history ring: one CTA per batch index and time tile (the phase table of
// the tile shared by all heads, as rope_pair_kernel), one thread per
// interleaved pair and head.  q -> oq contiguous [b,h,t,d]; k -> k_cache and
// v -> v_cache at [b, h, slot[b, t], :] of contiguous [b, h, S, d] rings.  A
// slot outside [0, S) is skipped and recorded in the device error word.
struct RopeKvArgs {
  RopeArgs r;
  const void* v;
  int64_t vs[4];
  const int64_t* slots;  // [b, t]
  void* k_cache;
  void* v_cache;
  int64_t cache_slots;
};

template <int DT>
__global__ void __launch_bounds__(256) rope_kv_kernel(RopeKvArgs ka) {
  extern __shared__ float smem[];
  const RopeArgs& a = ka.r;
  const int half = static_cast<int>(a.d >> 1);
  const int64_t ntiles = (a.t + a.tt - 1) / a.tt;
  const int64_t bi = blockIdx.x / ntiles;
  const int64_t t0 = (blockIdx.x % ntiles) * a.tt;
  const int tt = static_cast<int>(a.t - t0 < a.tt ? a.t - t0 : a.tt);
  float* sc = smem;
  float* ss = smem + a.tt * half;
  fill_phase(a, bi, t0, tt, half, sc, ss);
  __syncthreads();
  const int items = static_cast<int>(a.h) * tt * half;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int p = it % half;
    const int rest = it / half;
    const int tl = rest % tt;
    const int64_t hi = rest / tt;
    const int64_t ti = t0 + tl;
    const float c = sc[tl * half + p];
    const float s = ss[tl * half + p];
    const int64_t qb = bi * a.qs[0] + hi * a.qs[1] + ti * a.qs[2] + 2 * p * a.qs[3];
    const int64_t kb = bi * a.ks[0] + hi * a.ks[1] + ti * a.ks[2] + 2 * p * a.ks[3];
    const int64_t vb = bi * ka.vs[0] + hi * ka.vs[1] + ti * ka.vs[2] + 2 * p * ka.vs[3];
    float q0, q1, k0, k1;
    rotate_pair(load_as_f32<DT>(a.q, qb), load_as_f32<DT>(a.q, qb + a.qs[3]), c, s, q0, q1);
    rotate_pair(load_as_f32<DT>(a.k, kb), load_as_f32<DT>(a.k, kb + a.ks[3]), c, s, k0, k1);
    const int64_t o = ((bi * a.h + hi) * a.t + ti) * a.d + 2 * p;
    store_from_f32<DT>(a.oq, o, q0);
    store_from_f32<DT>(a.oq, o + 1, q1);
    const int64_t slot = ka.slots[bi * a.t + ti];
    if (slot < 0 || slot >= ka.cache_slots) {
      record_device_error(MOSS_ERR_VALUE);
      continue;
    }
    const int64_t co = ((bi * a.h + hi) * ka.cache_slots + slot) * a.d + 2 * p;
    store_from_f32<DT>(ka.k_cache, co, k0);
    store_from_f32<DT>(ka.k_cache, co + 1, k1);
    store_from_f32<DT>(ka.v_cache, co, load_as_f32<DT>(ka.v, vb));
    store_from_f32<DT>(ka.v_cache, co + 1, load_as_f32<DT>(ka.v, vb + ka.vs[3]));
  }
}

// Streaming path for q and k whose rows are contiguous within each head
// (innermost stride 1, time stride d): one CTA per SM.  A producer thread
// streams tiles (one batch index, TT time steps, all heads) of q and k into
// a ring of shared-memory stages with one bulk copy per head and tensor; the
// consumer warps evaluate the tile's (c, s) table (double-buffered), rotate
// from shared memory and store the outputs straight to global memory.
namespace rstream {
#ifndef MOSS_ROPE_CONSUMERS
#define MOSS_ROPE_CONSUMERS 512
#endif
constexpr int kConsumers = MOSS_ROPE_CONSUMERS;
constexpr int kThreads = kConsumers + 32;
#ifndef MOSS_ROPE_STAGES
#define MOSS_ROPE_STAGES 3
#endif
#ifndef MOSS_ROPE_STAGE_BYTES
#define MOSS_ROPE_STAGE_BYTES 49152
#endif
constexpr int kStages = MOSS_ROPE_STAGES;
constexpr int kStageBytes = MOSS_ROPE_STAGE_BYTES;
#ifndef MOSS_ROPE_MAX_PAIRS
#define MOSS_ROPE_MAX_PAIRS 2048
#endif
constexpr int kMaxPairs = MOSS_ROPE_MAX_PAIRS;  // (c, s) pairs per tile table
// Items (16 bytes of q and 16 of k) per consumer thread and tile.
constexpr int kSlots = (kStageBytes / 32 + kConsumers - 1) / kConsumers;

struct Args {
  RopeArgs r;
  uint32_t ntiles;
  FastDiv tiles_per_b;  // time tiles per batch index
  FastDiv nvec;         // 16-byte items per row (d / VW)
  FastDiv tt;           // time steps per tile
  FastDiv half;         // d / 2
  uint32_t fpad;        // floats reserved for freq (d/2 rounded up to 4)
};

inline size_t smem_bytes(int tt, int half, bool tables) {
  size_t b = static_cast<size_t>(kStages) * kStageBytes;
  if (!tables) b += sizeof(float) * (((half + 3) & ~3) + 4 * static_cast<size_t>(tt) * half);
  return b + (2 * kStages + 2) * 8;
}
}  // namespace rstream

template <int DT, bool TABLES>
__global__ void __launch_bounds__(rstream::kThreads, 1) rope_stream_kernel(const rstream::Args sa) {
  using namespace rstream;
  constexpr int VW = DT == MOSS_BF16 ? 8 : 4;
  constexpr int kEs = DT == MOSS_BF16 ? 2 : 4;
  const RopeArgs& a = sa.r;
  extern __shared__ __align__(128) unsigned char sbuf[];
  const int half = static_cast<int>(sa.half.d);
  const int tt_full = static_cast<int>(sa.tt.d);
  const int tbl = tt_full * half;
  float* freq = reinterpret_cast<float*>(sbuf + kStages * kStageBytes);
  float* tabs = freq + sa.fpad;
  unsigned long long* full = reinterpret_cast<unsigned long long*>(
      sbuf + kStages * kStageBytes + (TABLES ? 0 : sizeof(float) * (sa.fpad + 4 * tbl)));
  unsigned long long* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2 * kStages);
  const int tid = threadIdx.x;
  const uint32_t head_bytes = static_cast<uint32_t>(tt_full * a.d * kEs);  // per head in a stage
  const uint32_t k_off = static_cast<uint32_t>(a.h) * head_bytes;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      pipe::mbar_init(&full[s], 1);
      pipe::mbar_init(&empty[s], kConsumers / 32);
    }
    *abort_flag = 0;
    pipe::fence_mbar_init();
  }
  if constexpr (!TABLES) {
    for (int j = tid; j < half; j += blockDim.x) freq[j] = expf(__fmul_rn(static_cast<float>(j), a.coef));
  }
  __syncthreads();

  if (tid >= kConsumers) {  // producer warp: one thread issues every copy
    if (tid != kConsumers) return;
    uint32_t i = 0;
    for (uint32_t tile = blockIdx.x; tile < sa.ntiles; tile += gridDim.x, ++i) {
      const int s = static_cast<int>(i % kStages);
      if (i >= kStages && !pipe::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      const uint32_t bi = fast_div(tile, sa.tiles_per_b);
      const int64_t t0 = static_cast<int64_t>(tile - bi * sa.tiles_per_b.d) * tt_full;
      const int ttc = static_cast<int>(a.t - t0 < tt_full ? a.t - t0 : tt_full);
      const uint32_t run = static_cast<uint32_t>(ttc * a.d * kEs);
      pipe::mbar_arrive_expect_tx(&full[s], 2u * static_cast<uint32_t>(a.h) * run);
      unsigned char* st = sbuf + s * kStageBytes;
      const char* q = static_cast<const char*>(a.q) + (bi * a.qs[0] + t0 * a.qs[2]) * kEs;
      const char* k = static_cast<const char*>(a.k) + (bi * a.ks[0] + t0 * a.ks[2]) * kEs;
      for (int64_t hi = 0; hi < a.h; ++hi) {
        pipe::bulk_g2s(st + hi * head_bytes, q + hi * a.qs[1] * kEs, run, &full[s]);
        pipe::bulk_g2s(st + k_off + hi * head_bytes, k + hi * a.ks[1] * kEs, run, &full[s]);
      }
    }
    // Drain: the copies of the last issued tiles must land before exit.
    for (uint32_t j = i > kStages ? i - kStages : 0; j < i; ++j)
      pipe::mbar_wait(&full[j % kStages], (j / kStages) & 1);
    return;
  }

  // Consumer warps.  Every consumer runs the same tiles and barriers; after
  // a timeout (anywhere) the remaining tiles are skipped.  A thread's items
  // sit at the same place in every tile, so their offsets are computed once.
  const int lane = tid & 31;
  const uint32_t items_full = static_cast<uint32_t>(a.h) * tt_full * sa.nvec.d;
  uint32_t so[kSlots];   // byte offset of the q item in a stage
  int tlv[kSlots];       // time step within the tile (large: no item)
  int toff[kSlots];      // first (c, s) pair of the item in the tile table
  int64_t orel[kSlots];  // output element offset from the tile's base
#pragma unroll
  for (int m = 0; m < kSlots; ++m) {
    const uint32_t it = tid + m * kConsumers;
    so[m] = 0;
    toff[m] = 0;
    orel[m] = 0;
    tlv[m] = 0x3fffffff;
    if (it < items_full) {
      const uint32_t rest = fast_div(it, sa.nvec);
      const uint32_t vec = it - rest * sa.nvec.d;
      const uint32_t hi = fast_div(rest, sa.tt);
      const int tl = static_cast<int>(rest - hi * sa.tt.d);
      so[m] = hi * head_bytes + static_cast<uint32_t>((tl * a.d + vec * VW) * kEs);
      tlv[m] = tl;
      toff[m] = tl * half + static_cast<int>(vec) * (VW / 2);
      orel[m] = (static_cast<int64_t>(hi) * a.t + tl) * a.d + vec * VW;
    }
  }
  bool alive = true;
  uint32_t i = 0;
  for (uint32_t tile = blockIdx.x; tile < sa.ntiles; tile += gridDim.x, ++i) {
    const int s = static_cast<int>(i % kStages);
    const uint32_t bi = fast_div(tile, sa.tiles_per_b);
    const int64_t t0 = static_cast<int64_t>(tile - bi * sa.tiles_per_b.d) * tt_full;
    const int ttc = static_cast<int>(a.t - t0 < tt_full ? a.t - t0 : tt_full);
    float* sc = tabs + (i & 1) * 2 * tbl;
    float* ss = sc + tbl;
    if (alive && *abort_flag) alive = false;
    if constexpr (!TABLES) {
      if (alive) {
        const float off = offset_as_float(a.offset, a.offset_dtype, bi);
        for (int e = tid; e < ttc * half; e += kConsumers) {
          const int tl = static_cast<int>(fast_div(static_cast<uint32_t>(e), sa.half));
          const int j = e - tl * half;
          const float ts = __fadd_rn(off, static_cast<float>(t0 + tl));
          const float phase = __fmul_rn(freq[j], ts);
          sc[e] = cosf(phase);
          ss[e] = sinf(phase);
        }
      }
      pipe::consumer_sync(kConsumers);
    }
    if (alive && !pipe::mbar_wait(&full[s], (i / kStages) & 1)) {
      alive = false;
      *abort_flag = 1;
    }
    if (alive) {
      const unsigned char* st = sbuf + s * kStageBytes;
      const int64_t ob = (static_cast<int64_t>(bi) * a.h * a.t + t0) * a.d;
      const int64_t tb = (static_cast<int64_t>(bi) * a.t + t0) * half;
#pragma unroll
      for (int m = 0; m < kSlots; ++m) {
        if (tlv[m] >= ttc) continue;
        const uint4 qraw = *reinterpret_cast<const uint4*>(st + so[m]);
        const uint4 kraw = *reinterpret_cast<const uint4*>(st + k_off + so[m]);
        float c[VW / 2], sn[VW / 2];
        if constexpr (TABLES) {
#pragma unroll
          for (int p = 0; p < VW / 2; ++p) {
            c[p] = a.cos_t[tb + toff[m] + p];
            sn[p] = a.sin_t[tb + toff[m] + p];
          }
        } else {
#pragma unroll
          for (int p = 0; p < VW / 2; ++p) {
            c[p] = sc[toff[m] + p];
            sn[p] = ss[toff[m] + p];
          }
        }
        float qv[VW], kv[VW], qo[VW], ko[VW];
        if constexpr (DT == MOSS_BF16) {
          unpack_bf16x8(qraw, qv);
          unpack_bf16x8(kraw, kv);
        } else {
          qv[0] = __uint_as_float(qraw.x); qv[1] = __uint_as_float(qraw.y);
          qv[2] = __uint_as_float(qraw.z); qv[3] = __uint_as_float(qraw.w);
          kv[0] = __uint_as_float(kraw.x); kv[1] = __uint_as_float(kraw.y);
          kv[2] = __uint_as_float(kraw.z); kv[3] = __uint_as_float(kraw.w);
        }
#pragma unroll
        for (int p = 0; p < VW / 2; ++p) {
          rotate_pair(qv[2 * p], qv[2 * p + 1], c[p], sn[p], qo[2 * p], qo[2 * p + 1]);
          rotate_pair(kv[2 * p], kv[2 * p + 1], c[p], sn[p], ko[2 * p], ko[2 * p + 1]);
        }
        const int64_t o = ob + orel[m];
        if constexpr (DT == MOSS_BF16) {
          *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.oq) + o) = pack_bf16x8(qo);
          *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.ok) + o) = pack_bf16x8(ko);
        } else {
          *reinterpret_cast<float4*>(static_cast<float*>(a.oq) + o) = make_float4(qo[0], qo[1], qo[2], qo[3]);
          *reinterpret_cast<float4*>(static_cast<float*>(a.ok) + o) = make_float4(ko[0], ko[1], ko[2], ko[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0 && alive) pipe::mbar_arrive(&empty[s]);
  }
}

// Launches the streaming path when the layout allows it; false otherwise.
static bool rope_stream(RopeArgs a, int dtype, bool tables, cudaStream_t s) {
  using namespace rstream;
  const int esize = dtype == MOSS_F32 ? 4 : 2;
  const int half = static_cast<int>(a.d / 2);
  if (a.qs[2] != a.d || a.ks[2] != a.d) return false;
  const int64_t per_t = 2 * a.h * a.d * esize;  // stage bytes per time step
  int64_t tt = kStageBytes / per_t;
  if (!tables && tt * half > kMaxPairs) tt = kMaxPairs / half;
  if (tt > a.t) tt = a.t;
  if (tt < 1) return false;
  const int64_t tiles_per_b = (a.t + tt - 1) / tt;
  const int64_t ntiles = a.b * tiles_per_b;
  if (ntiles > 0x7fffffffLL || a.h * tt * (a.d / (16 / esize)) > 0x7fffffffLL) return false;
  Args sa{};
  a.tt = static_cast<int>(tt);
  sa.r = a;
  sa.ntiles = static_cast<uint32_t>(ntiles);
  sa.tiles_per_b = make_fastdiv(static_cast<uint32_t>(tiles_per_b));
  sa.nvec = make_fastdiv(static_cast<uint32_t>(a.d / (16 / esize)));
  sa.tt = make_fastdiv(static_cast<uint32_t>(tt));
  sa.half = make_fastdiv(static_cast<uint32_t>(half));
  sa.fpad = static_cast<uint32_t>((half + 3) & ~3);
  const size_t shmem = smem_bytes(static_cast<int>(tt), half, tables);
  const uint32_t grid = sa.ntiles < static_cast<uint32_t>(sm_count()) ? sa.ntiles
                                                                      : static_cast<uint32_t>(sm_count());
  const size_t smax = smem_bytes(kMaxPairs, 1, false) + 1024 * sizeof(float);
#define MOSS_ROPE_S(DT, TB)                                                    \
  do {                                                                         \
    static bool attr_done[kMaxDevices] = {};                                   \
    allow_dynamic_smem(rope_stream_kernel<DT, TB>, smax, attr_done);           \
    rope_stream_kernel<DT, TB><<<grid, kThreads, shmem, s>>>(sa);              \
  } while (0)
  if (dtype == MOSS_BF16) {
    if (tables) MOSS_ROPE_S(MOSS_BF16, true);
    else MOSS_ROPE_S(MOSS_BF16, false);
  } else {
    if (tables) MOSS_ROPE_S(MOSS_F32, true);
    else MOSS_ROPE_S(MOSS_F32, false);
  }
#undef MOSS_ROPE_S
  return true;
}

static int rope_common(const char* name, RopeArgs a, int dtype, bool tables, void* stream) {
  if (a.b < 0 || a.h < 0 || a.t < 0 || a.d < 2 || (a.d & 1))
    return fail(MOSS_ERR_VALUE, "%s: expected equal B,H,T,even-D rotary inputs", name);
  if (dtype != MOSS_F32 && dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: q/k dtype must be float32 or bfloat16", name);
  if (a.d > 1024) return fail(MOSS_ERR_UNSUPPORTED, "%s: head dim above 1024", name);
  if (a.h > 65536) return fail(MOSS_ERR_UNSUPPORTED, "%s: more than 65536 heads", name);
  const int64_t n = a.b * a.h * a.t;
  if (n == 0) return MOSS_OK;
  if (!a.q || !a.k || !a.oq || !a.ok) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (tables && (!a.cos_t || !a.sin_t)) return fail(MOSS_ERR_VALUE, "%s: null table", name);
  if (!tables && !a.offset) return fail(MOSS_ERR_VALUE, "%s: null offset", name);
  if (!tables && (a.offset_dtype < 0 || a.offset_dtype > 2))
    return fail(MOSS_ERR_VALUE, "%s: offset dtype must be int64, int32 or float32", name);
  const int half = static_cast<int>(a.d / 2);
  const int esize = dtype == MOSS_F32 ? 4 : 2;
  const int vw = dtype == MOSS_F32 ? 4 : 8;
  bool vec = (a.d % vw == 0) && a.qs[3] == 1 && a.ks[3] == 1 && aligned16(a.q) && aligned16(a.k) &&
             aligned16(a.oq) && aligned16(a.ok);
  for (int i = 0; i < 3 && vec; ++i) {
    if ((a.qs[i] * esize) % 16 != 0 || (a.ks[i] * esize) % 16 != 0) vec = false;
  }
  cudaStream_t s = as_stream(stream);
  if (vec && rope_stream(a, dtype, tables, s)) return launch_status(name);
  if (vec) {
    // Tiles of tt time steps with at most 256 * KI items (KI items per
    // thread); KI = kRopeItems, or 4 when one time step alone has more.
    const int64_t per_t = a.h * (a.d / vw);
    const int ki = per_t <= 256 * kRopeItems ? kRopeItems : 4;
    int tt = static_cast<int>(256 * ki / per_t);
    if (tt < 1) vec = false;
    if (vec) {
      if (tt > a.t) tt = static_cast<int>(a.t);
      a.tt = tt;
      const int64_t ntiles = a.b * ((a.t + tt - 1) / tt);
      if (ntiles > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too many tiles", name);
      const size_t shmem = tables ? 0 : sizeof(float) * (((half + 3) & ~3) + 4 * tt * half);
      // Persistent grid: as many blocks as fit on the device at once.
#define MOSS_ROPE_V(DT, TB, KI)                                                               \
  do {                                                                                        \
    const int64_t grid = persistent_grid(rope_vec_kernel<DT, TB, KI>, 256, shmem, ntiles);         \
    rope_vec_kernel<DT, TB, KI><<<static_cast<unsigned>(grid), 256, shmem, s>>>(a, static_cast<uint32_t>(ntiles));   \
  } while (0)
      if (dtype == MOSS_BF16) {
        if (tables) { if (ki == kRopeItems) MOSS_ROPE_V(MOSS_BF16, true, kRopeItems); else MOSS_ROPE_V(MOSS_BF16, true, 4); }
        else { if (ki == kRopeItems) MOSS_ROPE_V(MOSS_BF16, false, kRopeItems); else MOSS_ROPE_V(MOSS_BF16, false, 4); }
      } else {
        if (tables) { if (ki == kRopeItems) MOSS_ROPE_V(MOSS_F32, true, kRopeItems); else MOSS_ROPE_V(MOSS_F32, true, 4); }
        else { if (ki == kRopeItems) MOSS_ROPE_V(MOSS_F32, false, kRopeItems); else MOSS_ROPE_V(MOSS_F32, false, 4); }
      }
#undef MOSS_ROPE_V
      return launch_status(name);
    }
  }
  // Generic path: 256 (c, s) pairs per tile.
  int tt = 256 / half;
  if (tt < 1) tt = 1;
  if (tt > a.t) tt = static_cast<int>(a.t);
  a.tt = tt;
  const int64_t ntiles = (a.t + tt - 1) / tt;
  if (a.b * ntiles > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: grid too large", name);
  if (a.h * tt * half > 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too many heads for one CTA tile", name);
  const unsigned grid = static_cast<unsigned>(a.b * ntiles);
  const size_t shmem = tables ? 0 : sizeof(float) * 2 * tt * half;
#define MOSS_ROPE(KERNEL, DT, TB) KERNEL<DT, TB><<<grid, 256, shmem, s>>>(a)
  if (dtype == MOSS_BF16) {
    if (tables) MOSS_ROPE(rope_pair_kernel, MOSS_BF16, true);
    else MOSS_ROPE(rope_pair_kernel, MOSS_BF16, false);
  } else {
    if (tables) MOSS_ROPE(rope_pair_kernel, MOSS_F32, true);
    else MOSS_ROPE(rope_pair_kernel, MOSS_F32, false);
  }
#undef MOSS_ROPE
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

extern "C" int moss_rope_kv(const void* q, const void* k, const void* v, int dtype,
                            const void* offset, int offset_dtype, float freq_coef,
                            const int64_t* slots, void* oq, void* k_cache, void* v_cache,
                            int64_t b, int64_t h, int64_t t, int64_t d, int64_t cache_slots,
                            const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, void* stream) {
  const char* name = "moss_rope_kv";
  if (!q_strides || !k_strides || !v_strides) return fail(MOSS_ERR_VALUE, "%s: null strides", name);
  if (b < 0 || h < 0 || t < 0 || d < 2 || (d & 1) || cache_slots < 1)
    return fail(MOSS_ERR_VALUE, "%s: expected equal B,H,T,even-D inputs and a non-empty ring", name);
  if (dtype != MOSS_F32 && dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: q/k/v dtype must be float32 or bfloat16", name);
  if (offset_dtype < 0 || offset_dtype > 2)
    return fail(MOSS_ERR_VALUE, "%s: offset dtype must be int64, int32 or float32", name);
  if (d > 1024) return fail(MOSS_ERR_UNSUPPORTED, "%s: head dim above 1024", name);
  if (b * h * t == 0) return MOSS_OK;
  if (!q || !k || !v || !offset || !slots || !oq || !k_cache || !v_cache)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  RopeKvArgs ka{};
  RopeArgs& a = ka.r;
  a.q = q; a.k = k; a.offset = offset; a.offset_dtype = offset_dtype; a.coef = freq_coef;
  a.oq = oq; a.ok = nullptr;
  a.b = b; a.h = h; a.t = t; a.d = d;
  for (int i = 0; i < 4; ++i) {
    a.qs[i] = q_strides[i];
    a.ks[i] = k_strides[i];
    ka.vs[i] = v_strides[i];
  }
  ka.v = v; ka.slots = slots; ka.k_cache = k_cache; ka.v_cache = v_cache;
  ka.cache_slots = cache_slots;
  const int half = static_cast<int>(d / 2);
  int tt = 256 / half;
  if (tt < 1) tt = 1;
  if (tt > t) tt = static_cast<int>(t);
  a.tt = tt;
  const int64_t ntiles = (t + tt - 1) / tt;
  if (b * ntiles > 0x7fffffffLL || h * tt * half > 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: grid too large", name);
  const unsigned grid = static_cast<unsigned>(b * ntiles);
  const size_t shmem = sizeof(float) * 2 * tt * half;
  cudaStream_t s = as_stream(stream);
  if (dtype == MOSS_BF16) rope_kv_kernel<MOSS_BF16><<<grid, 256, shmem, s>>>(ka);
  else rope_kv_kernel<MOSS_F32><<<grid, 256, shmem, s>>>(ka);
  return launch_status(name);
}
