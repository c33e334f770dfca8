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
// Work decomposition: the phase does not depend on the head, so each
// kernel evaluates a time step's d/2 (c, s) pairs once into shared memory
// and rotates every head's row of that step with them.
//   * rope_stream_kernel, for q and k whose time rows are contiguous within
//     each head: one CTA per SM takes an even share of the b*t rows (in
//     chunks whose phase table it evaluates once); a tile is a group of
//     heads over a chunk, staged by one bulk copy per head, tensor and
//     batch run (a producer warp), rotated by 16 consumer warps that write
//     16-byte vectors straight to global memory;
//   * rope_vec_kernel, for other layouts with 16-byte rows (innermost
//     stride 1, e.g. a qkv projection output viewed as [b,h,t,d]): a tile
//     is one batch index and TT time steps for all heads; persistent blocks
//     issue the next tile's loads and phase table before rotating the
//     current one;
//   * rope_pair_kernel, one interleaved pair per item, for any strides.
#include "pipeline.cuh"
#include "rotary.cuh"

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

// Vector form of rope_kv_kernel for rows that are 16-byte vectors (innermost
// stride 1, aligned): one thread per 16-byte item of q, k and v (one batch
// index, head, time step and VW elements), its VW/2 (c, s) pairs evaluated
// by the thread with fill_phase's arithmetic.  Enough threads to fill the
// device at a few tokens per batch index, where the tile kernel above has
// one CTA per batch index.
template <int DT>
__global__ void __launch_bounds__(256) rope_kv_vec_kernel(RopeKvArgs ka, int64_t items) {
  constexpr int VW = DT == MOSS_BF16 ? 8 : 4;
  constexpr int kEs = DT == MOSS_BF16 ? 2 : 4;
  const RopeArgs& a = ka.r;
  const int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (it >= items) return;
  const int64_t nvec = a.d / VW;
  const int64_t vec = it % nvec;
  int64_t rest = it / nvec;
  const int64_t ti = rest % a.t;
  rest /= a.t;
  const int64_t hi = rest % a.h;
  const int64_t bi = rest / a.h;
  const int64_t slot = ka.slots[bi * a.t + ti];
  const char* qp = static_cast<const char*>(a.q) + (bi * a.qs[0] + hi * a.qs[1] + ti * a.qs[2] + vec * VW) * kEs;
  const char* kp = static_cast<const char*>(a.k) + (bi * a.ks[0] + hi * a.ks[1] + ti * a.ks[2] + vec * VW) * kEs;
  const char* vp = static_cast<const char*>(ka.v) + (bi * ka.vs[0] + hi * ka.vs[1] + ti * ka.vs[2] + vec * VW) * kEs;
  const uint4 qraw = *reinterpret_cast<const uint4*>(qp);
  const uint4 kraw = *reinterpret_cast<const uint4*>(kp);
  const uint4 vraw = *reinterpret_cast<const uint4*>(vp);
  const float off = offset_as_float(a.offset, a.offset_dtype, bi);
  const float ts = __fadd_rn(off, static_cast<float>(ti));
  float c[VW / 2], sn[VW / 2];
#pragma unroll
  for (int p = 0; p < VW / 2; ++p) {
    const int j = static_cast<int>(vec) * (VW / 2) + p;
    const float freq = expf(__fmul_rn(static_cast<float>(j), a.coef));
    const float phase = __fmul_rn(freq, ts);
    c[p] = cosf(phase);
    sn[p] = sinf(phase);
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
  const int64_t o = ((bi * a.h + hi) * a.t + ti) * a.d + vec * VW;
  uint4 qw, kw;
  if constexpr (DT == MOSS_BF16) {
    qw = pack_bf16x8(qo);
    kw = pack_bf16x8(ko);
  } else {
    qw = make_uint4(__float_as_uint(qo[0]), __float_as_uint(qo[1]), __float_as_uint(qo[2]), __float_as_uint(qo[3]));
    kw = make_uint4(__float_as_uint(ko[0]), __float_as_uint(ko[1]), __float_as_uint(ko[2]), __float_as_uint(ko[3]));
  }
  *reinterpret_cast<uint4*>(static_cast<char*>(a.oq) + o * kEs) = qw;
  if (slot < 0 || slot >= ka.cache_slots) {
    record_device_error(MOSS_ERR_VALUE);
    return;
  }
  const int64_t co = ((bi * a.h + hi) * ka.cache_slots + slot) * a.d + vec * VW;
  *reinterpret_cast<uint4*>(static_cast<char*>(ka.k_cache) + co * kEs) = kw;
  *reinterpret_cast<uint4*>(static_cast<char*>(ka.v_cache) + co * kEs) = vraw;
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
#define MOSS_ROPE_STAGES 6
#endif
#ifndef MOSS_ROPE_STAGE_BYTES
#define MOSS_ROPE_STAGE_BYTES 32768
#endif
constexpr int kStages = MOSS_ROPE_STAGES;
constexpr int kStageBytes = MOSS_ROPE_STAGE_BYTES;
// Most (c, s) pairs of a chunk's phase table: a CTA's rows are walked in
// chunks whose table is evaluated once, behind one barrier, for all heads.
constexpr int kWindowPairs = 4096;
// Items (16 bytes of q and 16 of k) per consumer thread and tile.
constexpr int kSlots = (kStageBytes / 32 + kConsumers - 1) / kConsumers;

struct Args {
  RopeArgs r;
  uint32_t rows;            // b * t flattened (batch-major) time rows
  FastDiv t;                // time steps per batch index
  FastDiv nvec;             // 16-byte items per row (d / VW)
  FastDiv crow;             // rows per chunk (a tile's rows; the phase window)
  uint32_t heads_per_tile;  // heads of a tile
  FastDiv half;             // d / 2
  uint32_t fpad;            // floats reserved for freq (d/2 rounded up to 4)
};

inline size_t smem_bytes(int chunk_rows, int half, bool tables) {
  size_t b = static_cast<size_t>(kStages) * kStageBytes;
  if (!tables) b += sizeof(float) * (((half + 3) & ~3) + 2 * static_cast<size_t>(chunk_rows) * half);
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
  const uint32_t R = sa.crow.d;             // rows per chunk
  const uint32_t G = sa.heads_per_tile;     // heads per tile
  const uint32_t H = static_cast<uint32_t>(a.h);
  const uint32_t T = sa.t.d;
  const uint32_t win_pairs = R * sa.half.d;
  float* freq = reinterpret_cast<float*>(sbuf + kStages * kStageBytes);
  float* tab_c = freq + sa.fpad;  // [R][half] cosines of the chunk's rows, then sines
  float* tab_s = tab_c + win_pairs;
  unsigned long long* full = reinterpret_cast<unsigned long long*>(
      sbuf + kStages * kStageBytes + (TABLES ? 0 : sizeof(float) * (sa.fpad + 2 * win_pairs)));
  unsigned long long* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2 * kStages);
  const int tid = threadIdx.x;
  const uint32_t row_bytes = static_cast<uint32_t>(a.d * kEs);
  const uint32_t slab = R * row_bytes;  // one head's chunk rows in a stage
  const uint32_t k_off = G * slab;      // k slabs follow the q slabs
  // This CTA's rows: an even share of the b * t rows, in order.
  const uint32_t lo = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * sa.rows / gridDim.x);
  const uint32_t hi = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * sa.rows / gridDim.x);
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

  // Tiles, in the same order on both sides: for each chunk of R rows, the
  // heads in groups of G; a tile is q and k of its heads over the chunk.
  if (tid >= kConsumers) {  // producer warp: lane j copies heads j, j+32, ... of a tile
    const int pl = tid - kConsumers;
    uint32_t i = 0;
    bool stop = false;
    for (uint32_t c0 = lo; c0 < hi && !stop; c0 += R) {
      const uint32_t nr = hi - c0 < R ? hi - c0 : R;
      for (uint32_t h0 = 0; h0 < H; h0 += G, ++i) {
        const uint32_t ng = H - h0 < G ? H - h0 : G;
        const int s = static_cast<int>(i % kStages);
        int go = 1;
        if (pl == 0) {
          if (i >= kStages && !pipe::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) *abort_flag = 1;
          go = !*abort_flag;
        }
        if (!__shfl_sync(0xffffffffu, go, 0)) {
          stop = true;
          break;
        }
        if (pl == 0) pipe::mbar_arrive_expect_tx(&full[s], 2u * ng * nr * row_bytes);
        __syncwarp();
        unsigned char* st = sbuf + s * kStageBytes;
        for (uint32_t g = pl; g < ng; g += 32) {
          const int64_t hh = h0 + g;
          for (uint32_t r0 = 0; r0 < nr;) {  // runs of rows, cut at batch boundaries
            const uint32_t row = c0 + r0;
            const uint32_t bi = fast_div(row, sa.t);
            const uint32_t t0 = row - bi * T;
            const uint32_t n = T - t0 < nr - r0 ? T - t0 : nr - r0;
            const char* q = static_cast<const char*>(a.q) + (bi * a.qs[0] + hh * a.qs[1] + t0 * a.qs[2]) * kEs;
            const char* k = static_cast<const char*>(a.k) + (bi * a.ks[0] + hh * a.ks[1] + t0 * a.ks[2]) * kEs;
            pipe::bulk_g2s(st + g * slab + r0 * row_bytes, q, n * row_bytes, &full[s]);
            pipe::bulk_g2s(st + k_off + g * slab + r0 * row_bytes, k, n * row_bytes, &full[s]);
            r0 += n;
          }
        }
      }
    }
    // Drain: the copies of the last issued tiles must land before exit.
    if (pl == 0) {
      for (uint32_t j = i > kStages ? i - kStages : 0; j < i; ++j)
        pipe::mbar_wait(&full[j % kStages], (j / kStages) & 1);
    }
    __syncwarp();
    return;
  }

  // Consumer warps.  Every consumer runs the same tiles and barriers; after
  // a timeout (anywhere) the remaining tiles are skipped.  A thread's items
  // (head g of the tile, row r of the chunk, 16-byte vector) sit at the same
  // place in every tile.
  const int lane = tid & 31;
  const uint32_t items_full = G * R * sa.nvec.d;
  uint32_t so[kSlots];   // byte offset of the q item in a stage
  uint32_t rv[kSlots];   // row within the chunk
  uint32_t gv[kSlots];   // head within the tile (large: no item)
  uint32_t vo[kSlots];   // element offset of the vector within the row
#pragma unroll
  for (int m = 0; m < kSlots; ++m) {
    const uint32_t it = tid + m * kConsumers;
    const uint32_t rest = fast_div(it, sa.nvec);
    const uint32_t vec = it - rest * sa.nvec.d;
    const uint32_t g = fast_div(rest, sa.crow);
    rv[m] = rest - g * R;
    gv[m] = it < items_full ? g : 0x7fffffffu;
    vo[m] = vec * VW;
    so[m] = g * slab + rv[m] * row_bytes + vec * VW * kEs;
  }
  bool alive = true;
  uint32_t i = 0;
  for (uint32_t c0 = lo; c0 < hi; c0 += R) {
    const uint32_t nr = hi - c0 < R ? hi - c0 : R;
    if (alive && *abort_flag) alive = false;
    if constexpr (!TABLES) {  // the chunk's (c, s) pairs; the same decision in every consumer
      if (c0 != lo) pipe::consumer_sync(kConsumers);  // all reads of the previous chunk done
      if (alive) {
        const uint32_t n = nr * sa.half.d;
        for (uint32_t e = tid; e < n; e += kConsumers) {
          const uint32_t r = fast_div(e, sa.half);
          const uint32_t j = e - r * sa.half.d;
          const uint32_t row = c0 + r;
          const uint32_t bi = fast_div(row, sa.t);
          const float off = offset_as_float(a.offset, a.offset_dtype, bi);
          const float ts = __fadd_rn(off, static_cast<float>(row - bi * T));
          const float phase = __fmul_rn(freq[j], ts);
          tab_c[e] = cosf(phase);
          tab_s[e] = sinf(phase);
        }
      }
      pipe::consumer_sync(kConsumers);
    }
    // Output element offset of each item without its head term, and its
    // first (c, s) pair (in the window, or in the given tables).
    int64_t ob[kSlots];
    int64_t tb[kSlots];
#pragma unroll
    for (int m = 0; m < kSlots; ++m) {
      const uint32_t row = c0 + rv[m];
      const uint32_t bi = fast_div(row, sa.t);
      ob[m] = (static_cast<int64_t>(bi) * H * T + (row - bi * T)) * a.d + vo[m];
      tb[m] = TABLES ? static_cast<int64_t>(row) * half + vo[m] / 2
                     : static_cast<int64_t>(rv[m]) * half + vo[m] / 2;
    }
    for (uint32_t h0 = 0; h0 < H; h0 += G, ++i) {
      const uint32_t ng = H - h0 < G ? H - h0 : G;
      const int s = static_cast<int>(i % kStages);
      if (alive && *abort_flag) alive = false;
      if (alive && !pipe::mbar_wait(&full[s], (i / kStages) & 1)) {
        alive = false;
        *abort_flag = 1;
      }
      if (alive) {
        const unsigned char* st = sbuf + s * kStageBytes;
#pragma unroll
        for (int m = 0; m < kSlots; ++m) {
          if (gv[m] >= ng || rv[m] >= nr) continue;
          const uint4 qraw = *reinterpret_cast<const uint4*>(st + so[m]);
          const uint4 kraw = *reinterpret_cast<const uint4*>(st + k_off + so[m]);
          float c[VW / 2], sn[VW / 2];
          if constexpr (TABLES) {
#pragma unroll
            for (int p = 0; p < VW / 2; ++p) {
              c[p] = a.cos_t[tb[m] + p];
              sn[p] = a.sin_t[tb[m] + p];
            }
          } else if constexpr (VW == 8) {  // 16-byte aligned: half is a multiple of 4
            const float4 cv = *reinterpret_cast<const float4*>(tab_c + tb[m]);
            const float4 sv = *reinterpret_cast<const float4*>(tab_s + tb[m]);
            c[0] = cv.x; c[1] = cv.y; c[2] = cv.z; c[3] = cv.w;
            sn[0] = sv.x; sn[1] = sv.y; sn[2] = sv.z; sn[3] = sv.w;
          } else {  // 8-byte aligned: half is even
            const float2 cv = *reinterpret_cast<const float2*>(tab_c + tb[m]);
            const float2 sv = *reinterpret_cast<const float2*>(tab_s + tb[m]);
            c[0] = cv.x; c[1] = cv.y;
            sn[0] = sv.x; sn[1] = sv.y;
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
          const int64_t o = ob[m] + static_cast<int64_t>(h0 + gv[m]) * T * a.d;
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
}

// Launches the streaming path when the layout allows it; false otherwise.
static bool rope_stream(RopeArgs a, int dtype, bool tables, cudaStream_t s) {
  using namespace rstream;
  const int esize = dtype == MOSS_F32 ? 4 : 2;
  const int half = static_cast<int>(a.d / 2);
  if (a.qs[2] != a.d || a.ks[2] != a.d) return false;
  const int64_t row_head = 2 * a.d * esize;  // q and k bytes of one head and row
  const int64_t rows = a.b * a.t;
  if (row_head > kStageBytes || rows > 0x7fffffffLL || a.h > 0x7fffffffLL) return false;
  // An even share of the rows per CTA, at least one stage of work each.
  int64_t grid = (rows * a.h * row_head + kStageBytes - 1) / kStageBytes;
  if (grid > sm_count()) grid = sm_count();
  if (grid > rows) grid = rows;
  const int64_t share = (rows + grid - 1) / grid;  // most rows of one CTA
  // Chunk rows R: the share in the fewest chunks with R * row_head within a
  // stage and R * d/2 within the phase window (fewer chunks = fewer, longer
  // bulk copies: one per head, tensor and batch run of a chunk).  Heads per
  // tile G: as many as fit a stage with R rows, in even groups.
  int64_t rmax = kStageBytes / row_head;
  if (rmax > kWindowPairs / half) rmax = kWindowPairs / half;
  const int64_t chunks = (share + rmax - 1) / rmax;
  const int64_t chunk_rows = (share + chunks - 1) / chunks;
  int64_t head_group = kStageBytes / (chunk_rows * row_head);
  if (head_group > a.h) head_group = a.h;
  const int64_t groups = (a.h + head_group - 1) / head_group;
  head_group = (a.h + groups - 1) / groups;
  Args sa{};
  sa.r = a;
  sa.rows = static_cast<uint32_t>(rows);
  sa.t = make_fastdiv(static_cast<uint32_t>(a.t));
  sa.nvec = make_fastdiv(static_cast<uint32_t>(a.d / (16 / esize)));
  sa.crow = make_fastdiv(static_cast<uint32_t>(chunk_rows));
  sa.heads_per_tile = static_cast<uint32_t>(head_group);
  sa.half = make_fastdiv(static_cast<uint32_t>(half));
  sa.fpad = static_cast<uint32_t>((half + 3) & ~3);
  const size_t shmem = smem_bytes(static_cast<int>(chunk_rows), half, tables);
  // largest request: d = 1024 (512 freq floats) and a full window
  const size_t smax = static_cast<size_t>(kStages) * kStageBytes +
                      sizeof(float) * (512 + 2 * static_cast<size_t>(kWindowPairs)) + (2 * kStages + 2) * 8;
#define MOSS_ROPE_S(DT, TB)                                                    \
  do {                                                                         \
    static bool attr_done[kMaxDevices] = {};                                   \
    allow_dynamic_smem(rope_stream_kernel<DT, TB>, smax, attr_done);           \
    rope_stream_kernel<DT, TB><<<static_cast<unsigned>(grid), kThreads, shmem, s>>>(sa); \
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
  cudaStream_t s = as_stream(stream);
  {
    const int esize = dtype == MOSS_F32 ? 4 : 2;
    const int vw = dtype == MOSS_F32 ? 4 : 8;
    bool vec = d % vw == 0 && q_strides[3] == 1 && k_strides[3] == 1 && v_strides[3] == 1 &&
               aligned16(q) && aligned16(k) && aligned16(v) && aligned16(oq) &&
               aligned16(k_cache) && aligned16(v_cache);
    for (int i = 0; i < 3 && vec; ++i)
      vec = (q_strides[i] * esize) % 16 == 0 && (k_strides[i] * esize) % 16 == 0 &&
            (v_strides[i] * esize) % 16 == 0;
    const int64_t items = b * h * t * (d / vw);
    if (vec && (items + 255) / 256 <= 0x7fffffffLL) {
      const unsigned grid = static_cast<unsigned>((items + 255) / 256);
      if (dtype == MOSS_BF16) rope_kv_vec_kernel<MOSS_BF16><<<grid, 256, 0, s>>>(ka, items);
      else rope_kv_vec_kernel<MOSS_F32><<<grid, 256, 0, s>>>(ka, items);
      return launch_status(name);
    }
  }
  int tt = 256 / half;
  if (tt < 1) tt = 1;
  if (tt > t) tt = static_cast<int>(t);
  a.tt = tt;
  const int64_t ntiles = (t + tt - 1) / tt;
  if (b * ntiles > 0x7fffffffLL || h * tt * half > 0x7fffffffLL)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: grid too large", name);
  const unsigned grid = static_cast<unsigned>(b * ntiles);
  const size_t shmem = sizeof(float) * 2 * tt * half;
  if (dtype == MOSS_BF16) rope_kv_kernel<MOSS_BF16><<<grid, 256, shmem, s>>>(ka);
  else rope_kv_kernel<MOSS_F32><<<grid, 256, shmem, s>>>(ka);
  return launch_status(name);
}
