// Fused qkv projection with the rotary embedding in its epilogue (sm_100a,
// tcgen05 bf16 MMA, FP32 accumulation in tensor memory).
//
//   y = x W^T + bias      x [M, K] bf16 (row m = b * T + t), W [3 H 64, K]
//                         bf16, one bf16 rounding of (accumulator + bias):
//                         the reference's cached bf16 Linear
//                         (fast_moss/v2_runtime.py:77-106)
//   q = y[:, 0 : 64H], k = y[:, 64H : 128H], v = y[:, 128H :], heads of 64
//   q and k rotated as the reference's rotary forward
//   (fast_moss/v2_runtime.py:209-224: freq_j = expf(j * coef), phase =
//   freq_j * (float(offset[b]) + t), cosf/sinf; rotation
//   fast_moss/v2_pointwise.py:8-47: float32, every product and sum rounded,
//   one bf16 rounding)
//   q -> oq [B, H, T, 64]; rotated k and v -> k_cache / v_cache
//   [B, H, S, 64] at slot slots[b, t]
//
// These are the bits of the Linear followed by moss_rope_kv whenever the
// two accumulations round to the same bf16 value; the summation order of
// the dot products is this kernel's (16-wide K steps of the tensor core in
// ascending K), not cuBLAS's.
//
// The projection is skinny (a streaming chunk has 4 tokens per stream) and
// bound by the weight read, so the grid is wide: a CTA computes 32 token
// rows x 32 output features (half a head of q, k or v) over the whole K
// (at most 1536), with all of its operands resident in shared memory.
//   warps 0-3  issue the CTA's loads at once as 16-byte cp.async requests
//              (40 per thread on the benchmark shape, all in flight: one
//              round trip; bulk copies from DRAM arrived one after another
//              here): the weight blocks (pre-packed 4 KB blocks of 32 rows x
//              64 columns in the MMA's no-swizzle K-major core-matrix order,
//              so the copy is contiguous), the token rows in the same layout
//              (4 KB per 64-wide chunk), the tile's bias and its rows' ring
//              slots; they evaluate the rows' (c, s) table while the loads
//              fly; then warp 0 is the epilogue, one row per thread (TMEM
//              lane = row), with no global load left;
//   warp 4     allocates 32 TMEM columns and issues 4 MMAs per chunk
//              (kind::f16, bf16 operands, M=128, N=32, K=16).  The MMA reads
//              128 operand rows; rows 32-127 fall on the next chunks' bytes
//              (in bounds: 12 KB of slack follow the last chunk) and land in
//              TMEM lanes that are never read.
// Every wait is bounded (~2 s) and records MOSS_ERR_TIMEOUT; a ring slot
// out of range records MOSS_ERR_VALUE and that row's k/v store is skipped.
#include "rotary.cuh"
#include "tcgen05.cuh"

namespace moss {
namespace qkvr {

constexpr int kRows = 32;      // token rows per CTA
constexpr int kMmaRows = 128;  // MMA M (TMEM lanes)
constexpr int kCols = 32;      // output features per CTA: half a head
constexpr int kChunk = 64;     // K per MMA group (128 bytes of bf16 per row)
constexpr int kMaxChunks = 24;  // K <= 1536
constexpr uint32_t kAChunk = kRows * kChunk * 2;               // 4 KB of token rows per chunk
constexpr uint32_t kASlack = (kMmaRows - kRows) * kChunk * 2;  // rows 32-127 of the last chunk
constexpr uint32_t kBBytes = kCols * kChunk * 2;               // 4 KB weight block
// Loader warps: 4.  With 8 or 12 the one-stream launch takes the same time
// (8.9-9.0 us on B200): what limits a CTA is its SM's rate of outstanding
// global loads, not the number of warps issuing them.
#ifndef MOSS_QKV_LOADER_WARPS
#define MOSS_QKV_LOADER_WARPS 4
#endif
constexpr int kLoaderWarps = MOSS_QKV_LOADER_WARPS;
constexpr int kLoaderThreads = kLoaderWarps * 32;
constexpr int kThreads = kLoaderThreads + 32;  // loader warps (warp 0 also the epilogue), then MMA
constexpr uint32_t kTmemCols = 32;

// Shared-memory layout (offsets from a 128-byte aligned base).
struct Layout {
  uint32_t a, b, tab, bias, slots, freq, tmem, a_full, acc, total;
};
__host__ __device__ inline Layout layout(int chunks) {
  Layout l;
  l.a = 0;
  l.b = static_cast<uint32_t>(chunks) * kAChunk + kASlack;
  l.tab = l.b + static_cast<uint32_t>(chunks) * kBBytes;
  l.bias = l.tab + kRows * (kCols / 2) * 4u * 2u;
  l.slots = l.bias + kCols * 2u;
  l.freq = l.slots + kRows * 8u;
  l.tmem = l.freq + (kCols / 2) * 4u;
  l.a_full = (l.tmem + 4u + 7u) & ~7u;
  l.acc = l.a_full + 8u;
  l.total = l.acc + 8u;
  return l;
}

struct Args {
  const uint16_t* x;        // [M, K]
  const uint16_t* w_image;  // [N / 32][K / 64] blocks of kBBytes
  const uint16_t* bias;     // [N] or null
  const void* offset;
  int offset_dtype;
  float coef;
  const int64_t* slots;  // [B, T]
  uint16_t* oq;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int64_t m, k, b, h, t, cache_slots;
};

// Byte offset of (row, k core) in a chunk's no-swizzle K-major layout: core
// matrix (row / 8, k / 8) at ((row / 8) * 8 + k / 8) * 128, row % 8 at
// 16-byte steps inside it.  The host packs the weight blocks with the same
// formula (32 rows per block), so a block copies as 4 contiguous KB.
__device__ __forceinline__ uint32_t core_offset(int row, int kcore) {
  return static_cast<uint32_t>(((row >> 3) * 8 + kcore) * 128 + (row & 7) * 16);
}

// Shared-memory matrix descriptor, K-major, no swizzle: K-adjacent core
// matrices 128 bytes apart (LBO), 8-row groups 1024 bytes apart (SBO).
__device__ __forceinline__ uint64_t desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (8ull << 16) | (64ull << 32) | (1ull << 46);
}
// Instruction descriptor: kind::f16, D f32, A and B bf16, both K-major,
// N = 32, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kCols >> 3) << 17) |
                            ((kMmaRows >> 4) << 24);

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}

// 16-byte asynchronous global -> shared copy (completion by wait_group).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1) qkv_rope_kernel(const Args a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sb =
      smem_raw + ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u);
  const int chunks = static_cast<int>(a.k / kChunk);
  const Layout L = layout(chunks);
  float* tab_c = reinterpret_cast<float*>(sb + L.tab);  // [kRows][16]
  float* tab_s = tab_c + kRows * (kCols / 2);
  const uint16_t* bias_s = reinterpret_cast<const uint16_t*>(sb + L.bias);
  int64_t* slot_s = reinterpret_cast<int64_t*>(sb + L.slots);
  float* freq = reinterpret_cast<float*>(sb + L.freq);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sb + L.tmem);
  unsigned long long* a_full = reinterpret_cast<unsigned long long*>(sb + L.a_full);
  unsigned long long* acc_full = reinterpret_cast<unsigned long long*>(sb + L.acc);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nt = blockIdx.x;  // 32-feature tile
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kRows;
  const int which = static_cast<int>(nt / (2 * a.h));  // 0 q, 1 k, 2 v
  const int64_t head = (nt / 2) % a.h;
  const int pair0 = (nt & 1) * (kCols / 2);  // first rotary pair of the tile
  const int rows_here = static_cast<int>(a.m - m0 < kRows ? a.m - m0 : kRows);

  if (tid == 0) {
    pipe::mbar_init(a_full, kLoaderThreads);
    pipe::mbar_init(acc_full, 1);
    pipe::fence_mbar_init();
  }
  if (tid < kCols / 2) freq[tid] = expf(__fmul_rn(static_cast<float>(pair0 + tid), a.coef));
  if (warp == kLoaderWarps) tc::alloc(tmem_slot, kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kLoaderWarps) {
    // ---------------------------------------------------------- MMA
    if (lane == 0) {
      const bool ok = pipe::mbar_wait(a_full, 0);
      tc::fence_after();
      const uint32_t ab = pipe::smem_u32(sb + L.a), bb = pipe::smem_u32(sb + L.b);
      if (ok) {
        for (int c = 0; c < chunks; ++c) {
#pragma unroll
          for (int kk = 0; kk < kChunk / 16; ++kk)
            mma(tmem, desc(ab + c * kAChunk + kk * 256u), desc(bb + c * kBBytes + kk * 256u),
                (c > 0 || kk > 0) ? 1u : 0u);
        }
        tc::commit(acc_full);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- loads, then the epilogue
    {
      const uint32_t ab = pipe::smem_u32(sb + L.a), bb = pipe::smem_u32(sb + L.b);
      // the tile's weight blocks: one contiguous run
      const unsigned char* wsrc =
          reinterpret_cast<const unsigned char*>(a.w_image) + static_cast<int64_t>(nt) * chunks * kBBytes;
      const int wgran = chunks * static_cast<int>(kBBytes / 16);
      for (int g = tid; g < wgran; g += kLoaderThreads) cp_async16(bb + g * 16u, wsrc + g * 16);
      // the token rows, chunk by chunk, in the core-matrix layout
      const int per = rows_here * 8;
      const int xgran = per * chunks;
      for (int g = tid; g < xgran; g += kLoaderThreads) {
        const int c = g / per, rem = g - c * per;
        const int j = rem >> 3, kc = rem & 7;
        cp_async16(ab + static_cast<uint32_t>(c) * kAChunk + core_offset(j, kc),
                   a.x + (m0 + j) * a.k + c * kChunk + kc * 8);
      }
      if (a.bias && tid < kCols * 2 / 16)
        cp_async16(pipe::smem_u32(sb + L.bias) + tid * 16u, a.bias + nt * kCols + tid * 8);
      if (which > 0 && tid < rows_here) slot_s[tid] = a.slots[m0 + tid];
      // the rows' (c, s) pairs while the loads fly
      if (which < 2) {
        for (int e = tid; e < rows_here * (kCols / 2); e += kLoaderThreads) {
          const int r = e / (kCols / 2), p = e % (kCols / 2);
          const int64_t rr = m0 + r;
          const int64_t bi = rr / a.t;
          const float ts = __fadd_rn(offset_as_float(a.offset, a.offset_dtype, bi),
                                     static_cast<float>(rr - bi * a.t));
          const float phase = __fmul_rn(freq[p], ts);
          tab_c[r * (kCols / 2) + p] = cosf(phase);
          tab_s[r * (kCols / 2) + p] = sinf(phase);
        }
      }
      cp_async_wait_all();
      tc::fence_async_shared();
      pipe::mbar_arrive(a_full);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kLoaderThreads) : "memory");
    if (warp == 0) {
      const bool ok = pipe::mbar_wait(acc_full, 0);
      tc::fence_after();
      uint32_t acc[32];
      tc::load32(tmem, acc);  // lanes 0-31 = the CTA's rows
      tc::wait_ld(acc);
      const int rl = lane;
      const int64_t row = m0 + rl;
      if (ok && rl < rows_here) {
        float y[kCols];
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          float v = __uint_as_float(acc[j]);
          if (a.bias) v = __fadd_rn(v, bf16_bits_to_f32(bias_s[j]));
          y[j] = round_to<MOSS_BF16>(v);  // the Linear's bf16 output
        }
        if (which < 2) {
#pragma unroll
          for (int p = 0; p < kCols / 2; ++p) {
            float o0, o1;
            rotate_pair(y[2 * p], y[2 * p + 1], tab_c[rl * (kCols / 2) + p],
                        tab_s[rl * (kCols / 2) + p], o0, o1);
            y[2 * p] = o0;
            y[2 * p + 1] = o1;
          }
        }
        const int64_t bi = row / a.t, ti = row - bi * a.t;
        uint16_t* dst = nullptr;
        if (which == 0) {
          dst = a.oq + ((bi * a.h + head) * a.t + ti) * 64;
        } else {
          const int64_t slot = slot_s[rl];
          if (slot < 0 || slot >= a.cache_slots) {
            record_device_error(MOSS_ERR_VALUE);
          } else {
            dst = (which == 1 ? a.k_cache : a.v_cache) + ((bi * a.h + head) * a.cache_slots + slot) * 64;
          }
        }
        if (dst) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + (nt & 1) * kCols);
#pragma unroll
          for (int j = 0; j < kCols / 8; ++j) d4[j] = pack_bf16x8(y + 8 * j);
        }
      }
    }
  }

  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == kLoaderWarps) tc::dealloc(tmem, kTmemCols);
}

}  // namespace qkvr
}  // namespace moss

using namespace moss;

extern "C" int moss_qkv_rope(const void* x, const void* w_image, const void* bias, int64_t b,
                             int64_t t, int64_t h, int64_t k, const void* offset,
                             int offset_dtype, float freq_coef, const int64_t* slots, void* oq,
                             void* k_cache, void* v_cache, int64_t cache_slots, void* stream) {
  const char* name = "moss_qkv_rope";
  if (b < 0 || t < 0 || h < 1 || k < 1 || cache_slots < 1)
    return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (k % qkvr::kChunk != 0 || k / qkvr::kChunk > qkvr::kMaxChunks)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: the input width must be a multiple of 64, at most %d",
                name, qkvr::kMaxChunks * qkvr::kChunk);
  if (offset_dtype < 0 || offset_dtype > 2)
    return fail(MOSS_ERR_VALUE, "%s: offset dtype must be int64, int32 or float32", name);
  const int64_t m = b * t;
  if (m == 0) return MOSS_OK;
  if (!x || !w_image || !offset || !slots || !oq || !k_cache || !v_cache)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(w_image) || !aligned16(oq) || !aligned16(k_cache) ||
      !aligned16(v_cache) || (bias && !aligned16(bias)))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t ntiles = 3 * h * 2;  // 32-feature tiles of the 3 H 64 outputs
  const int64_t mtiles = (m + qkvr::kRows - 1) / qkvr::kRows;
  if (ntiles > 0x7fffffffLL || mtiles > 65535)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows or heads", name);
  const int chunks = static_cast<int>(k / qkvr::kChunk);
  const size_t smem = qkvr::layout(chunks).total + 128;
  const size_t smax = qkvr::layout(qkvr::kMaxChunks).total + 128;
  static bool configured[kMaxDevices] = {};
  allow_dynamic_smem(qkvr::qkv_rope_kernel, smax, configured);
  qkvr::Args a{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w_image),
               static_cast<const uint16_t*>(bias), offset, offset_dtype, freq_coef, slots,
               static_cast<uint16_t*>(oq), static_cast<uint16_t*>(k_cache),
               static_cast<uint16_t*>(v_cache), m, k, b, h, t, cache_slots};
  qkvr::qkv_rope_kernel<<<dim3(static_cast<unsigned>(ntiles), static_cast<unsigned>(mtiles)),
                          qkvr::kThreads, smem, as_stream(stream)>>>(a);
  return launch_status(name);
}
