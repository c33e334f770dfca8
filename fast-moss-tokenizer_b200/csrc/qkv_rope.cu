// Fused qkv projection with the rotary embedding in its epilogue (sm_100a,
// tcgen05 bf16 MMA, FP32 accumulation in tensor memory).
//
//   y = x W^T + bias      x [M, K] bf16 (row r = b * T + t), W [3 H 64, K]
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
// the dot products is this kernel's (per 16-wide K step in the tensor core,
// the steps in ascending K), not cuBLAS's.
//
// One CTA computes a 128-row x 32-column tile (half a head of q, k or v)
// over the whole K, in chunks of 64:
//   warps 0-3  write each chunk's x rows into shared memory in the MMA's
//              no-swizzle K-major layout (8-row x 16-byte core matrices);
//              then the epilogue, one row per thread (TMEM lane = row);
//   warp 4     bulk-copies each chunk's pre-packed 4 KB weight block;
//   warp 5     allocates 32 TMEM columns and issues 4 MMAs per chunk
//              (kind::f16, bf16 operands, M=128, N=32, K=16).
// Every wait is bounded (~2 s) and records MOSS_ERR_TIMEOUT; a ring slot
// out of range records MOSS_ERR_VALUE and its row's k/v store is skipped.
#include "rotary.cuh"
#include "tcgen05.cuh"

namespace moss {
namespace qkvr {

constexpr int kRows = 128;       // M tile
constexpr int kCols = 32;        // N tile: half a head
constexpr int kChunk = 64;       // K per stage (128 bytes of bf16 per row)
constexpr int kStages = 4;
constexpr uint32_t kABytes = kRows * kChunk * 2;  // 16 KB
constexpr uint32_t kBBytes = kCols * kChunk * 2;  // 4 KB
constexpr int kThreads = 192;
constexpr int kLoaderThreads = 128;
constexpr uint32_t kTmemCols = 32;

struct __align__(128) Smem {
  unsigned char a[kStages][kABytes];
  unsigned char b[kStages][kBBytes];
  float tab_c[kRows][kCols / 2];  // (c, s) of the tile's rows and pairs
  float tab_s[kRows][kCols / 2];
  float freq[kCols / 2];
  uint32_t tmem_base;
  alignas(8) unsigned long long full[kStages];
  alignas(8) unsigned long long empty[kStages];
  alignas(8) unsigned long long acc_full;
};

struct Args {
  const uint16_t* x;  // [M, K]
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

// Byte offset of (row, k) of a chunk in the no-swizzle K-major layout:
// core matrix (row / 8, k / 8) at ((row / 8) * 8 + k / 8) * 128, row % 8 at
// 16-byte steps inside it.  The weight image (rvq-style pre-packed blocks,
// built by the host) uses the same formula per 32-row block.
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
                            ((kRows >> 4) << 24);

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) qkv_rope_kernel(const Args a) {
  extern __shared__ unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(
      smem_raw +
      ((128u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 127u)) & 127u));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nt = blockIdx.x;  // 32-column tile
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kRows;
  const int chunks = static_cast<int>(a.k / kChunk);
  const int which = static_cast<int>(nt / (2 * a.h));  // 0 q, 1 k, 2 v
  const int head = static_cast<int>((nt / 2) % a.h);
  const int pair0 = (nt & 1) * (kCols / 2);  // first rotary pair of the tile

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      pipe::mbar_init(&sm.full[s], 1 + kLoaderThreads);
      pipe::mbar_init(&sm.empty[s], 1);
    }
    pipe::mbar_init(&sm.acc_full, 1);
    pipe::fence_mbar_init();
  }
  if (tid < kCols / 2) sm.freq[tid] = expf(__fmul_rn(static_cast<float>(pair0 + tid), a.coef));
  if (warp == 5) tc::alloc(&sm.tmem_base, kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 4) {
    // ---------------------------------------------------------- weights
    if (lane == 0) {
      const unsigned char* src =
          reinterpret_cast<const unsigned char*>(a.w_image) + static_cast<int64_t>(nt) * chunks * kBBytes;
      for (int c = 0; c < chunks; ++c) {
        const int s = c % kStages;
        if (c >= kStages && !pipe::mbar_wait(&sm.empty[s], ((c / kStages) - 1) & 1)) break;
        pipe::mbar_arrive_expect_tx(&sm.full[s], kBBytes);
        pipe::bulk_g2s(sm.b[s], src + static_cast<int64_t>(c) * kBBytes, kBBytes, &sm.full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = true;
      for (int c = 0; c < chunks && ok; ++c) {
        const int s = c % kStages;
        if (!pipe::mbar_wait(&sm.full[s], (c / kStages) & 1)) {
          ok = false;
          break;
        }
        tc::fence_after();
        const uint32_t ab = pipe::smem_u32(sm.a[s]), bb = pipe::smem_u32(sm.b[s]);
#pragma unroll
        for (int kk = 0; kk < kChunk / 16; ++kk)
          mma(tmem, desc(ab + kk * 256u), desc(bb + kk * 256u), (c > 0 || kk > 0) ? 1u : 0u);
        tc::commit(&sm.empty[s]);
      }
      if (ok) tc::commit(&sm.acc_full);
      // the last stages' commit arrivals land before the CTA can retire
      for (int c = chunks > kStages ? chunks - kStages : 0; ok && c < chunks; ++c)
        ok = pipe::mbar_wait(&sm.empty[c % kStages], (c / kStages) & 1);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- x rows, then the epilogue
    const int rl = tid;  // row in the tile = TMEM lane
    const int64_t row = m0 + rl;
    const bool valid = row < a.m;
    const uint4* xr = reinterpret_cast<const uint4*>(a.x + (valid ? row : 0) * a.k);
    bool ok = true;
    for (int c = 0; c < chunks; ++c) {
      const int s = c % kStages;
      if (ok && c >= kStages && !pipe::mbar_wait(&sm.empty[s], ((c / kStages) - 1) & 1)) ok = false;
      if (ok && valid) {
        const uint32_t base = pipe::smem_u32(sm.a[s]);
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = xr[c * 8 + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) st_shared_v4(base + core_offset(rl, j), v[j]);
      }
      tc::fence_async_shared();
      pipe::mbar_arrive(&sm.full[s]);
    }
    // the tile's (c, s) pairs while the last chunks are multiplied
    const int64_t rows_here = a.m - m0 < kRows ? a.m - m0 : kRows;
    if (which < 2) {
      for (int e = tid; e < rows_here * (kCols / 2); e += kLoaderThreads) {
        const int r = e / (kCols / 2), p = e % (kCols / 2);
        const int64_t rr = m0 + r;
        const int64_t bi = rr / a.t;
        const float ts = __fadd_rn(offset_as_float(a.offset, a.offset_dtype, bi),
                                   static_cast<float>(rr - bi * a.t));
        const float phase = __fmul_rn(sm.freq[p], ts);
        sm.tab_c[r][p] = cosf(phase);
        sm.tab_s[r][p] = sinf(phase);
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (ok) ok = pipe::mbar_wait(&sm.acc_full, 0);
    tc::fence_after();
    uint32_t acc[32];
    tc::load32(tmem + (static_cast<uint32_t>(warp * 32) << 16), acc);
    tc::wait_ld(acc);
    if (ok && valid) {
      const int64_t col0 = static_cast<int64_t>(nt) * kCols;
      float y[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        float v = __uint_as_float(acc[j]);
        if (a.bias) v = __fadd_rn(v, bf16_bits_to_f32(a.bias[col0 + j]));
        y[j] = round_to<MOSS_BF16>(v);  // the Linear's bf16 output
      }
      if (which < 2) {
#pragma unroll
        for (int p = 0; p < kCols / 2; ++p) {
          float o0, o1;
          rotate_pair(y[2 * p], y[2 * p + 1], sm.tab_c[rl][p], sm.tab_s[rl][p], o0, o1);
          y[2 * p] = o0;
          y[2 * p + 1] = o1;
        }
      }
      const int64_t bi = row / a.t, ti = row - bi * a.t;
      uint16_t* dst = nullptr;
      if (which == 0) {
        dst = a.oq + ((bi * a.h + head) * a.t + ti) * 64;
      } else {
        const int64_t slot = a.slots[row];
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

  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (warp == 5) tc::dealloc(tmem, kTmemCols);
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
  if (k % qkvr::kChunk != 0)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: the input width must be a multiple of 64", name);
  if (offset_dtype < 0 || offset_dtype > 2)
    return fail(MOSS_ERR_VALUE, "%s: offset dtype must be int64, int32 or float32", name);
  const int64_t m = b * t;
  if (m == 0) return MOSS_OK;
  if (!x || !w_image || !offset || !slots || !oq || !k_cache || !v_cache)
    return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(w_image) || !aligned16(oq) || !aligned16(k_cache) ||
      !aligned16(v_cache))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t ntiles = 3 * h * 2;  // 32-column tiles of the 3 H 64 outputs
  const int64_t mtiles = (m + qkvr::kRows - 1) / qkvr::kRows;
  if (ntiles > 0x7fffffffLL || mtiles > 65535)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too many rows or heads", name);
  const size_t smem = sizeof(qkvr::Smem) + 128;
  static bool configured[kMaxDevices] = {};
  allow_dynamic_smem(qkvr::qkv_rope_kernel, smem, configured);
  qkvr::Args a{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w_image),
               static_cast<const uint16_t*>(bias), offset, offset_dtype, freq_coef, slots,
               static_cast<uint16_t*>(oq), static_cast<uint16_t*>(k_cache),
               static_cast<uint16_t*>(v_cache), m, k, b, h, t, cache_slots};
  qkvr::qkv_rope_kernel<<<dim3(static_cast<unsigned>(ntiles), static_cast<unsigned>(mtiles)),
                          qkvr::kThreads, smem, as_stream(stream)>>>(a);
  return launch_status(name);
}
