// Linear layer on cached bf16 weights (sm_100a, tcgen05), with the bias and
// the feed-forward activation in its epilogue.
//
//   y[m, n] = bf16(x[m, :] . w[n, :] + bias[n])           (MOSS_LINEAR_BIAS)
//   y[m, n] = bf16(act(bf16(bf16(x . w) + bias[n])))        (MOSS_LINEAR_BIAS_ACT)
//
// x [M, K] bf16 row-major; w [N, K] bf16 (the cached bf16 copy of an FP32
// Linear weight, as the reference's cached Linear keeps it:
// fast_moss/v2_runtime.py:77-106), packed once by moss_linear_pack_weight;
// FP32 accumulation on the tensor cores.  The second form is the streaming
// stack's feed-forward input: a Linear without bias whose bf16 output goes
// through act(h + b), one rounding per torch op (moss_gated_act, ungated).
//
// Why this shape.  A streaming chunk has 4 tokens per stream, so M is 4 at
// one stream and 256 at 64; N and K are 1280-5120, and the weights dominate
// the bytes (13 MB for a 5120 x 1280 Linear).  So the weights are the MMA's
// M side -- 128 output features per tile, the 128 TMEM lanes -- and the
// tokens its N side (padded to a multiple of 16, at most 128 per tile).
// There are only N / 128 feature tiles (10 to 40), too few to pull the
// weights at HBM rate, so K is split across the CTAs of a thread-block
// cluster (1, 2, 4 or 8 CTAs):
//   warp 0     producer: per 64-wide K chunk one bulk copy of the weight
//              block (16 KB, contiguous: the packed image holds each tile's
//              chunks back to back, already in the MMA's 128-byte-swizzled
//              K-major layout) and one TMA load of the token tile [npad x 64]
//              (2-D tensor map, 128-byte swizzle, rows past M read as zeros),
//              completion counted in bytes on the stage's mbarrier;
//   warp 1     TMEM allocator + MMA issuer: per chunk 4 x tcgen05.mma
//              kind::f16 (M=128, N=npad, K=16) into one FP32 accumulator;
//   warps 2-5  epilogue: each thread owns one feature row of the
//              accumulator; it reads the row with tcgen05.ld and sends every
//              value straight to the cluster CTA that finishes that feature
//              (st.async into the owner's shared memory, counted in bytes on
//              the owner's mbarrier).  The owner adds the C partials of its
//              128 / C features in cluster-rank order from its own shared
//              memory, applies the epilogue and stores 8 outputs (16 bytes)
//              per item.
// Every output is therefore one fixed sum order: deterministic, but not
// cuBLAS's order, so it can differ from F.linear by the rounding of a
// different FP32 sum.  Every mbarrier wait is bounded (~2 s,
// MOSS_ERR_TIMEOUT); no load uses cluster multicast.
#include <cuda.h>

#include "activation.cuh"
#include "tcgen05.cuh"

namespace moss {
namespace lin {

constexpr int kFeat = 128;         // output features per tile (MMA M, TMEM lanes)
constexpr int kChunk = 64;         // K per stage: 128 bytes of bf16 per row
constexpr int kMaxTok = 128;       // tokens per tile (MMA N)
constexpr int kThreads = 192;      // producer, MMA, 4 epilogue warps
constexpr int kEpiThreads = 128;
constexpr int kMaxCluster = 8;
constexpr uint32_t kABytes = kFeat * kChunk * 2;  // 16 KB weight block
constexpr uint32_t kSmemBudget = 221184;          // 216 KB: stages + partials

struct Params {
  CUtensorMap x_map;        // x [M, K]: box {64, npad}
  const uint16_t* w_image;  // [N / 128][K / 64] blocks of 16 KB
  const uint16_t* bias;     // [N] bf16 or null
  uint16_t* y;              // [M, N] bf16
  int64_t m, n;
  int nchunks;   // K / 64
  int npad;      // tokens per tile, multiple of 16, <= 128
  int stages;
  int cluster;   // CTAs splitting K
  int epilogue;  // MOSS_LINEAR_*
  int act;       // MOSS_ACT_* (epilogue BIAS_ACT)
  int use_lut;   // the activation tables are built: look act(h) up
};

__host__ __device__ inline uint32_t stage_bytes(int npad) {
  return kABytes + static_cast<uint32_t>(npad) * 128u;
}
// Partial sums every CTA receives: [cluster][npad][128 / cluster] FP32.
__host__ __device__ inline uint32_t recv_bytes(int npad) {
  return static_cast<uint32_t>(npad) * kFeat * 4u;
}

// K-major operand tile of 128-byte rows with the 128-byte swizzle: 16-byte
// chunk c of row r at chunk c ^ (r % 8), 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// kind::f16, D f32, A and B bf16, both K-major, M = 128, N = npad.
__device__ __forceinline__ uint32_t idesc(int npad) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(npad >> 3) << 17) |
         (static_cast<uint32_t>(kFeat >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
// 2-D tiled TMA load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(pipe::smem_u32(bar))
      : "memory");
}
// 16 consecutive accumulator columns of this thread's TMEM lane (whole warp).
__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t (&r)[16]) {
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait16(uint32_t (&r)[16]) {
  __syncwarp();
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// 4 bytes into a cluster CTA's shared memory, counted on its mbarrier.
__device__ __forceinline__ void st_async(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(
                   addr),
               "f"(v), "r"(bar)
               : "memory");
}

// act(h) with h = f + bias rounded to bf16, f the Linear's bf16 output;
// without a bias there is no add (so -0 stays -0, as in the eager chain).
// With the tables built, act(h) rounded to bf16 is looked up (the tables
// hold activation_exact of every bf16 input: the same bits).
template <int ACT>
__device__ __forceinline__ float bias_act(float acc, float b, bool has_bias, bool lut) {
  const float f = round_to<MOSS_BF16>(acc);
  const float h = has_bias ? round_to<MOSS_BF16>(__fadd_rn(f, b)) : f;
  if (lut) return bf16_bits_to_f32(g_act_lut[ACT * 65536 + f32_to_bf16_bits(h)]);
  return activation_exact<ACT>(h);
}

__global__ void __launch_bounds__(kThreads, 1) linear_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment: the 128-byte swizzle pattern follows address bits
  unsigned char* sb = smem_raw + ((1024u - (static_cast<uint32_t>(
                                                __cvta_generic_to_shared(smem_raw)) & 1023u)) &
                                  1023u);
  const uint32_t sbytes = stage_bytes(p.npad);
  float* recv = reinterpret_cast<float*>(sb + p.stages * sbytes);  // [C][npad][R]
  unsigned long long* full =
      reinterpret_cast<unsigned long long*>(sb + p.stages * sbytes + recv_bytes(p.npad));
  unsigned long long* empty = full + p.stages;
  unsigned long long* acc_full = empty + p.stages;
  unsigned long long* red_full = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_full + 1);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int crank = static_cast<int>(cluster_rank());
  const int C = p.cluster;
  const int R = kFeat / C;  // features each CTA finishes
  const int ftile = blockIdx.y;
  const int ttile = blockIdx.z;
  // this CTA's share of the K chunks
  const int c0 = static_cast<int>(static_cast<int64_t>(p.nchunks) * crank / C);
  const int c1 = static_cast<int>(static_cast<int64_t>(p.nchunks) * (crank + 1) / C);
  const int nloc = c1 - c0;
  const uint32_t tcols = p.npad <= 32 ? 32u : (p.npad <= 64 ? 64u : 128u);

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      pipe::mbar_init(&full[s], 1);
      pipe::mbar_init(&empty[s], 1);
    }
    pipe::mbar_init(acc_full, 1);
    pipe::mbar_init(red_full, 1);
    // every peer's partials for this CTA's features: C x npad x R floats
    pipe::mbar_arrive_expect_tx(red_full, recv_bytes(p.npad));
    pipe::fence_mbar_init();
  }
  if (warp == 1) tc::alloc(tmem_slot, tcols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  // this CTA's mbarriers are initialised: peers may send once all have arrived
  cluster_arrive();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.x_map))
                   : "memory");
      const uint16_t* wsrc =
          p.w_image + (static_cast<int64_t>(ftile) * p.nchunks + c0) * (kABytes / 2);
      int issued = 0;
      for (int i = 0; i < nloc; ++i) {
        const int s = i % p.stages;
        if (!pipe::mbar_wait(&empty[s], ((i / p.stages) & 1) ^ 1)) {
          ok = false;
          break;
        }
        pipe::mbar_arrive_expect_tx(&full[s], sbytes);
        const uint32_t a = pipe::smem_u32(sb + s * sbytes);
        pipe::bulk_g2s(sb + s * sbytes, wsrc + static_cast<int64_t>(i) * (kABytes / 2), kABytes,
                       &full[s]);
        tma_load_2d(a + kABytes, &p.x_map, (c0 + i) * kChunk, ttile * kMaxTok, &full[s]);
        ++issued;
      }
      // copies still in flight land before this CTA may retire
      for (int i = issued > p.stages ? issued - p.stages : 0; i < issued; ++i)
        pipe::mbar_wait(&full[i % p.stages], (i / p.stages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t id = idesc(p.npad);
      for (int i = 0; i < nloc && ok; ++i) {
        const int s = i % p.stages;
        if (!pipe::mbar_wait(&full[s], (i / p.stages) & 1)) {
          ok = false;
          break;
        }
        tc::fence_after();
        const uint32_t a = pipe::smem_u32(sb + s * sbytes);
#pragma unroll
        for (int kk = 0; kk < kChunk / 16; ++kk)
          mma_bf16(tmem, sw128_desc(a + kk * 32u), sw128_desc(a + kABytes + kk * 32u), id,
                   (i > 0 || kk > 0) ? 1u : 0u);
        tc::commit(&empty[s]);
      }
      if (ok) {
        tc::commit(acc_full);
        pipe::mbar_wait(acc_full, 0);  // the commits have landed before the CTA retires
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may read
    const int feat = quarter * 32 + lane;
    const bool have = nloc > 0 && pipe::mbar_wait(acc_full, 0);
    tc::fence_after();
    cluster_wait();  // every peer's mbarriers are initialised
    // send this row's partial sums to the CTA that finishes feature `feat`
    const int owner = feat / R, lr = feat - owner * R;
    const uint32_t base = peer_addr(pipe::smem_u32(recv), static_cast<uint32_t>(owner));
    const uint32_t bar = peer_addr(pipe::smem_u32(red_full), static_cast<uint32_t>(owner));
    for (int j0 = 0; j0 < p.npad; j0 += 16) {
      uint32_t r[16];
      tmem_load16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(j0),
                  r);
      tmem_wait16(r);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t off = static_cast<uint32_t>(((crank * p.npad + j0 + j) * R + lr) * 4);
        st_async(base + off, have ? __uint_as_float(r[j]) : 0.0f, bar);
      }
    }
    // the C partials of this CTA's features, added in cluster-rank order
    pipe::mbar_wait(red_full, 0);
    const int et = tid - 64;
    const int groups = R / 8;
    const int64_t m0 = static_cast<int64_t>(ttile) * kMaxTok;
    const int tok = static_cast<int>(p.m - m0 < kMaxTok ? p.m - m0 : kMaxTok);
    for (int item = et; item < tok * groups; item += kEpiThreads) {
      const int j = item / groups, g = item - j * groups;
      float v[8];
      {
        const float4* src = reinterpret_cast<const float4*>(recv + j * R + g * 8);
        const float4 lo = src[0], hi = src[1];
        v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
        v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
      }
      for (int q = 1; q < C; ++q) {
        const float4* src = reinterpret_cast<const float4*>(recv + (q * p.npad + j) * R + g * 8);
        const float4 lo = src[0], hi = src[1];
        v[0] = __fadd_rn(v[0], lo.x); v[1] = __fadd_rn(v[1], lo.y);
        v[2] = __fadd_rn(v[2], lo.z); v[3] = __fadd_rn(v[3], lo.w);
        v[4] = __fadd_rn(v[4], hi.x); v[5] = __fadd_rn(v[5], hi.y);
        v[6] = __fadd_rn(v[6], hi.z); v[7] = __fadd_rn(v[7], hi.w);
      }
      const int64_t n0 = static_cast<int64_t>(ftile) * kFeat + crank * R + g * 8;
      float b[8];
      if (p.bias) {
        unpack_bf16x8(*reinterpret_cast<const uint4*>(p.bias + n0), b);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = 0.0f;
      }
      if (p.epilogue == MOSS_LINEAR_BIAS) {
        if (p.bias) {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], b[e]);
        }
      } else if (p.act == MOSS_ACT_SILU) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = bias_act<MOSS_ACT_SILU>(v[e], b[e], p.bias != nullptr, p.use_lut != 0);
      } else if (p.act == MOSS_ACT_GELU_ERF) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = bias_act<MOSS_ACT_GELU_ERF>(v[e], b[e], p.bias != nullptr, p.use_lut != 0);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = bias_act<MOSS_ACT_GELU_TANH>(v[e], b[e], p.bias != nullptr, p.use_lut != 0);
      }
      *reinterpret_cast<uint4*>(p.y + (m0 + j) * p.n + n0) = pack_bf16x8(v);
    }
  }
  if (warp < 2) cluster_wait();  // matches the arrive after set-up
  tc::fence_before();
  // every CTA has received all of its partials: no transfer is in flight
  // when the cluster leaves
  cluster_arrive();
  cluster_wait();
  tc::fence_after();
  if (warp == 1) tc::dealloc(tmem, tcols);
}

// The packed image: for every 128-row tile and 64-column chunk, 16 KB in
// the operand layout above (row r, 16-byte chunk c at byte
// (r / 8) * 1024 + (r % 8) * 128 + (c ^ (r % 8)) * 16), chunks of a tile
// back to back.  One thread per 16-byte unit of the image.
__global__ void __launch_bounds__(256) pack_kernel(const uint4* __restrict__ w, int64_t k,
                                                   int nchunks, int64_t units,
                                                   uint4* __restrict__ image) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const int64_t block = u >> 10;  // 1024 units of 16 bytes per block
  const int q = static_cast<int>(u & 1023);
  const int64_t ftile = block / nchunks;
  const int chunk = static_cast<int>(block - ftile * nchunks);
  const int r = (q >> 6) * 8 + ((q >> 3) & 7);
  const int c = (q & 7) ^ (r & 7);
  image[u] = w[((ftile * kFeat + r) * k + static_cast<int64_t>(chunk) * kChunk) / 8 + c];
}

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiled>(f);
  }();
  return fn;
}

// Row-major bf16 [rows, k] with a box of `box_rows` rows x 64 columns.
bool encode(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
  EncodeTiled fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace lin
}  // namespace moss

using namespace moss;

extern "C" int moss_linear_cluster(int64_t m, int64_t n, int64_t k) {
  if (m < 1 || n < lin::kFeat || k < lin::kChunk) return 1;
  const int64_t ftiles = n / lin::kFeat;
  const int64_t ttiles = (m + lin::kMaxTok - 1) / lin::kMaxTok;
  const int64_t nch = k / lin::kChunk;
  const int64_t sms = sm_count();
  int c = 1;
  while (c < lin::kMaxCluster && ftiles * ttiles * c * 2 <= sms && c * 2 <= nch) c *= 2;
  return c;
}

extern "C" int moss_linear_pack_weight(const void* w, int64_t n, int64_t k, void* image,
                                       void* stream) {
  const char* name = "moss_linear_pack_weight";
  if (n < 1 || k < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (k % lin::kChunk || n % lin::kFeat)
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: the input width must be a multiple of 64 and the output width a multiple "
                "of 128",
                name);
  if (!w || !image) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(w) || !aligned16(image))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t units = n * k / 8;
  const int64_t grid = (units + 255) / 256;
  if (grid > 0x7fffffffLL) return fail(MOSS_ERR_UNSUPPORTED, "%s: too large", name);
  lin::pack_kernel<<<static_cast<unsigned>(grid), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(w), k, static_cast<int>(k / lin::kChunk), units,
      static_cast<uint4*>(image));
  return launch_status(name);
}

extern "C" int moss_linear(const void* x, int64_t m, int64_t k, const void* w_image, int64_t n,
                           const void* bias, int epilogue, int act, void* y, void* stream) {
  const char* name = "moss_linear";
  if (m < 0 || k < 1 || n < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  if (epilogue != MOSS_LINEAR_BIAS && epilogue != MOSS_LINEAR_BIAS_ACT)
    return fail(MOSS_ERR_VALUE, "%s: unknown epilogue %d", name, epilogue);
  if (epilogue == MOSS_LINEAR_BIAS_ACT && (act < MOSS_ACT_SILU || act > MOSS_ACT_GELU_TANH))
    return fail(MOSS_ERR_VALUE, "%s: unknown activation %d", name, act);
  if (k % lin::kChunk || n % lin::kFeat)
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: the input width must be a multiple of 64 and the output width a multiple "
                "of 128",
                name);
  if (m == 0) return MOSS_OK;
  if (!x || !w_image || !y) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  if (!aligned16(x) || !aligned16(w_image) || !aligned16(y) || (bias && !aligned16(bias)))
    return fail(MOSS_ERR_VALUE, "%s: buffers must be 16-byte aligned", name);
  const int64_t ttiles = (m + lin::kMaxTok - 1) / lin::kMaxTok;
  if (n / lin::kFeat > 65535 || ttiles > 65535 || k / lin::kChunk > 0x7fffffff)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: too large", name);
  lin::Params p{};
  const int tok = static_cast<int>(m < lin::kMaxTok ? m : lin::kMaxTok);
  p.npad = (tok + 15) / 16 * 16;
  if (!lin::encode(&p.x_map, x, m, k, p.npad))
    return fail(MOSS_ERR_CUDA, "%s: tensor map encoding failed", name);
  p.w_image = static_cast<const uint16_t*>(w_image);
  p.bias = static_cast<const uint16_t*>(bias);
  p.y = static_cast<uint16_t*>(y);
  p.m = m;
  p.n = n;
  p.nchunks = static_cast<int>(k / lin::kChunk);
  p.cluster = moss_linear_cluster(m, n, k);
  p.epilogue = epilogue;
  p.act = act;
  p.use_lut = epilogue == MOSS_LINEAR_BIAS_ACT && act_lut_ready(as_stream(stream)) ? 1 : 0;
  const uint32_t sbytes = lin::stage_bytes(p.npad);
  int stages = static_cast<int>((lin::kSmemBudget - lin::recv_bytes(p.npad)) / sbytes);
  const int per_cta = (p.nchunks + p.cluster - 1) / p.cluster;
  if (stages > 8) stages = 8;
  if (stages > per_cta) stages = per_cta;
  if (stages < 2) stages = 2;
  p.stages = stages;
  // stages | received partials | 2 * stages + 2 mbarriers and the TMEM address
  const size_t smem = static_cast<size_t>(stages) * sbytes + lin::recv_bytes(p.npad) +
                      (2 * stages + 3) * 8 + 1024;
  static bool configured[kMaxDevices] = {};
  allow_dynamic_smem(lin::linear_kernel, 232448 - 1024, configured);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(p.cluster), static_cast<unsigned>(n / lin::kFeat),
                     static_cast<unsigned>(ttiles));
  cfg.blockDim = dim3(lin::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, lin::linear_kernel, p);
  if (e != cudaSuccess) return fail(MOSS_ERR_CUDA, "%s: launch failed: %s", name, cudaGetErrorString(e));
  return launch_status(name);
}
