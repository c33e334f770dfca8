// Bias + (gated) activation, one pass over HBM.
//
// The reference has no kernel for the FFN activation (it lives in the
// upstream model code); this reproduces the eager PyTorch chain that runs
// there, with one rounding to the storage dtype per torch op:
//   h    = round(x + bias)
//   a    = round(act(h_gate))           act evaluated in float32:
//            silu(v)      = v / (1 + expf(-v))
//            gelu_erf(v)  = v * 0.5 * (1 + erff(v * sqrt(1/2)))
//            gelu_tanh(v) = 0.5 * v * (1 + tanhf(k_beta * fma(0.044715, v^3, v)))
//   y    = round(a * h_up)              (gated)   or   y = a (ungated)
// For bf16 with the gate width a multiple of 8, each thread produces 8
// outputs from 16-byte loads of the gate half, the up half and the bias;
// the bias adds and the gating product run as packed bf16 operations,
// which give the same bits as the float32 op followed by the bf16 rounding.
#include <atomic>
#include <mutex>

#include "activation.cuh"
#include "pipeline.cuh"

namespace moss {

// Without a bias there is no add at all (so -0 stays -0, as in torch).
template <int DT, int ACT, bool GATED>
__device__ __forceinline__ float gate_value(float xg, float bg, float xu, float bu, bool hasb) {
  const float hg = hasb ? round_to<DT>(__fadd_rn(xg, bg)) : xg;
  const float a = round_to<DT>(activation<ACT, DT>(hg));
  if constexpr (GATED) {
    const float hu = hasb ? round_to<DT>(__fadd_rn(xu, bu)) : xu;
    return __fmul_rn(a, hu);
  } else {
    return a;
  }
}

// Eight bf16 outputs (four packed pairs) from packed gate, bias and up
// values, without branches.  Bit j of `redo` is set when output j must be
// recomputed by gate_exact_one: SiLU near a bf16 rounding midpoint (see
// silu_fast) or a gating product below 2^-125 (see bf16x2_mul).
template <int ACT, bool GATED>
__device__ __forceinline__ uint4 gate_item_fast(const uint4& g4, const uint4& bg4, const uint4& u4,
                                                const uint4& bu4, bool has_bias, uint32_t& redo) {
  const uint32_t xg[4] = {g4.x, g4.y, g4.z, g4.w};
  const uint32_t bg[4] = {bg4.x, bg4.y, bg4.z, bg4.w};
  uint32_t a[4];
  redo = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t hg = has_bias ? bf16x2_add(xg[p], bg[p]) : xg[p];  // exact
    const float v0 = __uint_as_float(hg << 16), v1 = __uint_as_float(hg & 0xffff0000u);
    if constexpr (ACT == MOSS_ACT_SILU) {
      bool r0, r1;
      const float q0 = silu_fast(v0, r0), q1 = silu_fast(v1, r1);
      redo |= (static_cast<uint32_t>(r0) | (static_cast<uint32_t>(r1) << 1)) << (2 * p);
      a[p] = pack_bf16x2(q0, q1);
    } else {
      a[p] = pack_bf16x2(activation<ACT, MOSS_BF16>(v0), activation<ACT, MOSS_BF16>(v1));
    }
  }
  if constexpr (GATED) {
    const uint32_t xu[4] = {u4.x, u4.y, u4.z, u4.w};
    const uint32_t bu[4] = {bu4.x, bu4.y, bu4.z, bu4.w};
    uint32_t y[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t hu = has_bias ? bf16x2_add(xu[p], bu[p]) : xu[p];
      y[p] = bf16x2_mul(a[p], hu);
      redo |= static_cast<uint32_t>(bf16x2_tiny(y[p])) * (3u << (2 * p));
    }
    return make_uint4(y[0], y[1], y[2], y[3]);
  } else {
    return make_uint4(a[0], a[1], a[2], a[3]);
  }
}

// One output from its bf16 inputs, the torch chain op by op in float32.
template <int ACT, bool GATED>
__device__ __forceinline__ uint16_t gate_exact_one(uint16_t xg, uint16_t bg, uint16_t xu,
                                                   uint16_t bu, bool has_bias) {
  const float hg = has_bias ? round_to<MOSS_BF16>(__fadd_rn(bf16_bits_to_f32(xg), bf16_bits_to_f32(bg)))
                            : bf16_bits_to_f32(xg);
  const float av = ACT == MOSS_ACT_SILU ? silu_exact(hg) : activation<ACT, MOSS_BF16>(hg);
  const float a = round_to<MOSS_BF16>(av);
  if constexpr (GATED) {
    const float hu = has_bias ? round_to<MOSS_BF16>(__fadd_rn(bf16_bits_to_f32(xu), bf16_bits_to_f32(bu)))
                              : bf16_bits_to_f32(xu);
    return f32_to_bf16_bits(__fmul_rn(a, hu));
  } else {
    return f32_to_bf16_bits(a);
  }
}

// Register-path item: fast outputs, then the flagged ones exactly (a
// warp-uniform test first, so the exact code runs only when needed).
template <int ACT, bool GATED>
__device__ __forceinline__ uint4 gate_item(const uint4& g4, const uint4& bg4, const uint4& u4,
                                           const uint4& bu4, bool has_bias) {
  uint32_t redo;
  uint4 y = gate_item_fast<ACT, GATED>(g4, bg4, u4, bu4, has_bias, redo);
  if (__builtin_expect(__any_sync(__activemask(), redo != 0u), 0)) {
    uint32_t w[4] = {y.x, y.y, y.z, y.w};
    const uint32_t xg[4] = {g4.x, g4.y, g4.z, g4.w}, bg[4] = {bg4.x, bg4.y, bg4.z, bg4.w};
    const uint32_t xu[4] = {u4.x, u4.y, u4.z, u4.w}, bu[4] = {bu4.x, bu4.y, bu4.z, bu4.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if ((redo >> j) & 1u) {
        const int p = j >> 1, sh = (j & 1) * 16;
        const uint16_t o = gate_exact_one<ACT, GATED>(
            static_cast<uint16_t>(xg[p] >> sh), static_cast<uint16_t>(bg[p] >> sh),
            static_cast<uint16_t>(xu[p] >> sh), static_cast<uint16_t>(bu[p] >> sh), has_bias);
        w[p] = (w[p] & ~(0xffffu << sh)) | (static_cast<uint32_t>(o) << sh);
      }
    }
    y = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return y;
}

// Vector path (bf16, 8 outputs per item).  out_w = width of the output row;
// rows * out_w / 8 < 2^31 (the host splits larger calls into row chunks).
template <int ACT, bool GATED>
__global__ void __launch_bounds__(256) gated_act_bf16x8_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ bias, uint16_t* __restrict__ y,
    uint32_t items, FastDiv per_row, int64_t width, int64_t out_w) {
  // Two items per iteration: all of their loads are issued before any math.
  constexpr int kU = 2;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  const bool has_bias = bias != nullptr;
  for (uint32_t it0 = blockIdx.x * blockDim.x + threadIdx.x; it0 < items; it0 += kU * stride) {
    uint4 rg[kU], rb[kU], ru[kU], rbu[kU];
    int64_t dst[kU];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const uint32_t it = it0 + j * stride;
      rg[j] = rb[j] = ru[j] = rbu[j] = zero;
      dst[j] = -1;
      if (it < items) {
        const uint32_t r = fast_div(it, per_row);
        const int64_t c = static_cast<int64_t>(it - r * per_row.d) * 8;
        const uint16_t* xr = x + static_cast<int64_t>(r) * width + c;
        rg[j] = *reinterpret_cast<const uint4*>(xr);
        if (has_bias) rb[j] = *reinterpret_cast<const uint4*>(bias + c);
        if constexpr (GATED) {
          ru[j] = *reinterpret_cast<const uint4*>(xr + out_w);
          if (has_bias) rbu[j] = *reinterpret_cast<const uint4*>(bias + out_w + c);
        }
        dst[j] = static_cast<int64_t>(r) * out_w + c;
      }
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      if (dst[j] < 0) continue;
      *reinterpret_cast<uint4*>(y + dst[j]) = gate_item<ACT, GATED>(rg[j], rb[j], ru[j], rbu[j], has_bias);
    }
  }
}

template <int DT, int ACT, bool GATED>
__global__ void __launch_bounds__(256) gated_act_scalar_kernel(const void* __restrict__ x,
                                                               const void* __restrict__ bias,
                                                               void* __restrict__ y, int64_t rows,
                                                               int64_t width, int64_t out_w) {
  const int64_t items = rows * out_w;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = it / out_w;
    const int64_t c = it - r * out_w;
    const float xg = load_as_f32<DT>(x, r * width + c);
    const float bg = bias ? load_as_f32<DT>(bias, c) : 0.0f;
    float xu = 0.0f, bu = 0.0f;
    if constexpr (GATED) {
      xu = load_as_f32<DT>(x, r * width + out_w + c);
      bu = bias ? load_as_f32<DT>(bias, out_w + c) : 0.0f;
    }
    store_from_f32<DT>(y, it, gate_value<DT, ACT, GATED>(xg, bg, xu, bu, bias != nullptr));
  }
}

// Activation tables.  The activation of a bf16 input rounded to bf16 is a
// function of the 65536 input bit patterns only, so each activation is
// tabulated once per device with the exact torch formula (activation_exact)
// and the streaming kernel looks the values up: every output is then the
// torch value by construction, whatever the input.
__device__ __align__(16) uint16_t g_act_lut[3 * 65536];

__global__ void act_lut_kernel() {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;  // grid covers 65536 exactly
  const float v = bf16_bits_to_f32(static_cast<uint16_t>(h));
  g_act_lut[h] = f32_to_bf16_bits(activation_exact<MOSS_ACT_SILU>(v));
  g_act_lut[65536 + h] = f32_to_bf16_bits(activation_exact<MOSS_ACT_GELU_ERF>(v));
  g_act_lut[2 * 65536 + h] = f32_to_bf16_bits(activation_exact<MOSS_ACT_GELU_TANH>(v));
}

// True once the tables of the current device are built.  The first call
// outside a graph capture builds them on `s` and waits for the build, so
// kernels on every stream (and in graphs captured later) find them written.
// While `s` is being captured nothing may be waited for, and a build
// recorded into the graph would run only at its replay: the caller then
// takes the register kernel, which gives the same bits.
bool act_lut_ready(cudaStream_t s) {
  static std::atomic<bool> ready[kMaxDevices];
  static std::mutex build;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  if (ready[dev].load(std::memory_order_acquire)) return true;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &capture) != cudaSuccess || capture != cudaStreamCaptureStatusNone)
    return false;
  std::lock_guard<std::mutex> lock(build);
  if (ready[dev].load(std::memory_order_acquire)) return true;
  act_lut_kernel<<<65536 / 256, 256, 0, s>>>();
  if (cudaPeekAtLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) return false;
  ready[dev].store(true, std::memory_order_release);
  return true;
}

// Streaming path (bf16, rows of at most kStageBytes): one CTA per SM.  A
// producer thread streams tiles of whole rows of x into a ring of
// shared-memory stages with bulk copies (the activation table once, beside
// them); the consumer warps compute 8 outputs per 16-byte item from shared
// memory and store them straight to y.  A consumer thread handles the same
// (row in tile, column) items in every tile, so its bias values stay in
// registers.
namespace gstream {
#ifndef MOSS_STREAM_CONSUMERS
#define MOSS_STREAM_CONSUMERS 512
#endif
constexpr int kConsumers = MOSS_STREAM_CONSUMERS;
constexpr int kThreads = kConsumers + 32;
constexpr int kStages = 6;
constexpr int kStageBytes = 16384;
constexpr int kLutBytes = 65536 * 2;
// 16-byte output items per consumer thread and tile (a stage holds at most
// kStageBytes / 16 items of gate input).
constexpr int kSlots = (kStageBytes / 16 + kConsumers - 1) / kConsumers;

struct Args {
  const uint16_t* x;
  const uint16_t* bias;
  uint16_t* y;
  int64_t rows, width, out_w;
  int tile_rows;        // rows per stage
  uint32_t ntiles;
  FastDiv per_row;      // 16-byte output items per row (out_w / 8)
};

// Layout: stages | table | barriers.
constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + kLutBytes +
                              (2 * kStages + 2) * 8;
}  // namespace gstream

// Two adjacent outputs from a packed pair of rounded gate inputs.
__device__ __forceinline__ uint32_t lut_pair(const uint16_t* lut, uint32_t hg) {
  return static_cast<uint32_t>(lut[hg & 0xffffu]) | (static_cast<uint32_t>(lut[hg >> 16]) << 16);
}

template <int ACT, bool GATED>
__global__ void __launch_bounds__(gstream::kThreads, 1)
    gated_act_stream_kernel(const gstream::Args a) {
  using namespace gstream;
  extern __shared__ __align__(128) unsigned char smem[];
  const uint16_t* lut = reinterpret_cast<const uint16_t*>(smem + kStages * kStageBytes);
  unsigned long long* full =
      reinterpret_cast<unsigned long long*>(smem + kStages * kStageBytes + kLutBytes);
  unsigned long long* empty = full + kStages;
  unsigned long long* lut_bar = full + 2 * kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2 * kStages + 1);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      pipe::mbar_init(&full[s], 1);
      pipe::mbar_init(&empty[s], kConsumers / 32);
    }
    pipe::mbar_init(lut_bar, 1);
    *abort_flag = 0;
    pipe::fence_mbar_init();
  }
  __syncthreads();

  if (tid >= kConsumers) {  // producer warp: one thread issues every copy
    if (tid != kConsumers) return;
    uint32_t i = 0;
    for (uint32_t tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++i) {
      const int s = static_cast<int>(i % kStages);
      if (i >= kStages && !pipe::mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      const int64_t r0 = static_cast<int64_t>(tile) * a.tile_rows;
      const int64_t nr = a.rows - r0 < a.tile_rows ? a.rows - r0 : a.tile_rows;
      const uint32_t bytes = static_cast<uint32_t>(nr * a.width * 2);
      pipe::mbar_arrive_expect_tx(&full[s], bytes);
      pipe::bulk_g2s(smem + s * kStageBytes, a.x + r0 * a.width, bytes, &full[s]);
      if (i == 0) {  // the first data tile is in flight; now the table
        pipe::mbar_arrive_expect_tx(lut_bar, kLutBytes);
        pipe::bulk_g2s(smem + kStages * kStageBytes, g_act_lut + ACT * 65536, kLutBytes, lut_bar);
      }
    }
    // Drain: the copies of the last issued tiles must land before exit.
    for (uint32_t j = i > kStages ? i - kStages : 0; j < i; ++j)
      pipe::mbar_wait(&full[j % kStages], (j / kStages) & 1);
    if (i > 0) pipe::mbar_wait(lut_bar, 0);
    return;
  }

  // Consumer warps (the grid never exceeds the tile count, so every CTA
  // has a first tile and the table copy is issued).
  const int lane = tid & 31;
  const bool has_bias = a.bias != nullptr;
  const uint32_t full_items = static_cast<uint32_t>(a.tile_rows) * a.per_row.d;
  uint32_t row[kSlots], col[kSlots];  // row in the tile (large: no item), column
  uint32_t bg[kSlots][4], bu[kSlots][4];
#pragma unroll
  for (int m = 0; m < kSlots; ++m) {
    const uint32_t it = tid + m * kConsumers;
    row[m] = 0x7fffffffu;
    col[m] = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) bg[m][p] = bu[m][p] = 0u;
    if (it < full_items) {
      row[m] = fast_div(it, a.per_row);
      col[m] = (it - row[m] * a.per_row.d) * 8;
      if (has_bias) {
        const uint4 b = *reinterpret_cast<const uint4*>(a.bias + col[m]);
        bg[m][0] = b.x; bg[m][1] = b.y; bg[m][2] = b.z; bg[m][3] = b.w;
        if constexpr (GATED) {
          const uint4 c = *reinterpret_cast<const uint4*>(a.bias + a.out_w + col[m]);
          bu[m][0] = c.x; bu[m][1] = c.y; bu[m][2] = c.z; bu[m][3] = c.w;
        }
      }
    }
  }
  if (!pipe::mbar_wait(lut_bar, 0)) {
    *abort_flag = 1;
    return;
  }
  uint32_t i = 0;
  for (uint32_t tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++i) {
    const int s = static_cast<int>(i % kStages);
    if (*abort_flag || !pipe::mbar_wait(&full[s], (i / kStages) & 1)) {
      *abort_flag = 1;
      return;
    }
    const int64_t r0 = static_cast<int64_t>(tile) * a.tile_rows;
    const uint32_t nr = static_cast<uint32_t>(a.rows - r0 < a.tile_rows ? a.rows - r0 : a.tile_rows);
    const uint16_t* st = reinterpret_cast<const uint16_t*>(smem + s * kStageBytes);
    uint16_t* yt = a.y + r0 * a.out_w;
    // Products below 2^-125 (see bf16x2_mul) are flagged and redone in
    // float32 afterwards, so the main loop has no data-dependent branch.
    uint32_t redo_all = 0;
#pragma unroll
    for (int m = 0; m < kSlots; ++m) {
      if (row[m] < nr) {
        const uint16_t* xr = st + row[m] * static_cast<uint32_t>(a.width) + col[m];
        const uint4 g4 = *reinterpret_cast<const uint4*>(xr);
        uint32_t out[4] = {g4.x, g4.y, g4.z, g4.w};
        uint4 u4 = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (GATED) u4 = *reinterpret_cast<const uint4*>(xr + a.out_w);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          if (has_bias) out[p] = bf16x2_add(out[p], bg[m][p]);  // exact, see bf16x2_add
          out[p] = lut_pair(lut, out[p]);
        }
        if constexpr (GATED) {
          uint32_t xu[4] = {u4.x, u4.y, u4.z, u4.w};
          uint32_t tiny = 0;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            if (has_bias) xu[p] = bf16x2_add(xu[p], bu[m][p]);
            out[p] = bf16x2_mul(out[p], xu[p]);
            tiny |= static_cast<uint32_t>(bf16x2_tiny(out[p])) << p;
          }
          redo_all |= tiny << (4 * m);
        }
        *reinterpret_cast<uint4*>(yt + static_cast<int64_t>(row[m]) * a.out_w + col[m]) =
            make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
    if constexpr (GATED) {
      const uint32_t am = __activemask();
      if (__builtin_expect(__any_sync(am, redo_all != 0u), 0)) {
        for (int m = 0; m < kSlots; ++m) {
          if (!((redo_all >> (4 * m)) & 0xfu)) continue;
          const uint16_t* xr = st + row[m] * static_cast<uint32_t>(a.width) + col[m];
          for (int j = 0; j < 8; ++j) {
            if (!((redo_all >> (4 * m + j / 2)) & 1u)) continue;
            float g = bf16_bits_to_f32(xr[j]), u = bf16_bits_to_f32(xr[a.out_w + j]);
            if (has_bias) {
              g = round_to<MOSS_BF16>(__fadd_rn(g, bf16_bits_to_f32(a.bias[col[m] + j])));
              u = round_to<MOSS_BF16>(__fadd_rn(u, bf16_bits_to_f32(a.bias[a.out_w + col[m] + j])));
            }
            const float av = bf16_bits_to_f32(lut[f32_to_bf16_bits(g)]);
            yt[static_cast<int64_t>(row[m]) * a.out_w + col[m] + j] =
                f32_to_bf16_bits(__fmul_rn(av, u));
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) pipe::mbar_arrive(&empty[s]);
  }
}

// Outputs from which the shared-memory table kernel is used.  Below it
// every block would load the 128 KB table for a few rows, and the register
// kernel (the same exact formula per element) is faster: measured on B200
// (bf16, width 5120, GELU) 1.57 against 2.89 us at 4 rows, 1.87 against
// 3.00 at 32, 3.33 against 3.71 at 256; equal at 1024 rows.
#ifndef MOSS_GATE_STREAM_MIN
#define MOSS_GATE_STREAM_MIN (1 << 22)
#endif
constexpr int64_t kStreamMinOutputs = MOSS_GATE_STREAM_MIN;

template <int ACT, bool GATED>
static void launch_gated(const void* x, const void* bias, void* y, int dtype, int64_t rows,
                         int64_t width, int64_t out_w, bool vec, cudaStream_t s) {
  const int sms = sm_count();
  if (vec && width * 2 <= gstream::kStageBytes && rows < 0x7fffffffLL &&
      rows * out_w >= kStreamMinOutputs && act_lut_ready(s)) {
    gstream::Args a{};
    a.x = static_cast<const uint16_t*>(x);
    a.bias = static_cast<const uint16_t*>(bias);
    a.y = static_cast<uint16_t*>(y);
    a.rows = rows;
    a.width = width;
    a.out_w = out_w;
    a.tile_rows = static_cast<int>(gstream::kStageBytes / (width * 2));
    a.ntiles = static_cast<uint32_t>((rows + a.tile_rows - 1) / a.tile_rows);
    a.per_row = make_fastdiv(static_cast<uint32_t>(out_w / 8));
    const size_t shmem = gstream::kSmemBytes;
    static bool attr_done[kMaxDevices] = {};  // per instantiation and device
    allow_dynamic_smem(gated_act_stream_kernel<ACT, GATED>, shmem, attr_done);
    const uint32_t grid = a.ntiles < static_cast<uint32_t>(sms) ? a.ntiles : static_cast<uint32_t>(sms);
    gated_act_stream_kernel<ACT, GATED><<<grid, gstream::kThreads, shmem, s>>>(a);
    return;
  }
  if (vec) {
    // Row chunks of fewer than 2^31 items of 8 outputs.
    const int64_t per_row = out_w / 8;
    const int64_t chunk = 0x7fffffffLL / per_row;
    const FastDiv fd = make_fastdiv(static_cast<uint32_t>(per_row));
    for (int64_t r0 = 0; r0 < rows; r0 += chunk) {
      const int64_t nr = rows - r0 < chunk ? rows - r0 : chunk;
      const int64_t items = nr * per_row;
      int64_t grid = (items + 255) / 256;
      if (grid > static_cast<int64_t>(sms) * 8) grid = static_cast<int64_t>(sms) * 8;
      gated_act_bf16x8_kernel<ACT, GATED><<<static_cast<unsigned>(grid), 256, 0, s>>>(
          static_cast<const uint16_t*>(x) + r0 * width, static_cast<const uint16_t*>(bias),
          static_cast<uint16_t*>(y) + r0 * out_w, static_cast<uint32_t>(items), fd, width, out_w);
    }
  } else {
    const int64_t items = rows * out_w;
    int64_t grid = (items + 255) / 256;
    if (grid > static_cast<int64_t>(sms) * 8) grid = static_cast<int64_t>(sms) * 8;
    if (dtype == MOSS_BF16) {
      gated_act_scalar_kernel<MOSS_BF16, ACT, GATED>
          <<<static_cast<unsigned>(grid), 256, 0, s>>>(x, bias, y, rows, width, out_w);
    } else {
      gated_act_scalar_kernel<MOSS_F32, ACT, GATED>
          <<<static_cast<unsigned>(grid), 256, 0, s>>>(x, bias, y, rows, width, out_w);
    }
  }
}

}  // namespace moss

using namespace moss;

extern "C" int moss_gated_act(const void* x, const void* bias, void* y, int dtype, int64_t rows,
                              int64_t width, int act, int gated, void* stream) {
  const char* name = "moss_gated_act";
  if (rows < 0 || width <= 0) return fail(MOSS_ERR_VALUE, "%s: rows >= 0 and width > 0 required", name);
  if (dtype != MOSS_F32 && dtype != MOSS_BF16)
    return fail(MOSS_ERR_VALUE, "%s: dtype must be float32 or bfloat16", name);
  if (act < MOSS_ACT_SILU || act > MOSS_ACT_GELU_TANH)
    return fail(MOSS_ERR_VALUE, "%s: unknown activation %d", name, act);
  if (gated && (width % 2)) return fail(MOSS_ERR_VALUE, "%s: gated width must be even", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !y) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  const int64_t out_w = gated ? width / 2 : width;
  const bool vec = dtype == MOSS_BF16 && (out_w % 8 == 0) && aligned16(x) && aligned16(y) &&
                   (bias == nullptr || aligned16(bias));
  cudaStream_t s = as_stream(stream);
#define MOSS_GA(A)                                                              \
  if (gated) launch_gated<A, true>(x, bias, y, dtype, rows, width, out_w, vec, s); \
  else launch_gated<A, false>(x, bias, y, dtype, rows, width, out_w, vec, s);
  if (act == MOSS_ACT_SILU) {
    MOSS_GA(MOSS_ACT_SILU)
  } else if (act == MOSS_ACT_GELU_ERF) {
    MOSS_GA(MOSS_ACT_GELU_ERF)
  } else {
    MOSS_GA(MOSS_ACT_GELU_TANH)
  }
#undef MOSS_GA
  return launch_status(name);
}
