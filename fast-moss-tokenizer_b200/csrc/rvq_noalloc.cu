// Quantizer entry point for callers that cannot allocate device memory.
//
// moss_rvq_encode needs a prepared copy of the codebooks (code norms, the
// k-major copy and the tensor-core tile images) in buffers that the caller
// allocates.  This variant keeps that copy in a static device array of the
// library instead, so a caller that owns only its input and output buffers
// can still run the tensor-core quantizer: it prepares the codebooks into
// the array and then calls moss_rvq_encode on them, both on the caller's
// stream.  Capacity: 32 stages x 1024 codes x 64 dims.
#include "common.cuh"

#include <atomic>

namespace moss {
namespace rvq_static {

constexpr int64_t kMaxStages = 32;
constexpr int64_t kMaxCodes = 1024;
constexpr int64_t kDim = 64;
// moss_rvq_packed_floats(32, 1024, 64): the k-major copy (32 x 1024 x 64)
// plus 32 x 4 tensor-core tile images of 18,432 floats.
constexpr int64_t kPackedFloats = kMaxStages * kMaxCodes * kDim + kMaxStages * 4 * 18432;
constexpr int64_t kNormFloats = kMaxStages * kMaxCodes;
constexpr int64_t kStatsFloats = kMaxStages * 4;
constexpr int64_t kScratchFloats = kPackedFloats + kNormFloats + kStatsFloats;

// Prepared codebooks: packed | code norms | stats.  Every call rewrites all
// of it that the encode reads, so nothing here has to start at zero.
static __device__ __align__(256) float g_scratch[kScratchFloats];

// Device address of g_scratch, looked up once per device and kept for the
// life of the process (a lookup by two threads at once stores the same
// value; calls after cudaDeviceReset are not supported).
static std::atomic<float*> g_scratch_ptr[kMaxDevices] = {};

}  // namespace rvq_static
}  // namespace moss

using namespace moss;

extern "C" int moss_rvq_encode_static(const float* x, int64_t rows, int64_t d, const float* books,
                                      int64_t stages, int64_t k, int32_t* codes, float* recon,
                                      float* residual_out, void* stream) {
  using namespace rvq_static;
  const char* name = "moss_rvq_encode_static";
  if (rows < 0 || stages < 1 || k < 1 || d < 1) return fail(MOSS_ERR_VALUE, "%s: bad shape", name);
  // valid sizes this entry point does not cover: MOSS_ERR_UNSUPPORTED, as the
  // prepared-buffer entry points report sizes they do not cover
  if (d != kDim || stages > kMaxStages || k > kMaxCodes)
    return fail(MOSS_ERR_UNSUPPORTED,
                "%s: %lld stages x %lld codes x %lld dims exceed the static scratch "
                "(at most %lld stages x %lld codes x %lld dims); use moss_rvq_prepare_codebooks "
                "and moss_rvq_encode with caller buffers",
                name, static_cast<long long>(stages), static_cast<long long>(k),
                static_cast<long long>(d), static_cast<long long>(kMaxStages),
                static_cast<long long>(kMaxCodes), static_cast<long long>(kDim));
  if (moss_rvq_packed_floats(stages, k, d) > kPackedFloats)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: packed codebooks exceed the static scratch", name);
  if (rows == 0) return MOSS_OK;
  if (!x || !books || !codes || !recon) return fail(MOSS_ERR_VALUE, "%s: null pointer", name);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MOSS_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MOSS_ERR_UNSUPPORTED, "%s: device index %d out of range", name, dev);
  float* packed = g_scratch_ptr[dev].load(std::memory_order_relaxed);
  if (packed == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MOSS_ERR_CUDA, "%s: scratch address lookup failed: %s", name,
                  cudaGetErrorString(e));
    packed = static_cast<float*>(p);
    g_scratch_ptr[dev].store(packed, std::memory_order_relaxed);
  }
  float* code_norm = packed + kPackedFloats;
  float* stats = code_norm + kNormFloats;
  int st = moss_rvq_prepare_codebooks(books, stages, k, d, code_norm, packed, stats, stream);
  if (st != MOSS_OK) return st;
  return moss_rvq_encode(x, rows, d, books, packed, code_norm, stats, stages, k, codes, recon,
                         residual_out, stream);
}
