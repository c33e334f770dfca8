// Error reporting, version and device-error plumbing of the C ABI, and the
// self-test of the bounded-wait path.
#include "common.cuh"
#include "pipeline.cuh"

#include <string.h>

namespace moss {

__device__ int g_device_error = 0;

static thread_local char t_last_error[512] = "no error";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return fail(MOSS_ERR_CUDA, "%s: CUDA launch failed: %s", what, cudaGetErrorString(err));
  }
  return MOSS_OK;
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = c > 0 ? c : 148;
  }
  return counts[dev];
}

}  // namespace moss

extern "C" int moss_version(void) { return 100; }

extern "C" const char* moss_last_error(void) { return moss::t_last_error; }

extern "C" int moss_check_device_error(void* stream) {
  int value = 0;
  const int zero = 0;
  cudaStream_t s = moss::as_stream(stream);
  cudaError_t err = cudaMemcpyFromSymbolAsync(&value, moss::g_device_error, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err == cudaSuccess && value != 0) {
    err = cudaMemcpyToSymbolAsync(moss::g_device_error, &zero, sizeof(int), 0,
                                  cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  }
  if (err != cudaSuccess) {
    return moss::fail(MOSS_ERR_CUDA, "moss_check_device_error: %s", cudaGetErrorString(err));
  }
  if (value != 0) {
    return moss::fail(MOSS_ERR_TIMEOUT,
                      "device error word was %d (a bounded wait gave up or an index was out "
                      "of range)",
                      value);
  }
  return MOSS_OK;
}

namespace moss {

// One warp waits on an mbarrier through the kernels' own bounded wait
// (pipe::mbar_wait).  With `arrive` thread 0 completes the phase first, so
// the wait returns at once; without it nothing completes the phase and
// every thread gives up after limit_ns, recording MOSS_ERR_TIMEOUT.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, int arrive) {
  __shared__ unsigned long long bar;
  if (threadIdx.x == 0) {
    pipe::mbar_init(&bar, 1);
    pipe::fence_mbar_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) pipe::mbar_arrive(&bar);
  pipe::mbar_wait(&bar, 0, limit_ns);
}

}  // namespace moss

extern "C" int moss_test_bounded_wait(int64_t limit_ns, int arrive, void* stream) {
  const char* name = "moss_test_bounded_wait";
  if (limit_ns < 1000 || limit_ns > 100000000)
    return moss::fail(MOSS_ERR_VALUE, "%s: limit must be 1 us to 100 ms", name);
  moss::bounded_wait_probe_kernel<<<1, 32, 0, moss::as_stream(stream)>>>(
      static_cast<uint64_t>(limit_ns), arrive ? 1 : 0);
  return moss::launch_status(name);
}
