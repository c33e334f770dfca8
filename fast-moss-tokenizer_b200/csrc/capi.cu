// Error reporting, version and device-error plumbing of the C ABI.
#include "common.cuh"

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
