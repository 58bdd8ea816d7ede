// Library-wide state: last error text, SM count, the device error word.
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "soup_common.cuh"

namespace soup {

// Written by bounded waits that expire inside the GEMM kernels (0 = none).
// Kernels receive its address as an argument (see device_err_ptr).
__device__ int g_device_err = 0;

int* device_err_ptr() {
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_err) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

static thread_local char g_last_error[512] = "";

void set_last_error(const char* msg) {
  strncpy(g_last_error, msg, sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = 0;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return SOUP_OK;
  snprintf(g_last_error, sizeof(g_last_error), "CUDA error %d: %s", static_cast<int>(e),
           cudaGetErrorString(e));
  return SOUP_ERR_CUDA;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace soup

extern "C" {

int soup_version(void) { return 1; }

const char* soup_last_error(void) { return soup::g_last_error; }

int soup_device_error(void* stream, int* out_code) {
  if (!out_code) return SOUP_ERR_INVALID;
  int v = 0;
  cudaStream_t s = soup::as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, soup::g_device_err, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return soup::cuda_status(e);
  *out_code = v;
  if (v != 0) {
    int zero = 0;
    e = cudaMemcpyToSymbolAsync(soup::g_device_err, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return soup::cuda_status(e);
  }
  return SOUP_OK;
}

}  // extern "C"
