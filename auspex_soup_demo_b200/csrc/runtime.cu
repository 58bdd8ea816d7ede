// Library-wide state: last error text, SM count, the device error word, the
// wait limit of the GEMM kernels, and the lock of the per-device caches.
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "soup_common.cuh"

namespace soup {

std::mutex& cache_mutex() {
  static std::mutex mu;
  return mu;
}

// Written by bounded waits that expire inside the GEMM kernels (0 = none).
// Kernels receive its address as an argument (see device_err_ptr).
__device__ int g_device_err = 0;
// soup_device_error's read-and-clear writes the old value here.
__device__ int g_device_err_read = 0;

// Per-device addresses, filled once per device with that device current. They
// are not refreshed after cudaDeviceReset (the library assumes the contexts it
// has seen stay alive for the process).
int* device_err_ptr() {
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(cache_mutex());
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_err) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

// Make the current device's primary context current on this host thread. The
// driver-API tensor-map encoder needs one, and a thread such as autograd's
// backward worker may reach a library call before any runtime call bound it.
int bind_context() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  return cuda_status(e);
}

static std::atomic<unsigned long long> g_wait_limit_ns{0};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

namespace {
// One thread takes the error word and clears it in the same atomic step, so a
// code written meanwhile by a kernel on another stream is not lost.
__global__ void take_device_error_kernel() { g_device_err_read = atomicExch(&g_device_err, 0); }
}  // namespace

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
  std::lock_guard<std::mutex> lock(cache_mutex());
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
  cudaStream_t s = soup::as_stream(stream);
  // host callers are serialised too: the read-back slot is shared per device
  std::lock_guard<std::mutex> lock(soup::cache_mutex());
  soup::take_device_error_kernel<<<1, 1, 0, s>>>();
  cudaError_t e = cudaGetLastError();
  int v = 0;
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbolAsync(&v, soup::g_device_err_read, sizeof(int), 0,
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return soup::cuda_status(e);
  *out_code = v;
  return SOUP_OK;
}

int soup_set_wait_limit_ns(uint64_t ns) {
  if (ns != 0 && ns < 1000000ull) {
    soup::set_last_error("soup_set_wait_limit_ns: the limit must be 0 (default, 2 s) or >= 1 ms");
    return SOUP_ERR_INVALID;
  }
  soup::g_wait_limit_ns.store(ns, std::memory_order_relaxed);
  return SOUP_OK;
}

}  // extern "C"
