// Shared helpers for the sm_100a kernels: dtype traits, 128-bit vector
// access, warp/block reductions, status handling.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "../../include/soupb200.h"

namespace soup {

// ---------------------------------------------------------------- status ----
void set_last_error(const char* msg);
int cuda_status(cudaError_t e);                      // records the text, maps to SOUP_ERR_CUDA
inline int launch_status() { return cuda_status(cudaGetLastError()); }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();                                       // of the current device (cached)
int* device_err_ptr();                               // device error word of the current device
std::mutex& cache_mutex();                           // guards the library's per-device caches
int bind_context();                                  // current device's context on this thread
uint64_t wait_limit_ns();                            // soup_set_wait_limit_ns (0: the default)

// ---------------------------------------------------------------- dtypes ----
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// A 16-byte vector of T: 4 floats or 8 halves.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 u;
    T v[N];
  };
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld16(const T* p) {
  Vec16<T> r;
  r.u = *reinterpret_cast<const uint4*>(p);
  return r;
}
// Streaming load: data read once, keep it out of L1.
template <typename T>
__device__ __forceinline__ Vec16<T> ld16_stream(const T* p) {
  Vec16<T> r;
  r.u = __ldcs(reinterpret_cast<const uint4*>(p));
  return r;
}
template <typename T>
__device__ __forceinline__ void st16(T* p, const Vec16<T>& r) {
  *reinterpret_cast<uint4*>(p) = r.u;
}
template <typename T>
__device__ __forceinline__ void st16_stream(T* p, const Vec16<T>& r) {
  __stcs(reinterpret_cast<uint4*>(p), r.u);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ------------------------------------------- programmatic dependent launch --
// A kernel launched with launch_pdl() may start while the previous kernel in
// the stream finishes; it must call pdl_wait() before touching memory the
// previous kernel reads or writes. pdl_trigger() lets the next kernel launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------ reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// exp(x) through the hardware base-2 exponential: exp(x) = 2^(x*log2(e)).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes'
// worth of fma / add / mul on a 64-bit register pair).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t p, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(p));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
constexpr float kLn2 = 0.6931471805599453f;

// SwiGLU arithmetic shared by the elementwise kernels and the gate/up GEMM
// epilogue, so both give identical results (solution/kernels/swiglu.py:20-95):
// out = silu(g) u, du = dy silu(g), dg = dy u sigmoid(g) (1 + g (1 - sigmoid(g))).
// The sigmoid uses the hardware exponential and an approximate reciprocal
// division (like the reference's Triton sigmoid): the epilogue evaluates it on
// only 8 warps per SM, where an IEEE division would outlast the MMA of a tile.
// For g -> -inf the divisor overflows and the result is the limit 0.
__device__ __forceinline__ float swiglu_sigmoid(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }
__device__ __forceinline__ float swiglu_fwd_f(float g, float u) {
  const float sg = swiglu_sigmoid(g);
  return (g * sg) * u;
}
__device__ __forceinline__ void swiglu_bwd_f(float d, float g, float u, float& dg, float& du) {
  const float sg = swiglu_sigmoid(g);
  du = d * (g * sg);
  dg = d * u * sg * (1.0f + g * (1.0f - sg));
}

// Online-softmax state of one row segment: running max m, s = sum exp(z-m),
// w = sum z*exp(z-m), first index of the maximum.
struct SoftmaxState {
  float m, s, w;
  int idx;
};

__device__ __forceinline__ SoftmaxState sm_init() { return SoftmaxState{-INFINITY, 0.f, 0.f, 0x7fffffff}; }

// Merge b into a. Ties of the maximum keep the smaller index.
__device__ __forceinline__ SoftmaxState sm_merge(SoftmaxState a, SoftmaxState b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  float m = fmaxf(a.m, b.m);
  float ea = fast_exp2((a.m - m) * kLog2e);
  float eb = fast_exp2((b.m - m) * kLog2e);
  SoftmaxState r;
  r.m = m;
  r.s = a.s * ea + b.s * eb;
  r.w = a.w * ea + b.w * eb;
  if (a.m > b.m) r.idx = a.idx;
  else if (b.m > a.m) r.idx = b.idx;
  else r.idx = min(a.idx, b.idx);
  return r;
}

__device__ __forceinline__ SoftmaxState sm_shfl_xor(const SoftmaxState& a, int o) {
  SoftmaxState b;
  b.m = __shfl_xor_sync(0xffffffffu, a.m, o);
  b.s = __shfl_xor_sync(0xffffffffu, a.s, o);
  b.w = __shfl_xor_sync(0xffffffffu, a.w, o);
  b.idx = __shfl_xor_sync(0xffffffffu, a.idx, o);
  return b;
}

__device__ __forceinline__ SoftmaxState sm_warp_reduce(SoftmaxState a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = sm_merge(a, sm_shfl_xor(a, o));
  return a;
}

}  // namespace soup
