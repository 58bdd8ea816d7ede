// RMSNorm forward and backward (dx and dw in one pass over dy and x).
//
// One warp owns one row: 16-byte vector loads, the row kept in registers,
// a warp-shuffle sum of squares. The backward accumulates dw partials per
// lane across the rows its warp visits, reduces the CTA's 8 warps through
// shared memory in a fixed order into one partial row per CTA, and a second
// small kernel sums those partial rows column by column, again in a fixed
// order: no data atomics, bitwise reproducible.
//
// Semantics: solution/kernels/rmsnorm.py:22-57 (forward), :60-96 (dx) and
// :161-167 (dw, fp32, cast to the weight dtype).
#include <cstdio>
#include <initializer_list>
#include <utility>

#include "soup_common.cuh"

namespace soup {
namespace {

constexpr int kWarps = 8;  // rows per CTA in flight (one per warp)

// Load NE weights starting at w + c as floats (16-byte aligned base).
template <typename W, int NE>
__device__ __forceinline__ void load_w(const W* w, float (&o)[NE]) {
  if constexpr (sizeof(W) * NE == 16) {
    Vec16<W> v = ld16(w);
#pragma unroll
    for (int j = 0; j < NE; ++j) o[j] = Cvt<W>::to_f(v.v[j]);
  } else if constexpr (sizeof(W) * NE == 32) {
    Vec16<W> a = ld16(w), b = ld16(w + Vec16<W>::N);
#pragma unroll
    for (int j = 0; j < Vec16<W>::N; ++j) {
      o[j] = Cvt<W>::to_f(a.v[j]);
      o[j + Vec16<W>::N] = Cvt<W>::to_f(b.v[j]);
    }
  } else {  // 8 bytes: NE = 4 halves
    uint2 u = *reinterpret_cast<const uint2*>(w);
    const W* h = reinterpret_cast<const W*>(&u);
#pragma unroll
    for (int j = 0; j < NE; ++j) o[j] = Cvt<W>::to_f(h[j]);
  }
}

// VPL = 16-byte vectors of x per lane (row length <= 32 * VPL * NE).
template <typename T, typename W, int VPL>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_kernel(const T* __restrict__ x, int64_t xs,
                                                              const W* __restrict__ w,
                                                              T* __restrict__ y, int64_t ys,
                                                              float* __restrict__ rstd,
                                                              int64_t rows, int cols, float eps) {
  constexpr int NE = Vec16<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * xs;
  Vec16<T> xv[VPL];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * NE;
    if (c < cols) {
      xv[i] = ld16_stream(xr + c);
#pragma unroll
      for (int j = 0; j < NE; ++j) {
        const float f = Cvt<T>::to_f(xv[i].v[j]);
        ss = fmaf(f, f, ss);
      }
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  if (lane == 0) rstd[row] = r;
  T* yr = y + row * ys;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * NE;
    if (c < cols) {
      float wf[NE];
      load_w<W, NE>(w + c, wf);
      Vec16<T> o;
#pragma unroll
      for (int j = 0; j < NE; ++j) o.v[j] = Cvt<T>::from_f((Cvt<T>::to_f(xv[i].v[j]) * r) * wf[j]);
      st16_stream(yr + c, o);
    }
  }
}

// dx for every row; per-CTA dw partial row into `partial` (if non-null).
template <typename T, typename W, int VPL>
__global__ void __launch_bounds__(kWarps * 32) rms_bwd_kernel(
    const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
    const W* __restrict__ w, const float* __restrict__ rstd, T* __restrict__ dx, int64_t dxs,
    float* __restrict__ partial, int64_t rows, int cols) {
  constexpr int NE = Vec16<T>::N;
  extern __shared__ float red[];  // [kWarps][cols] when partial != nullptr
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[VPL][NE];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int j = 0; j < NE; ++j) acc[i][j] = 0.f;
  const float inv_cols = 1.0f / static_cast<float>(cols);

  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const T* dyr = dy + row * dys;
    const T* xr = x + row * xs;
    Vec16<T> dv[VPL], xv[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (i * 32 + lane) * NE;
      if (c < cols) {
        dv[i] = ld16_stream(dyr + c);
        xv[i] = ld16_stream(xr + c);
        float wf[NE];
        load_w<W, NE>(w + c, wf);
#pragma unroll
        for (int j = 0; j < NE; ++j)
          s = fmaf(Cvt<T>::to_f(dv[i].v[j]) * wf[j], Cvt<T>::to_f(xv[i].v[j]), s);
      }
    }
    s = warp_sum(s);
    const float r = rstd[row];
    const float k = r * r * s * inv_cols;
    T* dxr = dx + row * dxs;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (i * 32 + lane) * NE;
      if (c < cols) {
        float wf[NE];
        load_w<W, NE>(w + c, wf);
        Vec16<T> o;
#pragma unroll
        for (int j = 0; j < NE; ++j) {
          const float d = Cvt<T>::to_f(dv[i].v[j]);
          const float xx = Cvt<T>::to_f(xv[i].v[j]);
          o.v[j] = Cvt<T>::from_f(r * (d * wf[j] - xx * k));
          acc[i][j] = fmaf(d, xx * r, acc[i][j]);
        }
        st16_stream(dxr + c, o);
      }
    }
  }
  if (partial == nullptr) return;
  // CTA reduction of the 8 warps' dw partials, fixed order.
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (i * 32 + lane) * NE;
    if (c < cols) {
#pragma unroll
      for (int j = 0; j < NE; ++j) red[warp * cols + c + j] = acc[i][j];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) t += red[q * cols + c];
    partial[(int64_t)blockIdx.x * cols + c] = t;
  }
}

// dw[c] = sum over the G partial rows, fixed order: 8 warps split the rows,
// lanes own columns, then the warps' sums are added in warp order.
template <typename W>
__global__ void __launch_bounds__(256) rms_dw_reduce_kernel(const float* __restrict__ partial, int g,
                                                            int cols, W* __restrict__ dw) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float t = 0.f;
  if (c < cols)
    for (int q = warp; q < g; q += 8) t += partial[(int64_t)q * cols + c];
  red[warp][lane] = t;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) s += red[q][lane];
    dw[c] = Cvt<W>::from_f(s);
  }
}

// Generic path (any cols, any alignment): two passes over the row in global
// memory, scalar loads. Same arithmetic.
template <typename T, typename W>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_generic(const T* __restrict__ x, int64_t xs,
                                                               const W* __restrict__ w,
                                                               T* __restrict__ y, int64_t ys,
                                                               float* __restrict__ rstd,
                                                               int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * xs;
  float ss = 0.f;
  for (int c = lane; c < cols; c += 32) {
    const float f = Cvt<T>::to_f(xr[c]);
    ss = fmaf(f, f, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
  if (lane == 0) rstd[row] = r;
  T* yr = y + row * ys;
  for (int c = lane; c < cols; c += 32)
    yr[c] = Cvt<T>::from_f((Cvt<T>::to_f(xr[c]) * r) * Cvt<W>::to_f(w[c]));
}

template <typename T, typename W>
__global__ void __launch_bounds__(kWarps * 32) rms_bwd_generic(
    const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
    const W* __restrict__ w, const float* __restrict__ rstd, T* __restrict__ dx, int64_t dxs,
    float* __restrict__ partial, int64_t rows, int cols) {
  // dw partials: one partial row per warp (partial has gridDim.x * kWarps rows).
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + warp;
  if (partial)
    for (int c = lane; c < cols; c += 32) partial[gw * cols + c] = 0.f;
  for (int64_t row = gw; row < rows; row += (int64_t)gridDim.x * kWarps) {
    const T* dyr = dy + row * dys;
    const T* xr = x + row * xs;
    float s = 0.f;
    for (int c = lane; c < cols; c += 32)
      s = fmaf(Cvt<T>::to_f(dyr[c]) * Cvt<W>::to_f(w[c]), Cvt<T>::to_f(xr[c]), s);
    s = warp_sum(s);
    const float r = rstd[row];
    const float k = r * r * s / static_cast<float>(cols);
    T* dxr = dx + row * dxs;
    for (int c = lane; c < cols; c += 32) {
      const float d = Cvt<T>::to_f(dyr[c]);
      const float xx = Cvt<T>::to_f(xr[c]);
      dxr[c] = Cvt<T>::from_f(r * (d * Cvt<W>::to_f(w[c]) - xx * k));
      if (partial) partial[gw * cols + c] += d * (xx * r);
    }
  }
}

// ----------------------------------------------------------- dispatch ------
template <typename T>
int vpl_for(int64_t cols) {
  const int64_t per = 32 * Vec16<T>::N;
  const int64_t need = (cols + per - 1) / per;
  const int opts[] = {1, 2, 4, 6, 8, 12, 16};
  for (int o : opts)
    if (need <= o) return o;
  return 0;
}

template <typename T, typename W>
bool vec_ok(int64_t cols, std::initializer_list<std::pair<const void*, int64_t>> mats, const void* w) {
  if (cols % Vec16<T>::N) return false;
  if (!aligned16(w)) return false;
  for (auto& m : mats)
    if (!aligned16(m.first) || ((m.second * (int64_t)sizeof(T)) % 16) != 0) return false;
  return vpl_for<T>(cols) > 0;
}

template <typename T, typename W>
int fwd_impl(const void* x, int64_t xs, const void* w, void* y, int64_t ys, float* rstd,
             int64_t rows, int64_t cols, float eps, cudaStream_t st) {
  const T* X = static_cast<const T*>(x);
  const W* Wt = static_cast<const W*>(w);
  T* Y = static_cast<T*>(y);
  const unsigned grid = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
  if (vec_ok<T, W>(cols, {{x, xs}, {y, ys}}, w)) {
    switch (vpl_for<T>(cols)) {
#define SOUP_RMS_F(V)                                                                     \
  case V:                                                                                 \
    rms_fwd_kernel<T, W, V><<<grid, kWarps * 32, 0, st>>>(X, xs, Wt, Y, ys, rstd, rows,   \
                                                          (int)cols, eps);                \
    break;
      SOUP_RMS_F(1) SOUP_RMS_F(2) SOUP_RMS_F(4) SOUP_RMS_F(6) SOUP_RMS_F(8) SOUP_RMS_F(12)
      SOUP_RMS_F(16)
#undef SOUP_RMS_F
    }
  } else {
    rms_fwd_generic<T, W><<<grid, kWarps * 32, 0, st>>>(X, xs, Wt, Y, ys, rstd, rows, (int)cols, eps);
  }
  return launch_status();
}

// Number of CTAs of the backward (and of dw partial rows).
int bwd_grid(int64_t rows) {
  int64_t g = (rows + kWarps - 1) / kWarps;
  const int64_t cap = num_sms();
  return static_cast<int>(g < cap ? g : cap);
}

template <typename T, typename W>
int bwd_impl(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
             const float* rstd, void* dx, int64_t dxs, void* dw, void* ws, size_t ws_bytes,
             int64_t rows, int64_t cols, cudaStream_t st) {
  const int grid = bwd_grid(rows);
  const bool vec = vec_ok<T, W>(cols, {{dy, dys}, {x, xs}, {dx, dxs}}, w);
  const int prows = vec ? grid : grid * kWarps;
  float* partial = nullptr;
  if (dw) {
    if (!ws || ws_bytes < (size_t)prows * cols * sizeof(float) || !aligned16(ws)) {
      set_last_error("soup_rmsnorm_bwd: workspace too small");
      return SOUP_ERR_WORKSPACE;
    }
    partial = static_cast<float*>(ws);
  }
  const T* DY = static_cast<const T*>(dy);
  const T* X = static_cast<const T*>(x);
  const W* Wt = static_cast<const W*>(w);
  T* DX = static_cast<T*>(dx);
  if (vec) {
    const size_t smem = dw ? (size_t)kWarps * cols * sizeof(float) : 0;
    switch (vpl_for<T>(cols)) {
#define SOUP_RMS_B(V)                                                                         \
  case V: {                                                                                   \
    auto k = rms_bwd_kernel<T, W, V>;                                                         \
    if (smem > 48 * 1024) {                                                                   \
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                           (int)smem);                                        \
      if (e != cudaSuccess) return cuda_status(e);                                            \
    }                                                                                         \
    k<<<grid, kWarps * 32, smem, st>>>(DY, dys, X, xs, Wt, rstd, DX, dxs, partial, rows,      \
                                       (int)cols);                                            \
    break;                                                                                    \
  }
      SOUP_RMS_B(1) SOUP_RMS_B(2) SOUP_RMS_B(4) SOUP_RMS_B(6) SOUP_RMS_B(8) SOUP_RMS_B(12)
      SOUP_RMS_B(16)
#undef SOUP_RMS_B
    }
  } else {
    rms_bwd_generic<T, W><<<grid, kWarps * 32, 0, st>>>(DY, dys, X, xs, Wt, rstd, DX, dxs, partial,
                                                        rows, (int)cols);
  }
  int rc = launch_status();
  if (rc || !dw) return rc;
  rms_dw_reduce_kernel<W><<<(unsigned)((cols + 31) / 32), 256, 0, st>>>(partial, prows, (int)cols,
                                                                       static_cast<W*>(dw));
  return launch_status();
}

}  // namespace
}  // namespace soup

using namespace soup;

#define SOUP_DISPATCH_XW(XD, WD, CALL)                                                   \
  do {                                                                                    \
    if ((XD) == SOUP_F32 && (WD) == SOUP_F32) return CALL(float, float);                  \
    if ((XD) == SOUP_F32 && (WD) == SOUP_BF16) return CALL(float, __nv_bfloat16);         \
    if ((XD) == SOUP_F32 && (WD) == SOUP_F16) return CALL(float, __half);                 \
    if ((XD) == SOUP_BF16 && (WD) == SOUP_BF16) return CALL(__nv_bfloat16, __nv_bfloat16); \
    if ((XD) == SOUP_BF16 && (WD) == SOUP_F32) return CALL(__nv_bfloat16, float);         \
    if ((XD) == SOUP_BF16 && (WD) == SOUP_F16) return CALL(__nv_bfloat16, __half);        \
    if ((XD) == SOUP_F16 && (WD) == SOUP_F16) return CALL(__half, __half);                \
    if ((XD) == SOUP_F16 && (WD) == SOUP_F32) return CALL(__half, float);                 \
    if ((XD) == SOUP_F16 && (WD) == SOUP_BF16) return CALL(__half, __nv_bfloat16);        \
  } while (0)

extern "C" {

int soup_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, void* y,
                     int64_t y_row_stride, float* rstd, int64_t rows, int64_t cols, float eps,
                     int x_dtype, int w_dtype, void* stream) {
  if (!x || !weight || !y || !rstd || rows < 0 || cols <= 0 || cols > (1 << 20) ||
      x_row_stride < cols || y_row_stride < cols) {
    set_last_error("soup_rmsnorm_fwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  cudaStream_t st = as_stream(stream);
#define CALL(T, W) fwd_impl<T, W>(x, x_row_stride, weight, y, y_row_stride, rstd, rows, cols, eps, st)
  SOUP_DISPATCH_XW(x_dtype, w_dtype, CALL);
#undef CALL
  set_last_error("soup_rmsnorm_fwd: unsupported dtype");
  return SOUP_ERR_INVALID;
}

size_t soup_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  // generic path keeps one partial row per warp; the vector path one per CTA
  return (size_t)bwd_grid(rows) * kWarps * (size_t)cols * sizeof(float);
}

int soup_rmsnorm_bwd(const void* dy, int64_t dy_row_stride, const void* x, int64_t x_row_stride,
                     const void* weight, const float* rstd, void* dx, int64_t dx_row_stride,
                     void* dw, void* workspace, size_t workspace_bytes, int64_t rows,
                     int64_t cols, int x_dtype, int w_dtype, void* stream) {
  if (!dy || !x || !weight || !rstd || !dx || rows < 0 || cols <= 0 || cols > (1 << 20) ||
      dy_row_stride < cols || x_row_stride < cols || dx_row_stride < cols) {
    set_last_error("soup_rmsnorm_bwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  cudaStream_t st = as_stream(stream);
#define CALL(T, W)                                                                        \
  bwd_impl<T, W>(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx, dx_row_stride, dw, \
                 workspace, workspace_bytes, rows, cols, st)
  SOUP_DISPATCH_XW(x_dtype, w_dtype, CALL);
#undef CALL
  set_last_error("soup_rmsnorm_bwd: unsupported dtype");
  return SOUP_ERR_INVALID;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// RMSNorm backward that allocates nothing.
//
// For callers that cannot hand the library a scratch buffer: code that runs
// under an allocator owning all device memory (a framework's caching pool that
// has reserved the GPU, a fixed-budget serving process), or host code that
// must not call cudaMalloc because cudaMalloc may synchronise the device. The
// dw reduction's per-CTA partial rows live in the file-scope array below
// instead; every GPU that loads this library holds it until the process exits.
// ---------------------------------------------------------------------------
namespace soup {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
__device__ __align__(256) float g_rms_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the array, looked up once per device with that device
// current. In host code the array's name is only a host-side stand-in, so the
// kernels must receive this address instead.
float* noalloc_scratch(int* status) {
  static float* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = cuda_status(e);
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    set_last_error("soup_rmsnorm_bwd_noalloc: device index out of range");
    *status = SOUP_ERR_UNSUPPORTED;
    return nullptr;
  }
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rms_noalloc_scratch);
    if (e != cudaSuccess) {
      *status = cuda_status(e);
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  *status = SOUP_OK;
  return addr[dev];
}

// Bytes of dw partial rows the backward writes for these operands.
template <typename T, typename W>
size_t bwd_partial_bytes(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
                         const void* dx, int64_t dxs, int64_t rows, int64_t cols) {
  const bool vec = vec_ok<T, W>(cols, {{dy, dys}, {x, xs}, {dx, dxs}}, w);
  const size_t prows = static_cast<size_t>(vec ? bwd_grid(rows) : bwd_grid(rows) * kWarps);
  return prows * static_cast<size_t>(cols) * sizeof(float);
}

size_t bwd_partial_bytes_any(int xd, int wd, const void* dy, int64_t dys, const void* x,
                             int64_t xs, const void* w, const void* dx, int64_t dxs, int64_t rows,
                             int64_t cols) {
#define NEED(T, W) bwd_partial_bytes<T, W>(dy, dys, x, xs, w, dx, dxs, rows, cols)
  SOUP_DISPATCH_XW(xd, wd, NEED);
#undef NEED
  return 0;  // unsupported dtype pair
}

}  // namespace
}  // namespace soup

extern "C" {

int soup_rmsnorm_bwd_noalloc(const void* dy, int64_t dy_row_stride, const void* x,
                             int64_t x_row_stride, const void* weight, const float* rstd,
                             void* dx, int64_t dx_row_stride, void* dw, int64_t rows,
                             int64_t cols, int x_dtype, int w_dtype, void* stream) {
  if (!dy || !x || !weight || !rstd || !dx || rows < 0 || cols <= 0 || cols > (1 << 20) ||
      dy_row_stride < cols || x_row_stride < cols || dx_row_stride < cols) {
    set_last_error("soup_rmsnorm_bwd_noalloc: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  if (dw) {
    const size_t need = bwd_partial_bytes_any(x_dtype, w_dtype, dy, dy_row_stride, x, x_row_stride,
                                              weight, dx, dx_row_stride, rows, cols);
    if (need == 0) {
      set_last_error("soup_rmsnorm_bwd_noalloc: unsupported dtype");
      return SOUP_ERR_INVALID;
    }
    if (need > kNoAllocScratchBytes) {
      char msg[200];
      snprintf(msg, sizeof(msg),
               "soup_rmsnorm_bwd_noalloc: dw needs %zu bytes of scratch, the built-in buffer holds "
               "%zu; pass a workspace to soup_rmsnorm_bwd instead",
               need, kNoAllocScratchBytes);
      set_last_error(msg);
      return SOUP_ERR_WORKSPACE;
    }
    int status = SOUP_OK;
    ws = noalloc_scratch(&status);
    if (!ws) return status;
    ws_bytes = kNoAllocScratchBytes;
  }
  cudaStream_t st = as_stream(stream);
#define CALL(T, W)                                                                        \
  bwd_impl<T, W>(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx, dx_row_stride, dw, \
                 ws, ws_bytes, rows, cols, st)
  SOUP_DISPATCH_XW(x_dtype, w_dtype, CALL);
#undef CALL
  set_last_error("soup_rmsnorm_bwd_noalloc: unsupported dtype");
  return SOUP_ERR_INVALID;
}

}  // extern "C"
