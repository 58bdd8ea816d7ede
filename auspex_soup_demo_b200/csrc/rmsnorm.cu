// RMSNorm forward and backward (dx and dw in one pass over dy and x).
//
// Vector path (16-byte aligned rows, cols a multiple of the vector width): a
// CTA owns one row at a time (grid-stride over rows; as many CTAs as fit on
// the GPU at once), each thread one to four 16-byte vectors of the row, the
// next row's vectors loaded before the current row is reduced, a fixed-order
// block reduction. The backward keeps a dw partial per thread in registers
// across its CTA's rows and writes one partial row per CTA; a second small
// kernel adds those rows column by column in a fixed order: no data
// atomics, bitwise reproducible. Kernels launch with programmatic dependent
// launch so a kernel's start overlaps the previous kernel's tail.
// Generic path (any alignment): one warp per row, scalar accesses.
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

// ---------------------------------------------------------------------------
// Vector path: one CTA owns one row at a time (grid-stride over rows, the
// next row's loads issued before the current row is reduced), every thread
// one or more 16-byte vectors of the row, a fixed-order block reduction.
// The weight row stays in registers for all the CTA's rows.
// ---------------------------------------------------------------------------

// Sum of one float per thread over the CTA, same value returned to every
// thread; warp sums, then the warp totals added in warp order.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] is reused row after row
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// Row kernels: a CTA owns one row at a time (grid-stride over rows, one CTA
// per SM slot), each thread VPT 16-byte vectors of it, the next row's vectors
// loaded before the current row is reduced. Few registers per thread keep
// several CTAs (rows) in flight per SM; the weight row stays in registers.
template <typename T, typename W, int VPT>
__global__ void __launch_bounds__(512) rms_fwd_rows(const T* __restrict__ x, int64_t xs,
                                                    const W* __restrict__ w, T* __restrict__ y,
                                                    int64_t ys, float* __restrict__ rstd,
                                                    int64_t rows, int cols, float eps) {
  constexpr int NE = Vec16<T>::N;
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int nvec = cols / NE;
  float wf[VPT][NE];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int j = threadIdx.x + v * blockDim.x;
    if (j < nvec) load_w<W, NE>(w + j * NE, wf[v]);
  }
  Vec16<T> cur[VPT], nxt[VPT];
  int64_t row = blockIdx.x;
  if (row < rows) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) cur[v] = ld16_stream(x + row * xs + j * NE);
    }
  }
  for (; row < rows; row += gridDim.x) {
    const int64_t nrow = row + gridDim.x;
    if (nrow < rows) {
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int j = threadIdx.x + v * blockDim.x;
        if (j < nvec) nxt[v] = ld16_stream(x + nrow * xs + j * NE);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          const float f = Cvt<T>::to_f(cur[v].v[e]);
          ss = fmaf(f, f, ss);
        }
      }
    }
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
    if (threadIdx.x == 0) rstd[row] = r;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
        Vec16<T> o;
#pragma unroll
        for (int e = 0; e < NE; ++e) o.v[e] = Cvt<T>::from_f((Cvt<T>::to_f(cur[v].v[e]) * r) * wf[v][e]);
        st16_stream(y + row * ys + j * NE, o);
      }
    }
#pragma unroll
    for (int v = 0; v < VPT; ++v) cur[v] = nxt[v];
  }
}

// dx for the CTA's rows; with partial != nullptr the CTA's dw partial
// (registers, fixed row order) is written as partial[blockIdx.x][cols].
template <typename T, typename W, int VPT, bool DW>
__global__ void __launch_bounds__(512) rms_bwd_rows(
    const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
    const W* __restrict__ w, const float* __restrict__ rstd, T* __restrict__ dx, int64_t dxs,
    float* __restrict__ partial, int64_t rows, int cols) {
  constexpr int NE = Vec16<T>::N;
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int nvec = cols / NE;
  const float inv_cols = 1.0f / static_cast<float>(cols);
  float wf[VPT][NE], acc[VPT][NE];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int j = threadIdx.x + v * blockDim.x;
#pragma unroll
    for (int e = 0; e < NE; ++e) acc[v][e] = 0.f;
    if (j < nvec) load_w<W, NE>(w + j * NE, wf[v]);
  }
  Vec16<T> cd[VPT], cx[VPT], nd[VPT], nx[VPT];
  int64_t row = blockIdx.x;
  if (row < rows) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
        cd[v] = ld16_stream(dy + row * dys + j * NE);
        cx[v] = ld16_stream(x + row * xs + j * NE);
      }
    }
  }
  for (; row < rows; row += gridDim.x) {
    const int64_t nrow = row + gridDim.x;
    if (nrow < rows) {
#pragma unroll
      for (int v = 0; v < VPT; ++v) {
        const int j = threadIdx.x + v * blockDim.x;
        if (j < nvec) {
          nd[v] = ld16_stream(dy + nrow * dys + j * NE);
          nx[v] = ld16_stream(x + nrow * xs + j * NE);
        }
      }
    }
    const float r = rstd[row];
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
#pragma unroll
        for (int e = 0; e < NE; ++e)
          s = fmaf(Cvt<T>::to_f(cd[v].v[e]) * wf[v][e], Cvt<T>::to_f(cx[v].v[e]), s);
      }
    }
    s = block_sum(s, red);
    const float k = r * r * s * inv_cols;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
        Vec16<T> o;
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          const float d = Cvt<T>::to_f(cd[v].v[e]);
          const float xx = Cvt<T>::to_f(cx[v].v[e]);
          o.v[e] = Cvt<T>::from_f(r * (d * wf[v][e] - xx * k));
          if (DW) acc[v][e] = fmaf(d, xx * r, acc[v][e]);
        }
        st16_stream(dx + row * dxs + j * NE, o);
      }
    }
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      cd[v] = nd[v];
      cx[v] = nx[v];
    }
  }
  if constexpr (DW) {
    float* dst = partial + (int64_t)blockIdx.x * cols;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const int j = threadIdx.x + v * blockDim.x;
      if (j < nvec) {
#pragma unroll
        for (int q = 0; q < NE; q += 4)
          *reinterpret_cast<float4*>(dst + j * NE + q) =
              make_float4(acc[v][q], acc[v][q + 1], acc[v][q + 2], acc[v][q + 3]);
      }
    }
  }
}

// dw[c] = sum of the partial rows, fixed order: lanes own 4 columns (float4),
// the 32 warps of the CTA split the rows (warp w takes rows w, w+32, ...,
// eight of them in flight per lane), then the warp totals are added in warp
// order.
template <typename W>
__global__ void __launch_bounds__(1024) rms_dw_reduce_vec(const float* __restrict__ partial, int g,
                                                          int cols, W* __restrict__ dw) {
  __shared__ float4 red[32][32];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = (blockIdx.x * 32 + lane) * 4;
  float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < cols) {
    for (int q0 = warp; q0 < g; q0 += 32 * 8) {
      float4 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = q0 + 32 * u;
        a[u] = q < g ? *reinterpret_cast<const float4*>(partial + (int64_t)q * cols + c)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        t.x += a[u].x;
        t.y += a[u].y;
        t.z += a[u].z;
        t.w += a[u].w;
      }
    }
  }
  red[warp][lane] = t;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float4 s = red[0][lane];
    for (int i = 1; i < 32; ++i) {
      s.x += red[i][lane].x;
      s.y += red[i][lane].y;
      s.z += red[i][lane].z;
      s.w += red[i][lane].w;
    }
    dw[c] = Cvt<W>::from_f(s.x);
    dw[c + 1] = Cvt<W>::from_f(s.y);
    dw[c + 2] = Cvt<W>::from_f(s.z);
    dw[c + 3] = Cvt<W>::from_f(s.w);
  }
}

// dw[c] = sum over the G partial rows, fixed order: 8 warps split the rows,
// lanes own columns, then the warps' sums are added in warp order.
template <typename W>
__global__ void __launch_bounds__(256) rms_dw_reduce_kernel(const float* __restrict__ partial, int g,
                                                            int cols, W* __restrict__ dw) {
  __shared__ float red[8][33];
  pdl_wait();
  pdl_trigger();
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
// Vectors per thread for the row kernels: the smallest VPT in {1, 2, 4}
// that keeps the CTA at <= 512 threads; 0 (generic path) when the row is
// longer than 2048 vectors.
template <typename T>
int vpt_for(int64_t cols) {
  const int64_t nvec = cols / Vec16<T>::N;
  for (int v : {1, 2, 4})
    if ((nvec + v - 1) / v <= 512) return v;
  return 0;
}

template <typename T>
int row_threads(int64_t cols, int vpt) {
  const int64_t nvec = cols / Vec16<T>::N;
  const int64_t t = (nvec + vpt - 1) / vpt;
  return static_cast<int>((t + 31) / 32 * 32);
}

template <typename T, typename W>
bool vec_ok(int64_t cols, std::initializer_list<std::pair<const void*, int64_t>> mats, const void* w) {
  if (cols % Vec16<T>::N) return false;
  if (!aligned16(w)) return false;
  for (auto& m : mats)
    if (!aligned16(m.first) || ((m.second * (int64_t)sizeof(T)) % 16) != 0) return false;
  return vpt_for<T>(cols) > 0;
}

// Resident CTAs per SM of a kernel at this block size / shared memory (cached).
template <typename K>
int ctas_per_sm(K kernel, int threads, size_t smem) {
  struct Entry {
    const void* k;
    int threads;
    size_t smem;
    int dev;
    int n;
  };
  static Entry cache[64];
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(cache_mutex());
  for (int i = 0; i < used; ++i)
    if (cache[i].k == (const void*)kernel && cache[i].threads == threads && cache[i].smem == smem &&
        cache[i].dev == dev)
      return cache[i].n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1)
    n = 1;
  if (used < 64) cache[used++] = Entry{(const void*)kernel, threads, smem, dev, n};
  return n;
}

template <typename T, typename W, int VPT>
int fwd_rows_launch(const T* X, int64_t xs, const W* Wt, T* Y, int64_t ys, float* rstd, int64_t rows,
                    int cols, float eps, cudaStream_t st) {
  const int threads = row_threads<T>(cols, VPT);
  auto k = rms_fwd_rows<T, W, VPT>;
  const int64_t cap = (int64_t)num_sms() * ctas_per_sm(k, threads, 0);
  const int grid = static_cast<int>(rows < cap ? rows : cap);
  return cuda_status(launch_pdl(k, dim3(grid), dim3(threads), 0, st, X, xs, Wt, Y, ys, rstd, rows,
                                cols, eps));
}

template <typename T, typename W>
int fwd_impl(const void* x, int64_t xs, const void* w, void* y, int64_t ys, float* rstd,
             int64_t rows, int64_t cols, float eps, cudaStream_t st) {
  const T* X = static_cast<const T*>(x);
  const W* Wt = static_cast<const W*>(w);
  T* Y = static_cast<T*>(y);
  if (vec_ok<T, W>(cols, {{x, xs}, {y, ys}}, w)) {
    switch (vpt_for<T>(cols)) {
      case 1: return fwd_rows_launch<T, W, 1>(X, xs, Wt, Y, ys, rstd, rows, (int)cols, eps, st);
      case 2: return fwd_rows_launch<T, W, 2>(X, xs, Wt, Y, ys, rstd, rows, (int)cols, eps, st);
      default: return fwd_rows_launch<T, W, 4>(X, xs, Wt, Y, ys, rstd, rows, (int)cols, eps, st);
    }
  }
  const unsigned grid = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
  rms_fwd_generic<T, W><<<grid, kWarps * 32, 0, st>>>(X, xs, Wt, Y, ys, rstd, rows, (int)cols, eps);
  return launch_status();
}

// Grid of the generic backward (one dw partial row per warp).
int bwd_grid(int64_t rows) {
  int64_t g = (rows + kWarps - 1) / kWarps;
  const int64_t cap = num_sms();
  return static_cast<int>(g < cap ? g : cap);
}

// Grid of the vector backward with dw: at most 3 CTAs per SM (bounds the
// partial rows: at most 3 x #SMs rows of cols floats).
template <typename T, typename W, int VPT>
int bwd_rows_grid(int64_t rows, int cols) {
  const int threads = row_threads<T>(cols, VPT);
  auto k = rms_bwd_rows<T, W, VPT, true>;
  int per_sm = ctas_per_sm(k, threads, 0);
  if (per_sm > 3) per_sm = 3;
  const int64_t cap = (int64_t)num_sms() * per_sm;
  return static_cast<int>(rows < cap ? rows : cap);
}

template <typename T, typename W, int VPT>
int bwd_rows_launch(const T* DY, int64_t dys, const T* X, int64_t xs, const W* Wt, const float* rstd,
                    T* DX, int64_t dxs, W* dw, void* ws, size_t ws_bytes, int64_t rows, int cols,
                    cudaStream_t st) {
  const int threads = row_threads<T>(cols, VPT);
  if (!dw) {
    auto k = rms_bwd_rows<T, W, VPT, false>;
    const int64_t cap = (int64_t)num_sms() * ctas_per_sm(k, threads, 0);
    const int grid = static_cast<int>(rows < cap ? rows : cap);
    return cuda_status(launch_pdl(k, dim3(grid), dim3(threads), 0, st, DY, dys, X, xs, Wt, rstd, DX,
                                  dxs, static_cast<float*>(nullptr), rows, cols));
  }
  const int grid = bwd_rows_grid<T, W, VPT>(rows, cols);
  if (!ws || ws_bytes < (size_t)grid * cols * sizeof(float) || !aligned16(ws)) {
    set_last_error("soup_rmsnorm_bwd: workspace too small");
    return SOUP_ERR_WORKSPACE;
  }
  float* partial = static_cast<float*>(ws);
  int rc = cuda_status(launch_pdl(rms_bwd_rows<T, W, VPT, true>, dim3(grid), dim3(threads), 0, st, DY,
                                  dys, X, xs, Wt, rstd, DX, dxs, partial, rows, cols));
  if (rc) return rc;
  return cuda_status(launch_pdl(rms_dw_reduce_vec<W>, dim3((unsigned)((cols + 127) / 128)), dim3(1024),
                                0, st, static_cast<const float*>(partial), grid, cols, dw));
}

template <typename T, typename W>
int bwd_impl(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
             const float* rstd, void* dx, int64_t dxs, void* dw, void* ws, size_t ws_bytes,
             int64_t rows, int64_t cols, cudaStream_t st) {
  const T* DY = static_cast<const T*>(dy);
  const T* X = static_cast<const T*>(x);
  const W* Wt = static_cast<const W*>(w);
  T* DX = static_cast<T*>(dx);
  W* DW = static_cast<W*>(dw);
  if (vec_ok<T, W>(cols, {{dy, dys}, {x, xs}, {dx, dxs}}, w)) {
    const int c = static_cast<int>(cols);
    switch (vpt_for<T>(cols)) {
      case 1: return bwd_rows_launch<T, W, 1>(DY, dys, X, xs, Wt, rstd, DX, dxs, DW, ws, ws_bytes, rows, c, st);
      case 2: return bwd_rows_launch<T, W, 2>(DY, dys, X, xs, Wt, rstd, DX, dxs, DW, ws, ws_bytes, rows, c, st);
      default: return bwd_rows_launch<T, W, 4>(DY, dys, X, xs, Wt, rstd, DX, dxs, DW, ws, ws_bytes, rows, c, st);
    }
  }
  // generic path: one partial row per warp
  const int grid = bwd_grid(rows);
  const int prows = grid * kWarps;
  float* partial = nullptr;
  if (dw) {
    if (!ws || ws_bytes < (size_t)prows * cols * sizeof(float) || !aligned16(ws)) {
      set_last_error("soup_rmsnorm_bwd: workspace too small");
      return SOUP_ERR_WORKSPACE;
    }
    partial = static_cast<float*>(ws);
  }
  rms_bwd_generic<T, W><<<grid, kWarps * 32, 0, st>>>(DY, dys, X, xs, Wt, rstd, DX, dxs, partial,
                                                      rows, (int)cols);
  int rc = launch_status();
  if (rc || !dw) return rc;
  rms_dw_reduce_kernel<W><<<(unsigned)((cols + 31) / 32), 256, 0, st>>>(partial, prows, (int)cols, DW);
  return launch_status();
}

// Bytes of dw partial rows the backward writes for these operands.
template <typename T, typename W>
size_t bwd_partial_rows(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
                        const void* dx, int64_t dxs, int64_t rows, int64_t cols) {
  if (vec_ok<T, W>(cols, {{dy, dys}, {x, xs}, {dx, dxs}}, w)) {
    switch (vpt_for<T>(cols)) {
      case 1: return bwd_rows_grid<T, W, 1>(rows, (int)cols);
      case 2: return bwd_rows_grid<T, W, 2>(rows, (int)cols);
      default: return bwd_rows_grid<T, W, 4>(rows, (int)cols);
    }
  }
  return static_cast<size_t>(bwd_grid(rows)) * kWarps;
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
  // upper bound: the generic path keeps one partial row per warp; the vector
  // path one per CTA (at most 3 per SM)
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
// current (under the library's cache lock, so concurrent first calls from
// several host threads are safe). In host code the array's name is only a
// host-side stand-in, so the kernels must receive this address instead. The
// cached address is not refreshed after cudaDeviceReset: a process that resets
// a device must not call this entry point on it again.
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
  std::lock_guard<std::mutex> lock(cache_mutex());
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

template <typename T, typename W>
size_t bwd_partial_bytes(const void* dy, int64_t dys, const void* x, int64_t xs, const void* w,
                         const void* dx, int64_t dxs, int64_t rows, int64_t cols) {
  return bwd_partial_rows<T, W>(dy, dys, x, xs, w, dx, dxs, rows, cols) *
         static_cast<size_t>(cols) * sizeof(float);
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
