// SwiGLU forward out = g*sigmoid(g)*u and its backward with sigmoid
// recomputed from g (solution/kernels/swiglu.py:20-50 and :53-95).
//
// Grid-stride over 16-byte vectors (8 bf16/fp16 or 4 fp32 per thread step),
// streaming loads/stores; the grid is a multiple of the SM count. Rows may
// have independent strides (gate/up can be column slices of one fused
// projection); fully contiguous operands take a flat 1-D walk.
#include "soup_common.cuh"

namespace soup {
namespace {

template <typename T>
struct FwdOp {
  static constexpr int kIn = 2, kOut = 1;
  __device__ __forceinline__ static void apply(const float (&in)[kIn], float (&out)[kOut]) {
    out[0] = swiglu_fwd_f(in[0], in[1]);
  }
};

template <typename T>
struct BwdOp {
  static constexpr int kIn = 3, kOut = 2;  // (dy, g, u) -> (dg, du)
  __device__ __forceinline__ static void apply(const float (&in)[kIn], float (&out)[kOut]) {
    swiglu_bwd_f(in[0], in[1], in[2], out[0], out[1]);
  }
};

template <typename T, int NI, int NO>
struct Ptrs {
  const T* in[NI];
  int64_t in_ld[NI];
  T* out[NO];
  int64_t out_ld[NO];
};

// Vector path: every row start 16-byte aligned, cols % NE == 0.
template <typename T, class Op>
__global__ void __launch_bounds__(256) ew_vec_kernel(Ptrs<T, Op::kIn, Op::kOut> p, int64_t rows,
                                                     int64_t cols, int flat) {
  constexpr int NE = Vec16<T>::N;
  pdl_wait();
  pdl_trigger();
  const int64_t vpr = cols / NE;
  const int64_t total = rows * vpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r, c;
    if (flat) {
      r = 0;
      c = i * NE;
    } else {
      r = i / vpr;
      c = (i - r * vpr) * NE;
    }
    Vec16<T> in[Op::kIn];
#pragma unroll
    for (int k = 0; k < Op::kIn; ++k) in[k] = ld16_stream(p.in[k] + r * p.in_ld[k] + c);
    Vec16<T> out[Op::kOut];
#pragma unroll
    for (int j = 0; j < NE; ++j) {
      float a[Op::kIn], b[Op::kOut];
#pragma unroll
      for (int k = 0; k < Op::kIn; ++k) a[k] = Cvt<T>::to_f(in[k].v[j]);
      Op::apply(a, b);
#pragma unroll
      for (int k = 0; k < Op::kOut; ++k) out[k].v[j] = Cvt<T>::from_f(b[k]);
    }
#pragma unroll
    for (int k = 0; k < Op::kOut; ++k) st16_stream(p.out[k] + r * p.out_ld[k] + c, out[k]);
  }
}

// Scalar path for ragged or misaligned operands.
template <typename T, class Op>
__global__ void __launch_bounds__(256) ew_scalar_kernel(Ptrs<T, Op::kIn, Op::kOut> p, int64_t rows,
                                                        int64_t cols) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    float a[Op::kIn], b[Op::kOut];
#pragma unroll
    for (int k = 0; k < Op::kIn; ++k) a[k] = Cvt<T>::to_f(p.in[k][r * p.in_ld[k] + c]);
    Op::apply(a, b);
#pragma unroll
    for (int k = 0; k < Op::kOut; ++k) p.out[k][r * p.out_ld[k] + c] = Cvt<T>::from_f(b[k]);
  }
}

template <typename T, class Op>
int run(const Ptrs<T, Op::kIn, Op::kOut>& p, int64_t rows, int64_t cols, cudaStream_t st) {
  constexpr int NE = Vec16<T>::N;
  bool vec = (cols % NE) == 0;
  bool flat = true;
  for (int k = 0; k < Op::kIn; ++k) {
    vec = vec && aligned16(p.in[k]) && ((p.in_ld[k] * (int64_t)sizeof(T)) % 16 == 0);
    flat = flat && (p.in_ld[k] == cols || rows == 1);
  }
  for (int k = 0; k < Op::kOut; ++k) {
    vec = vec && aligned16(p.out[k]) && ((p.out_ld[k] * (int64_t)sizeof(T)) % 16 == 0);
    flat = flat && (p.out_ld[k] == cols || rows == 1);
  }
  const int64_t work = vec ? rows * cols / NE : rows * cols;
  const int64_t per_wave = (int64_t)num_sms() * 8 * 256;  // 8 resident CTAs of 256 per SM
  int64_t blocks = (work + 255) / 256;
  if (blocks > per_wave / 256) blocks = per_wave / 256;
  if (blocks < 1) blocks = 1;
  if (vec) {
    Ptrs<T, Op::kIn, Op::kOut> q = p;
    // flat: one row of rows*cols elements
    return cuda_status(launch_pdl(ew_vec_kernel<T, Op>, dim3((unsigned)blocks), dim3(256), 0, st, q,
                                  flat ? int64_t(1) : rows, flat ? rows * cols : cols, flat ? 1 : 0));
  } else {
    ew_scalar_kernel<T, Op><<<(unsigned)blocks, 256, 0, st>>>(p, rows, cols);
  }
  return launch_status();
}

}  // namespace
}  // namespace soup

using namespace soup;

extern "C" {

int soup_swiglu_fwd(const void* gate, int64_t gate_row_stride, const void* up,
                    int64_t up_row_stride, void* out, int64_t out_row_stride, int64_t rows,
                    int64_t cols, int dtype, void* stream) {
  if (!gate || !up || !out || rows < 0 || cols <= 0 || gate_row_stride < cols ||
      up_row_stride < cols || out_row_stride < cols) {
    set_last_error("soup_swiglu_fwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  cudaStream_t st = as_stream(stream);
#define RUN(T)                                                                               \
  do {                                                                                       \
    Ptrs<T, 2, 1> p{{static_cast<const T*>(gate), static_cast<const T*>(up)},                \
                    {gate_row_stride, up_row_stride},                                        \
                    {static_cast<T*>(out)},                                                  \
                    {out_row_stride}};                                                       \
    return run<T, FwdOp<T>>(p, rows, cols, st);                                              \
  } while (0)
  if (dtype == SOUP_BF16) RUN(__nv_bfloat16);
  if (dtype == SOUP_F16) RUN(__half);
  if (dtype == SOUP_F32) RUN(float);
#undef RUN
  set_last_error("soup_swiglu_fwd: unsupported dtype");
  return SOUP_ERR_INVALID;
}

int soup_swiglu_bwd(const void* dy, int64_t dy_row_stride, const void* gate,
                    int64_t gate_row_stride, const void* up, int64_t up_row_stride, void* dgate,
                    int64_t dgate_row_stride, void* dup, int64_t dup_row_stride, int64_t rows,
                    int64_t cols, int dtype, void* stream) {
  if (!dy || !gate || !up || !dgate || !dup || rows < 0 || cols <= 0 || dy_row_stride < cols ||
      gate_row_stride < cols || up_row_stride < cols || dgate_row_stride < cols ||
      dup_row_stride < cols) {
    set_last_error("soup_swiglu_bwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  cudaStream_t st = as_stream(stream);
#define RUN(T)                                                                               \
  do {                                                                                       \
    Ptrs<T, 3, 2> p{{static_cast<const T*>(dy), static_cast<const T*>(gate),                 \
                     static_cast<const T*>(up)},                                             \
                    {dy_row_stride, gate_row_stride, up_row_stride},                         \
                    {static_cast<T*>(dgate), static_cast<T*>(dup)},                          \
                    {dgate_row_stride, dup_row_stride}};                                     \
    return run<T, BwdOp<T>>(p, rows, cols, st);                                              \
  } while (0)
  if (dtype == SOUP_BF16) RUN(__nv_bfloat16);
  if (dtype == SOUP_F16) RUN(__half);
  if (dtype == SOUP_F32) RUN(float);
#undef RUN
  set_last_error("soup_swiglu_bwd: unsupported dtype");
  return SOUP_ERR_INVALID;
}

}  // extern "C"
