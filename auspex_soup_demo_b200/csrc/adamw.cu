// AdamW update of the QLoRA step's flat LoRA buffers in one pass.
//
// The trainable LoRA factors, their gradients and both moment estimates live
// in flat fp32 buffers of n elements. One launch reads param, grad, m and v
// once and writes param, m, v and (optionally) the 16-bit copy of the
// parameters that the step's GEMMs read, instead of a multi-tensor optimiser
// plus separate cast kernels. Per element, torch.optim.AdamW's decoupled
// weight-decay form (the optimiser of the HF Trainer that the reference's
// `soup train` runs, task/task.yaml:10-22):
//   p  = p * (1 - lr * weight_decay)
//   m  = m + (1 - beta1) * (g - m)
//   v  = beta2 * v + (1 - beta2) * g * g
//   p  = p - lr / (1 - beta1^t) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
// t is read from a device scalar (the step count including this update), so
// the launch can be recorded once in a CUDA graph and replayed.
#include "soup_common.cuh"

namespace soup {
namespace {

struct AdamHyper {
  float lr, beta1, beta2, eps, wd;
};

template <typename H>
__device__ __forceinline__ void store4_16(H* dst, float a, float b, float c, float d) {
  union {
    uint2 u;
    H h[4];
  } o;
  o.h[0] = Cvt<H>::from_f(a);
  o.h[1] = Cvt<H>::from_f(b);
  o.h[2] = Cvt<H>::from_f(c);
  o.h[3] = Cvt<H>::from_f(d);
  *reinterpret_cast<uint2*>(dst) = o.u;
}

__device__ __forceinline__ float adam_one(float& p, float g, float& m, float& v, const AdamHyper& h,
                                          float step_size, float inv_sqrt_bc2) {
  p *= 1.f - h.lr * h.wd;
  m = fmaf(1.f - h.beta1, g - m, m);
  v = fmaf((1.f - h.beta2) * g, g, v * h.beta2);
  p -= step_size * m / (sqrtf(v) * inv_sqrt_bc2 + h.eps);
  return p;
}

// Vector path: float4 accesses (n % 4 == 0, 16-byte aligned buffers).
template <typename H>
__global__ void __launch_bounds__(256) adamw_flat_kernel(float4* __restrict__ param,
                                                         const float4* __restrict__ grad,
                                                         float4* __restrict__ m4,
                                                         float4* __restrict__ v4, int64_t n4,
                                                         const float* __restrict__ step,
                                                         AdamHyper h, H* __restrict__ p16,
                                                         int64_t n_scaled, float scale) {
  pdl_wait();
  pdl_trigger();
  const float t = *step;
  const float bc1 = 1.f - powf(h.beta1, t);
  const float bc2 = 1.f - powf(h.beta2, t);
  const float step_size = h.lr / bc1;
  const float inv_sqrt_bc2 = 1.f / sqrtf(bc2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 p = param[i];
    const float4 g = __ldcs(grad + i);
    float4 m = m4[i], v = v4[i];
    adam_one(p.x, g.x, m.x, v.x, h, step_size, inv_sqrt_bc2);
    adam_one(p.y, g.y, m.y, v.y, h, step_size, inv_sqrt_bc2);
    adam_one(p.z, g.z, m.z, v.z, h, step_size, inv_sqrt_bc2);
    adam_one(p.w, g.w, m.w, v.w, h, step_size, inv_sqrt_bc2);
    param[i] = p;
    m4[i] = m;
    v4[i] = v;
    if (p16) {
      const float s = (i * 4 < n_scaled) ? scale : 1.f;  // n_scaled % 4 == 0
      store4_16(p16 + i * 4, s * p.x, s * p.y, s * p.z, s * p.w);
    }
  }
}

// Scalar path (any length / alignment).
template <typename H>
__global__ void __launch_bounds__(256) adamw_flat_scalar(float* __restrict__ param,
                                                         const float* __restrict__ grad,
                                                         float* __restrict__ m,
                                                         float* __restrict__ v, int64_t n,
                                                         const float* __restrict__ step,
                                                         AdamHyper h, H* __restrict__ p16,
                                                         int64_t n_scaled, float scale) {
  pdl_wait();
  pdl_trigger();
  const float t = *step;
  const float step_size = h.lr / (1.f - powf(h.beta1, t));
  const float inv_sqrt_bc2 = 1.f / sqrtf(1.f - powf(h.beta2, t));
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float p = param[i], mm = m[i], vv = v[i];
    adam_one(p, grad[i], mm, vv, h, step_size, inv_sqrt_bc2);
    param[i] = p;
    m[i] = mm;
    v[i] = vv;
    if (p16) p16[i] = Cvt<H>::from_f(i < n_scaled ? scale * p : p);
  }
}

template <typename H>
int adamw_run(float* param, const float* grad, float* m, float* v, int64_t n, const float* step,
              const AdamHyper& h, void* p16v, int64_t n_scaled, float scale, cudaStream_t st) {
  H* p16 = static_cast<H*>(p16v);
  const bool vec = (n % 4) == 0 && (n_scaled % 4) == 0 && aligned16(param) && aligned16(grad) &&
                   aligned16(m) && aligned16(v) &&
                   (p16 == nullptr || (reinterpret_cast<uintptr_t>(p16) & 7) == 0);
  const int64_t work = vec ? n / 4 : n;
  int64_t grid = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  cudaError_t e;
  if (vec)
    e = launch_pdl(adamw_flat_kernel<H>, dim3((unsigned)grid), dim3(256), 0, st,
                   reinterpret_cast<float4*>(param), reinterpret_cast<const float4*>(grad),
                   reinterpret_cast<float4*>(m), reinterpret_cast<float4*>(v), work, step, h, p16,
                   n_scaled, scale);
  else
    e = launch_pdl(adamw_flat_scalar<H>, dim3((unsigned)grid), dim3(256), 0, st, param, grad, m, v,
                   n, step, h, p16, n_scaled, scale);
  return cuda_status(e);
}

}  // namespace
}  // namespace soup

using namespace soup;

extern "C" {

int soup_adamw_flat(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n,
                    const float* step, float lr, float beta1, float beta2, float eps,
                    float weight_decay, void* param16, int param16_dtype, int64_t n_scaled,
                    float scale, void* stream) {
  if (!param || !grad || !exp_avg || !exp_avg_sq || !step || n <= 0 || n_scaled < 0 ||
      n_scaled > n || !(beta1 >= 0.f && beta1 < 1.f) || !(beta2 >= 0.f && beta2 < 1.f) ||
      !(eps > 0.f)) {
    set_last_error("soup_adamw_flat: bad arguments");
    return SOUP_ERR_INVALID;
  }
  AdamHyper h{lr, beta1, beta2, eps, weight_decay};
  cudaStream_t st = as_stream(stream);
  if (!param16 || param16_dtype == SOUP_BF16)
    return adamw_run<__nv_bfloat16>(param, grad, exp_avg, exp_avg_sq, n, step, h, param16, n_scaled,
                                    scale, st);
  if (param16_dtype == SOUP_F16)
    return adamw_run<__half>(param, grad, exp_avg, exp_avg_sq, n, step, h, param16, n_scaled, scale,
                             st);
  set_last_error("soup_adamw_flat: param16 dtype must be BF16 or F16");
  return SOUP_ERR_INVALID;
}

}  // extern "C"
