// Cross-entropy with online metrics over an existing logits buffer, with the
// in-place gradient: the drop-in for the reference's
// _chunked_cross_entropy_fused_kernel (solution/kernels/chunked_ce.py:32-128).
//
// One CTA per row. Pass 1: every thread keeps an online-softmax state over
// its 16-byte vectors (vector max first, one rescale, then one exp per
// element), the CTA merges the states (ties keep the smaller index) and
// writes loss / entropy / hit. Pass 2 (optional) rewrites the row in place as
// (softmax - onehot) / denominator, or zeros for an ignored row.
#include "soup_common.cuh"

namespace soup {
namespace {

template <typename T, bool VEC>
__global__ void __launch_bounds__(512) ce_rows_kernel(T* __restrict__ logits, int64_t ld,
                                                      const int64_t* __restrict__ targets,
                                                      float* __restrict__ losses,
                                                      float* __restrict__ entropies,
                                                      int32_t* __restrict__ correct, int64_t vocab,
                                                      float inv_den, int64_t ignore_index,
                                                      int write_grad) {
  constexpr int NE = VEC ? Vec16<T>::N : 1;
  const int64_t row = blockIdx.x;
  T* z = logits + row * ld;
  SoftmaxState st = sm_init();
  const int64_t nv = vocab / NE;
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
    float v[NE];
    if constexpr (VEC) {
      Vec16<T> r = ld16(z + i * NE);
#pragma unroll
      for (int j = 0; j < NE; ++j) v[j] = Cvt<T>::to_f(r.v[j]);
    } else {
      v[0] = Cvt<T>::to_f(z[i]);
    }
    float vm = v[0];
    int vi = 0;
#pragma unroll
    for (int j = 1; j < NE; ++j)
      if (v[j] > vm) {
        vm = v[j];
        vi = j;
      }
    if (vm > st.m) {
      const float f = fast_exp2((st.m - vm) * kLog2e);
      st.s *= f;
      st.w *= f;
      st.m = vm;
      st.idx = static_cast<int>(i * NE + vi);
    }
    const float mb = st.m * kLog2e;
#pragma unroll
    for (int j = 0; j < NE; ++j) {
      const float e = fast_exp2(fmaf(v[j], kLog2e, -mb));
      st.s += e;
      st.w = fmaf(v[j], e, st.w);
    }
  }
  // ragged tail (vector path only)
  for (int64_t c = nv * NE + threadIdx.x; c < vocab; c += blockDim.x) {
    SoftmaxState b{Cvt<T>::to_f(z[c]), 1.f, Cvt<T>::to_f(z[c]), static_cast<int>(c)};
    st = sm_merge(st, b);
  }
  st = sm_warp_reduce(st);
  __shared__ SoftmaxState red[16];
  __shared__ float s_lse;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = st;
  __syncthreads();
  const int64_t t = targets[row];
  const bool ignored = t == ignore_index;
  if (threadIdx.x == 0) {
    SoftmaxState r = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = sm_merge(r, red[i]);
    const float safe_s = fmaxf(r.s, 1e-12f);
    const float lse = r.m + logf(safe_s);
    const bool in_range = t >= 0 && t < vocab;
    const float zt = in_range ? Cvt<T>::to_f(z[t]) : 0.f;
    losses[row] = ignored ? 0.f : lse - zt;
    entropies[row] = fmaxf(0.f, lse - r.w / safe_s);
    correct[row] = (!ignored && in_range && r.idx == static_cast<int>(t)) ? 1 : 0;
    s_lse = lse;
  }
  if (!write_grad) return;
  __syncthreads();
  const float lb = s_lse * kLog2e;
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
    if constexpr (VEC) {
      Vec16<T> r = ld16(z + i * NE), o;
#pragma unroll
      for (int j = 0; j < NE; ++j) {
        float g = 0.f;
        if (!ignored) {
          float p = fast_exp2(fmaf(Cvt<T>::to_f(r.v[j]), kLog2e, -lb));
          if (i * NE + j == t) p -= 1.f;
          g = p * inv_den;
        }
        o.v[j] = Cvt<T>::from_f(g);
      }
      st16(z + i * NE, o);
    } else {
      float g = 0.f;
      if (!ignored) {
        float p = fast_exp2(fmaf(Cvt<T>::to_f(z[i]), kLog2e, -lb));
        if (i == t) p -= 1.f;
        g = p * inv_den;
      }
      z[i] = Cvt<T>::from_f(g);
    }
  }
  for (int64_t c = nv * NE + threadIdx.x; c < vocab; c += blockDim.x) {
    float g = 0.f;
    if (!ignored) {
      float p = fast_exp2(fmaf(Cvt<T>::to_f(z[c]), kLog2e, -lb));
      if (c == t) p -= 1.f;
      g = p * inv_den;
    }
    z[c] = Cvt<T>::from_f(g);
  }
}

template <typename T>
int ce_rows_run(void* logits, int64_t ld, const int64_t* targets, float* losses, float* ents,
                int32_t* corr, int64_t rows, int64_t vocab, float den, int64_t ignore_index,
                int write_grad, cudaStream_t st) {
  const bool vec = aligned16(logits) && ((ld * (int64_t)sizeof(T)) % 16 == 0);
  const float inv_den = 1.f / den;
  T* L = static_cast<T*>(logits);
  if (vec)
    ce_rows_kernel<T, true><<<(unsigned)rows, 512, 0, st>>>(L, ld, targets, losses, ents, corr, vocab,
                                                            inv_den, ignore_index, write_grad);
  else
    ce_rows_kernel<T, false><<<(unsigned)rows, 512, 0, st>>>(L, ld, targets, losses, ents, corr, vocab,
                                                             inv_den, ignore_index, write_grad);
  return launch_status();
}

}  // namespace
}  // namespace soup

using namespace soup;

extern "C" {

int soup_ce_rows(void* logits, int64_t row_stride, const int64_t* targets, float* losses,
                 float* entropies, int32_t* correct, int64_t rows, int64_t vocab,
                 float denominator, int64_t ignore_index, int dtype, int write_grad,
                 void* stream) {
  if (!logits || !targets || !losses || !entropies || !correct || rows < 0 || vocab <= 0 ||
      vocab >= (int64_t(1) << 31) || row_stride < vocab || rows >= (int64_t(1) << 31)) {
    set_last_error("soup_ce_rows: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (rows == 0) return SOUP_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == SOUP_F16)
    return ce_rows_run<__half>(logits, row_stride, targets, losses, entropies, correct, rows, vocab,
                               denominator, ignore_index, write_grad, st);
  if (dtype == SOUP_BF16)
    return ce_rows_run<__nv_bfloat16>(logits, row_stride, targets, losses, entropies, correct, rows,
                                      vocab, denominator, ignore_index, write_grad, st);
  if (dtype == SOUP_F32)
    return ce_rows_run<float>(logits, row_stride, targets, losses, entropies, correct, rows, vocab,
                              denominator, ignore_index, write_grad, st);
  set_last_error("soup_ce_rows: unsupported dtype");
  return SOUP_ERR_INVALID;
}

}  // extern "C"
