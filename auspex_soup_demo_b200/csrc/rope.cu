// Rotate-half RoPE on Q and K in one launch (forward and inverse).
//
// Forward (solution/kernels/rope.py:52-67):  y1 = x1*c - x2*s, y2 = x1*s + x2*c
// Inverse (rope.py:102-117):                 dx1 = g1*c + g2*s, dx2 = g2*c - g1*s
// with x1 = x[..., :D/2], x2 = x[..., D/2:] and c, s the first D/2 entries of
// the cos/sin row of (batch, position) -- the reference kernel reads only that
// half, which equals the second half for tables built as cat(freqs, freqs).
//
// One thread handles NE consecutive pairs (a 16-byte vector of x1 and the
// matching vector of x2); 8 (bf16) or 16 (fp32) consecutive threads cover one
// (b, h, s) row of head_dim 128, so loads and stores are coalesced. Q items
// come first in the flat index space, then K.
#include "soup_common.cuh"

namespace soup {
namespace {

struct RopeTensor {
  const void* x;
  void* out;
  int64_t sb, sh, ss;     // input strides (elements)
  int64_t ob, oh, os;     // output strides
  int64_t heads;
};

// Vector path: CTA (blockIdx.x, blockIdx.y) covers positions
// [blockIdx.x * P, +P) of batch blockIdx.y for every head of Q and K; thread
// slot i = (head, 16-byte chunk) is fixed, so addresses are computed once and
// the loads of all P positions are in flight together.
template <typename T, typename CT, int P>
__global__ void __launch_bounds__(256) rope_rows_kernel(RopeTensor q, RopeTensor k,
                                                        const CT* __restrict__ cos,
                                                        const CT* __restrict__ sin, int64_t cb,
                                                        int64_t cs, int S, int half, float sign) {
  constexpr int NE = Vec16<T>::N;
  pdl_wait();
  pdl_trigger();
  const int chunks = half / NE;
  const int slots = static_cast<int>(q.heads + k.heads) * chunks;
  const int64_t b = blockIdx.y;
  const int s0 = blockIdx.x * P;
  for (int i = threadIdx.x; i < slots; i += blockDim.x) {
    const int h = i / chunks;
    const int d = (i - h * chunks) * NE;
    const bool isq = h < q.heads;
    const RopeTensor& t = isq ? q : k;
    const int64_t hh = isq ? h : h - q.heads;
    const T* xb = static_cast<const T*>(t.x) + b * t.sb + hh * t.sh + d;
    T* ob = static_cast<T*>(t.out) + b * t.ob + hh * t.oh + d;
    const CT* cbp = cos + b * cb + d;
    const CT* sbp = sin + b * cb + d;
    Vec16<T> x1[P], x2[P];
    if constexpr (sizeof(CT) == sizeof(T)) {
      // cos/sin rows stay packed until use (fewer registers, more CTAs per SM)
      Vec16<CT> cv[P], sv[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int s = s0 + p;
        if (s < S) {
          x1[p] = ld16_stream(xb + s * t.ss);
          x2[p] = ld16_stream(xb + s * t.ss + half);
          cv[p] = ld16(cbp + s * cs);
          sv[p] = ld16(sbp + s * cs);
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int s = s0 + p;
        if (s < S) {
          Vec16<T> y1, y2;
#pragma unroll
          for (int e = 0; e < NE; ++e) {
            const float a = Cvt<T>::to_f(x1[p].v[e]), bb = Cvt<T>::to_f(x2[p].v[e]);
            const float c = Cvt<CT>::to_f(cv[p].v[e]), sn = sign * Cvt<CT>::to_f(sv[p].v[e]);
            y1.v[e] = Cvt<T>::from_f(a * c - bb * sn);
            y2.v[e] = Cvt<T>::from_f(a * sn + bb * c);
          }
          st16_stream(ob + s * t.os, y1);
          st16_stream(ob + s * t.os + half, y2);
        }
      }
    } else {
      float c[P][NE], sn[P][NE];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int s = s0 + p;
        if (s < S) {
          x1[p] = ld16_stream(xb + s * t.ss);
          x2[p] = ld16_stream(xb + s * t.ss + half);
#pragma unroll
          for (int e = 0; e < NE; ++e) {
            c[p][e] = Cvt<CT>::to_f(cbp[s * cs + e]);
            sn[p][e] = sign * Cvt<CT>::to_f(sbp[s * cs + e]);
          }
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int s = s0 + p;
        if (s < S) {
          Vec16<T> y1, y2;
#pragma unroll
          for (int e = 0; e < NE; ++e) {
            const float a = Cvt<T>::to_f(x1[p].v[e]), bb = Cvt<T>::to_f(x2[p].v[e]);
            y1.v[e] = Cvt<T>::from_f(a * c[p][e] - bb * sn[p][e]);
            y2.v[e] = Cvt<T>::from_f(a * sn[p][e] + bb * c[p][e]);
          }
          st16_stream(ob + s * t.os, y1);
          st16_stream(ob + s * t.os + half, y2);
        }
      }
    }
  }
}

// Scalar path (any alignment): one pair per thread-iteration.
template <typename T, typename CT>
__global__ void __launch_bounds__(256) rope_scalar_kernel(RopeTensor q, RopeTensor k,
                                                          const CT* __restrict__ cos,
                                                          const CT* __restrict__ sin, int64_t cb,
                                                          int64_t cs, int64_t S, int64_t half,
                                                          float sign) {
  pdl_wait();
  pdl_trigger();
  const int64_t nq = q.heads * S * half;
  const int64_t per_b = nq + k.heads * S * half;
  const int64_t b = blockIdx.y;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_b;
       i += (int64_t)gridDim.x * blockDim.x) {
    const bool isq = i < nq;
    const RopeTensor& t = isq ? q : k;
    int64_t j = isq ? i : i - nq;
    const int64_t d = j % half;
    j /= half;
    const int64_t s = j % S;
    const int64_t h = j / S;
    const T* xp = static_cast<const T*>(t.x) + b * t.sb + h * t.sh + s * t.ss + d;
    T* op = static_cast<T*>(t.out) + b * t.ob + h * t.oh + s * t.os + d;
    const float c = Cvt<CT>::to_f(cos[b * cb + s * cs + d]);
    const float sn = sign * Cvt<CT>::to_f(sin[b * cb + s * cs + d]);
    const float a = Cvt<T>::to_f(xp[0]), bb = Cvt<T>::to_f(xp[half]);
    op[0] = Cvt<T>::from_f(a * c - bb * sn);
    op[half] = Cvt<T>::from_f(a * sn + bb * c);
  }
}

template <typename T, typename CT>
int rope_run(const RopeTensor& q, const RopeTensor& k, const void* cos, const void* sin, int64_t cb,
             int64_t cs, int64_t B, int64_t S, int64_t D, float sign, cudaStream_t st) {
  const int64_t half = D / 2;
  constexpr int NE = Vec16<T>::N;
  auto ok_t = [&](const RopeTensor& t) {
    if (t.heads == 0) return true;
    const int64_t es = sizeof(T);
    return aligned16(t.x) && aligned16(t.out) && (t.sb * es) % 16 == 0 && (t.sh * es) % 16 == 0 &&
           (t.ss * es) % 16 == 0 && (t.ob * es) % 16 == 0 && (t.oh * es) % 16 == 0 &&
           (t.os * es) % 16 == 0;
  };
  const int64_t ces = sizeof(CT);
  bool vec = (half % NE) == 0 && ok_t(q) && ok_t(k) && S < (int64_t(1) << 31);
  if (vec && sizeof(CT) == sizeof(T))
    vec = aligned16(cos) && aligned16(sin) && (cb * ces) % 16 == 0 && (cs * ces) % 16 == 0;
  const CT* C = static_cast<const CT*>(cos);
  const CT* Sn = static_cast<const CT*>(sin);
  cudaError_t e;
  if (vec) {
    constexpr int P = 4;
    const int64_t slots = (q.heads + k.heads) * (half / NE);
    int threads = static_cast<int>((slots + 31) / 32 * 32);
    if (threads > 256) threads = 256;
    dim3 grid(static_cast<unsigned>((S + P - 1) / P), static_cast<unsigned>(B));
    e = launch_pdl(rope_rows_kernel<T, CT, P>, grid, dim3(threads), 0, st, q, k, C, Sn, cb, cs,
                   static_cast<int>(S), static_cast<int>(half), sign);
  } else {
    const int64_t per_b = (q.heads + k.heads) * S * half;
    int64_t bx = (per_b + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8 / (B > 0 ? B : 1) + 1;
    if (bx > cap) bx = cap;
    if (bx < 1) bx = 1;
    e = launch_pdl(rope_scalar_kernel<T, CT>, dim3((unsigned)bx, (unsigned)B), dim3(256), 0, st, q, k,
                   C, Sn, cb, cs, S, half, sign);
  }
  return cuda_status(e);
}

}  // namespace
}  // namespace soup

using namespace soup;

extern "C" {

int soup_rope(const void* q, const int64_t* q_strides, void* q_out, const int64_t* q_out_strides,
              int64_t hq, const void* k, const int64_t* k_strides, void* k_out,
              const int64_t* k_out_strides, int64_t hk, const void* cos, const void* sin,
              int64_t cos_sb, int64_t cos_ss, int64_t batch, int64_t seq, int64_t head_dim,
              int dtype, int cos_dtype, int inverse, void* stream) {
  if (!q || !q_strides || !q_out || !q_out_strides || hq <= 0 || !cos || !sin || batch <= 0 ||
      seq <= 0 || head_dim <= 0 || (head_dim % 2) != 0 || batch > 65535 || hk < 0 ||
      (hk > 0 && (!k || !k_strides || !k_out || !k_out_strides))) {
    set_last_error("soup_rope: bad arguments");
    return SOUP_ERR_INVALID;
  }
  RopeTensor tq{q, q_out, q_strides[0], q_strides[1], q_strides[2],
                q_out_strides[0], q_out_strides[1], q_out_strides[2], hq};
  RopeTensor tk{q, q_out, 0, 0, 0, 0, 0, 0, 0};
  if (hk > 0)
    tk = RopeTensor{k, k_out, k_strides[0], k_strides[1], k_strides[2],
                    k_out_strides[0], k_out_strides[1], k_out_strides[2], hk};
  const float sign = inverse ? -1.f : 1.f;
  cudaStream_t st = as_stream(stream);
  if (cos_dtype != dtype && cos_dtype != SOUP_F32) {
    set_last_error("soup_rope: cos/sin must have the activation dtype or fp32");
    return SOUP_ERR_UNSUPPORTED;
  }
#define R(T, CT) return rope_run<T, CT>(tq, tk, cos, sin, cos_sb, cos_ss, batch, seq, head_dim, sign, st)
  if (dtype == SOUP_BF16 && cos_dtype == SOUP_BF16) R(__nv_bfloat16, __nv_bfloat16);
  if (dtype == SOUP_BF16 && cos_dtype == SOUP_F32) R(__nv_bfloat16, float);
  if (dtype == SOUP_F16 && cos_dtype == SOUP_F16) R(__half, __half);
  if (dtype == SOUP_F16 && cos_dtype == SOUP_F32) R(__half, float);
  if (dtype == SOUP_F32 && cos_dtype == SOUP_F32) R(float, float);
#undef R
  set_last_error("soup_rope: unsupported dtype");
  return SOUP_ERR_INVALID;
}

}  // extern "C"
