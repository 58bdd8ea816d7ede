// NF4 (4-bit NormalFloat) blockwise quantisation of frozen base weights and
// its dequantisation, for the QLoRA training step.
//
// Format: for every block of `blocksize` (64) consecutive weights, one fp32
// absmax; each weight is the index of the nearest of 16 code values
// (normalised by absmax), two indices per byte, the earlier element in the
// high nibble. Dequantised value = code[index] * absmax[block]. The 16 code
// values are passed in by the caller (the QLoRA paper's NF4 construction).
#include "soup_common.cuh"

namespace soup {
namespace {

struct Code16 {
  float v[16];
};

// One warp per block of 64: lane l quantises elements 2l and 2l+1.
template <typename T>
__global__ void __launch_bounds__(256) nf4_quantize_kernel(const T* __restrict__ w, int64_t nblocks,
                                                           Code16 code, uint8_t* __restrict__ packed,
                                                           float* __restrict__ absmax) {
  __shared__ float tbl[16];
  if (threadIdx.x < 16) tbl[threadIdx.x] = code.v[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks;
       b += warps) {
    const T* src = w + b * 64 + 2 * lane;
    const float x0 = Cvt<T>::to_f(src[0]);
    const float x1 = Cvt<T>::to_f(src[1]);
    float m = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? 1.f / m : 0.f;
    const float n0 = x0 * inv, n1 = x1 * inv;
    int q0 = 0, q1 = 0;
    float d0 = fabsf(tbl[0] - n0), d1 = fabsf(tbl[0] - n1);
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      const float e0 = fabsf(tbl[i] - n0), e1 = fabsf(tbl[i] - n1);
      if (e0 < d0) {
        d0 = e0;
        q0 = i;
      }
      if (e1 < d1) {
        d1 = e1;
        q1 = i;
      }
    }
    packed[b * 32 + lane] = static_cast<uint8_t>((q0 << 4) | q1);
    if (lane == 0) absmax[b] = m;
  }
}

// Dequantisation: thread i expands packed 32-bit word i (8 weights, bytes in
// memory order, the earlier weight of a byte in its high nibble) into one
// 16-byte output vector (two for fp32), so a warp's loads and stores are each
// one contiguous segment. U words per thread are in flight together. The
// stores use the default cache policy: the weight is read again right away
// by the GEMM that follows, which then finds it in L2.
template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    Vec16<T> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.v[e] = Cvt<T>::from_f(v[e]);
    st16(dst, o);
  } else {
    Vec16<T> a, b;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a.v[e] = Cvt<T>::from_f(v[e]);
      b.v[e] = Cvt<T>::from_f(v[4 + e]);
    }
    st16(dst, a);
    st16(dst + 4, b);
  }
}

template <typename T, int U>
__global__ void __launch_bounds__(256) nf4_dequant_kernel(const uint32_t* __restrict__ packed,
                                                          const float* __restrict__ absmax,
                                                          int64_t nwords, Code16 code,
                                                          T* __restrict__ out) {
  __shared__ float tbl[16];
  if (threadIdx.x < 16) tbl[threadIdx.x] = code.v[threadIdx.x];
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < nwords; i0 += stride * U) {
    uint32_t p[U];
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < nwords) {
        p[u] = __ldcs(packed + i);
        s[u] = __ldg(absmax + (i >> 3));  // 8 words = one block of 64 weights
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < nwords) {
        float v[8];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t byte = (p[u] >> (8 * b)) & 0xffu;
          v[2 * b] = tbl[byte >> 4] * s[u];
          v[2 * b + 1] = tbl[byte & 0xf] * s[u];
        }
        store8(out + i * 8, v);
      }
    }
  }
}

int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace soup

using namespace soup;

extern "C" {

int soup_nf4_quantize(const void* weight, int64_t n, int dtype, int blocksize, const float* code16,
                      uint8_t* packed, float* absmax, void* stream) {
  if (!weight || !code16 || !packed || !absmax || n <= 0 || blocksize != 64 || n % 64 != 0) {
    set_last_error("soup_nf4_quantize: bad arguments (blocksize must be 64, n a multiple of 64)");
    return SOUP_ERR_INVALID;
  }
  Code16 code;
  for (int i = 0; i < 16; ++i) code.v[i] = code16[i];
  const int64_t nb = n / 64;
  const int grid = grid_for(nb, 8);
  cudaStream_t st = as_stream(stream);
  if (dtype == SOUP_BF16)
    nf4_quantize_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(weight), nb,
                                                             code, packed, absmax);
  else if (dtype == SOUP_F16)
    nf4_quantize_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(weight), nb, code,
                                                      packed, absmax);
  else if (dtype == SOUP_F32)
    nf4_quantize_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(weight), nb, code,
                                                     packed, absmax);
  else {
    set_last_error("soup_nf4_quantize: unsupported dtype");
    return SOUP_ERR_INVALID;
  }
  return launch_status();
}

int soup_nf4_dequant(const uint8_t* packed, const float* absmax, int64_t n, int blocksize,
                     const float* code16, void* out, int dtype, void* stream) {
  if (!packed || !absmax || !code16 || !out || n <= 0 || blocksize != 64 || n % 64 != 0) {
    set_last_error("soup_nf4_dequant: bad arguments (blocksize must be 64, n a multiple of 64)");
    return SOUP_ERR_INVALID;
  }
  if (!aligned16(packed) || !aligned16(out)) {
    set_last_error("soup_nf4_dequant: packed and out must be 16-byte aligned");
    return SOUP_ERR_UNSUPPORTED;
  }
  Code16 code;
  for (int i = 0; i < 16; ++i) code.v[i] = code16[i];
  constexpr int U = 4;
  const int64_t nwords = n / 8;
  const int grid = grid_for(nwords, 256 * U);
  cudaStream_t st = as_stream(stream);
  const uint32_t* pw = reinterpret_cast<const uint32_t*>(packed);
  cudaError_t e = cudaSuccess;
  if (dtype == SOUP_BF16)
    e = launch_pdl(nf4_dequant_kernel<__nv_bfloat16, U>, dim3(grid), dim3(256), 0, st, pw, absmax,
                   nwords, code, static_cast<__nv_bfloat16*>(out));
  else if (dtype == SOUP_F16)
    e = launch_pdl(nf4_dequant_kernel<__half, U>, dim3(grid), dim3(256), 0, st, pw, absmax, nwords,
                   code, static_cast<__half*>(out));
  else if (dtype == SOUP_F32)
    e = launch_pdl(nf4_dequant_kernel<float, U>, dim3(grid), dim3(256), 0, st, pw, absmax, nwords,
                   code, static_cast<float*>(out));
  else {
    set_last_error("soup_nf4_dequant: unsupported dtype");
    return SOUP_ERR_INVALID;
  }
  return cuda_status(e);
}

}  // extern "C"
