// Fused lm_head cross-entropy on tcgen05, and the plain GEMM entry point.
//
// One soup_ce_linear call over `rows` tokens runs:
//   0. ce_shift (gradient only): per row a shift c = the target logit
//      (one dot product; column 0's for ignored rows and targets outside the
//      vocabulary) + a margin;
//   1. logits GEMM  L = H W^T  (M=rows, N=vocab, K=dim; A, B K-major) whose
//      epilogue, per row and 256-column vocab tile, keeps the online-softmax
//      state (max, sum exp, sum z*exp, first argmax), captures the target
//      logit, and stores E = exp(z - c) as bf16 into the workspace;
//   2. ce_stats: per row, merges the tile states (ties keep the smaller
//      index), writes loss / entropy / hit, the row factor
//      s = exp(c - lse) / denominator and E[t] = (p_t - 1) exp(lse - c), so
//      that s * E is the row of dlogits = (softmax - onehot) / denominator
//      (s = 0 for ignored rows, whose E stays finite); a gated second logits GEMM with c = lse
//      runs only if a row maximum came out far above its shift;
//   3. ce_sums: fixed-order sums of the per-row losses and hits;
//   4. dX GEMM  dH = diag(s) E W  (A = E K-major, B = W MN-major), split along
//      the vocab into fp32 partials, then a fixed-order reduce that applies s;
//   5. dW GEMM  dW = E^T diag(s) H  (A = E MN-major, B = s * H MN-major).
// No pass rewrites the [rows, vocab] buffer between the GEMMs.
// This follows the semantics of chunk_cross_entropy_triton and its kernel in
// the reference (solution/kernels/chunked_ce.py:32-128, 183-264).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>
#include <stdlib.h>

#include <atomic>

#include "soup_common.cuh"
#include "tc_gemm.cuh"

namespace soup {
namespace tc {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------- epilogues ---
// Each epilogue thread owns one accumulator row (TMEM lane). Stores go through
// the warp's shared-memory staging block (32 rows x 32 fp32): a thread writes
// its row's 32 values, then the warp writes the block out row by row, 8 lanes
// per row, so each global store covers a contiguous 64 B (bf16) or 128 B (fp32)
// row segment instead of scattered 16 B pieces.

__device__ __forceinline__ void stage_row(uint8_t* stage, int lane, const float (&v)[32], float a) {
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(stage + stage_off(lane, q)) =
        make_float4(a * v[4 * q], a * v[4 * q + 1], a * v[4 * q + 2], a * v[4 * q + 3]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// bf16 store of a whole staged 32 x 32 block with 16-byte stores: 4 lanes per
// 64-byte row segment, 8 rows per instruction (lane l: row 8i + l/4, columns
// 8 (l%4) .. +7, read as granules 2 (l%4) and 2 (l%4) + 1 of that row -- the
// XOR layout keeps the 8 lanes of each 128-bit access phase on distinct banks).
__device__ __forceinline__ void write_block_bf16_v16(const uint8_t* stage, int lane, bf16* C,
                                                     int64_t ldc, int row0, int M, int col0) {
  const int c8 = lane & 3;
  const int rsub = lane >> 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + rsub;
    const int grow = row0 + r;
    if (grow >= M) continue;
    const float4 a = *reinterpret_cast<const float4*>(stage + stage_off(r, 2 * c8));
    const float4 b = *reinterpret_cast<const float4*>(stage + stage_off(r, 2 * c8 + 1));
    *reinterpret_cast<uint4*>(C + (int64_t)grow * ldc + col0 + c8 * 8) =
        make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                   pack_bf16x2(b.z, b.w));
  }
}

// Write the staged block to C rows [row0, row0+32) x cols [col0, col0+32),
// clipped to M x N. `vec`: rows are 16-byte aligned (vector stores allowed).
template <bool BF16>
__device__ __forceinline__ void write_block(const uint8_t* stage, int lane, void* C, int64_t ldc,
                                            int row0, int M, int col0, int N, bool vec,
                                            bool accumulate) {
  if constexpr (BF16) {
    if (vec && !accumulate && col0 + 32 <= N) {
      write_block_bf16_v16(stage, lane, reinterpret_cast<bf16*>(C), ldc, row0, M, col0);
      return;
    }
  }
  const int cv = lane & 7;
  const int rsub = lane >> 3;
  const int gcol = col0 + cv * 4;
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int r = i * 4 + rsub;
    const int grow = row0 + r;
    if (grow >= M) continue;
    float4 x = *reinterpret_cast<const float4*>(stage + stage_off(r, cv));
    if (vec && gcol + 4 <= N) {
      if constexpr (BF16) {
        bf16* dst = reinterpret_cast<bf16*>(C) + (int64_t)grow * ldc + gcol;
        if (accumulate) {
          uint2 o = *reinterpret_cast<const uint2*>(dst);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&o);
          float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
          x.x += a.x;
          x.y += a.y;
          x.z += b.x;
          x.w += b.y;
        }
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(x.x, x.y), pack_bf16x2(x.z, x.w));
      } else {
        float* dst = reinterpret_cast<float*>(C) + (int64_t)grow * ldc + gcol;
        if (accumulate) {
          float4 o = *reinterpret_cast<const float4*>(dst);
          x.x += o.x;
          x.y += o.y;
          x.z += o.z;
          x.w += o.w;
        }
        *reinterpret_cast<float4*>(dst) = x;
      }
    } else {
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (gcol + e < N) {
          if constexpr (BF16) {
            bf16* dst = reinterpret_cast<bf16*>(C) + (int64_t)grow * ldc + gcol + e;
            float y = xs[e];
            if (accumulate) y += __bfloat162float(*dst);
            *dst = __float2bfloat16_rn(y);
          } else {
            float* dst = reinterpret_cast<float*>(C) + (int64_t)grow * ldc + gcol + e;
            *dst = accumulate ? *dst + xs[e] : xs[e];
          }
        }
      }
    }
  }
}

// A warp's 32 x 32 bf16 output block (thread t: row row0 + t, values a * v)
// stored by TMA: written into half (nstore & 1) of the warp's staging block in
// the store map's 64-byte swizzle (16-byte chunk q of row r at chunk
// q ^ ((r >> 1) & 3): the 8 lanes of every 128-bit access phase hit distinct
// banks), fenced for the async proxy, then one lane issues the store. Before a
// half is rewritten its store from two blocks earlier must have finished
// reading it (at most one bulk group still reading). Rows / columns outside
// the map are not written.
__device__ __forceinline__ void tma_store_block_bf16(const CUtensorMap* map, uint8_t* stage, int lane,
                                                     int& nstore, const float (&v)[32], float a,
                                                     int col0, int row0, int M) {
  if (row0 >= M) return;  // all 32 rows outside the output (warp-uniform)
  uint8_t* buf = stage + (nstore & 1) * 2048;
  if (lane == 0) bulk_wait_read1();
  __syncwarp();
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = make_uint4(pack_bf16x2(a * v[8 * q], a * v[8 * q + 1]),
                               pack_bf16x2(a * v[8 * q + 2], a * v[8 * q + 3]),
                               pack_bf16x2(a * v[8 * q + 4], a * v[8 * q + 5]),
                               pack_bf16x2(a * v[8 * q + 6], a * v[8 * q + 7]));
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((q ^ sw) << 4)) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, smem_u32(buf), col0, row0);
    bulk_commit();
  }
  ++nstore;
}

// Plain store: C = alpha * scale * acc (+ C). `scale` is an optional device
// scalar (e.g. the upstream gradient of the loss). `split_stride` > 0 writes
// k-split partial slices (fp32) at C + ks * split_stride.
template <int BN>
struct EpiStore {
  struct Params {
    void* c;
    int64_t ldc;
    int64_t split_stride;
    const float* scale;
    float alpha;
    int c_bf16;
    int accumulate;
    int vec_ok;  // 16-byte aligned rows
    int M, N;
    const bf16* bias;  // optional [N] added to every row after scaling
    int tma;           // bf16, no accumulate, no k split: store through tma_c
    const float* row_scale;  // optional [M]: row m scaled by row_scale[m]
  };
  static __device__ __forceinline__ void tile(const Params& p, const CUtensorMap* tmc, int row_base, int nt, int ks,
                                              int quarter, int lane, uint32_t taddr, uint8_t* stage,
                                              int group, int ngroups) {
    const int row0 = row_base + quarter * 32;
    float a = p.alpha * (p.scale ? *p.scale : 1.f);
    if (p.row_scale && row0 + lane < p.M) a *= p.row_scale[row0 + lane];  // lane = row
    const size_t es = p.c_bf16 ? 2 : 4;
    void* C = static_cast<uint8_t*>(p.c) + (size_t)ks * p.split_stride * es;
    const int nch = BN / 32 / ngroups;
    int nstore = 0;
#pragma unroll 1
    for (int c = group * nch; c < (group + 1) * nch; ++c) {
      float v[32];
      tmem_ld32(taddr + c * 32, v);
      const int col0 = nt * BN + c * 32;
      if (col0 >= p.N) continue;
      float sa = a;
      if (p.bias) {  // every lane reads the same 32 values (broadcast)
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = fmaf(a, v[j], col0 + j < p.N ? __bfloat162float(p.bias[col0 + j]) : 0.f);
        sa = 1.f;
      }
      if (p.tma) {
        tma_store_block_bf16(tmc, stage, lane, nstore, v, sa, col0, row0, p.M);
        continue;
      }
      stage_row(stage, lane, v, sa);
      __syncwarp();
      if (p.c_bf16)
        write_block<true>(stage, lane, C, p.ldc, row0, p.M, col0, p.N, p.vec_ok, p.accumulate);
      else
        write_block<false>(stage, lane, C, p.ldc, row0, p.M, col0, p.N, p.vec_ok, p.accumulate);
      __syncwarp();
    }
  }
};

// A 32 x 32 bf16 block of C (rows [row0, row0+32), cols [col0, col0+32),
// 16-byte aligned rows) in two steps, so the global loads can be in flight
// while the warp does other work: load_block_bf16 issues the loads (lane l
// takes rows 4i + l/8, columns 4 (l%8) .. +3; rows beyond M read as 0),
// stage_block_bf16 puts them into the warp's staging block as fp32 (the
// inverse of write_block's access pattern).
__device__ __forceinline__ void load_block_bf16(uint2 (&r)[8], int lane, const bf16* C, int64_t ldc,
                                                int row0, int M, int col0) {
  const int cv = lane & 7;
  const int rsub = lane >> 3;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int grow = row0 + i * 4 + rsub;
    r[i] = grow < M ? *reinterpret_cast<const uint2*>(C + (int64_t)grow * ldc + col0 + cv * 4)
                    : make_uint2(0u, 0u);
  }
}
__device__ __forceinline__ void stage_block_bf16(uint8_t* stage, int lane, const uint2 (&r)[8]) {
  const int cv = lane & 7;
  const int rsub = lane >> 3;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r[i]);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    *reinterpret_cast<float4*>(stage + stage_off(i * 4 + rsub, cv)) = make_float4(a.x, a.y, b.x, b.y);
  }
}

// SwiGLU epilogue of a gate/up GEMM whose weight rows are interleaved in
// blocks of 128 (rows [256 c, 256 c + 128) = gate rows [128 c, 128 c + 128),
// the next 128 = the same up rows): tile nt's 256 columns hold g (0-127) and
// u (128-255) for intermediate columns [128 nt, 128 nt + 128). g and u are
// first rounded to bf16 (+ bias) exactly as a plain bf16 GEMM output would be,
// so the results equal the unfused GEMM + SwiGLU kernels bit for bit.
//   mode 0: h = silu(g) u -> h [M, N/2]; with y != nullptr also g, u -> y [M, N]
//   mode 1: dh from h [M, N/2]; dg, du -> y [M, N] at the tile's g / u columns
template <int BN>
struct EpiSwiGLU {
  static constexpr bool kHalves = true;  // a warp reads g chunks and the u chunks BN/2 further
  struct Params {
    int mode;
    bf16* h;  // mode 0: output h; mode 1: input dh
    int64_t ldh;
    bf16* y;  // mode 0: optional [g | u] copy; mode 1: output [dg | du]
    int64_t ldy;
    const bf16* bias;  // [N] in the interleaved order, or nullptr
    int M, N;
  };
  // mode 1: the dh block of a warp's next chunk is in flight while the warp
  // waits (for the tile's accumulator, or on the previous chunk's work)
  struct Carry {
    uint2 d[8];
  };
  static __device__ __forceinline__ void prefetch(const Params& p, int row_base, int nt, int quarter,
                                                  int lane, int group, int ngroups, Carry& c) {
    constexpr int kHalf = BN / 2;
    if (p.mode == 1)
      load_block_bf16(c.d, lane, p.h, p.ldh, row_base + quarter * 32, p.M,
                      nt * kHalf + group * (kHalf / 32 / ngroups) * 32);
  }
  static __device__ __forceinline__ void tile(const Params& p, const CUtensorMap* tmc, int row_base, int nt, int ks,
                                              int quarter, int lane, uint32_t taddr, uint8_t* stage,
                                              int group, int ngroups, Carry& carry) {
    constexpr int kHalf = BN / 2;
    const int row0 = row_base + quarter * 32;
    const int nch = kHalf / 32 / ngroups;
    const int inter = p.N / 2;
    uint2 (&dnext)[8] = carry.d;
#pragma unroll 1
    for (int cc = group * nch; cc < (group + 1) * nch; ++cc) {
      float g[32], u[32];
      tmem_ld32(taddr + cc * 32, g);
      tmem_ld32(taddr + kHalf + cc * 32, u);
      const int gcol = nt * BN + cc * 32;  // g's columns in [M, N]; u's are kHalf further
      const int icol = nt * kHalf + cc * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float bg = p.bias ? __bfloat162float(p.bias[gcol + j]) : 0.f;
        const float bu = p.bias ? __bfloat162float(p.bias[gcol + kHalf + j]) : 0.f;
        g[j] = __bfloat162float(__float2bfloat16_rn(p.bias ? fmaf(1.f, g[j], bg) : g[j]));
        u[j] = __bfloat162float(__float2bfloat16_rn(p.bias ? fmaf(1.f, u[j], bu) : u[j]));
      }
      if (p.mode == 0) {
        if (p.y) {
          stage_row(stage, lane, g, 1.f);
          __syncwarp();
          write_block<true>(stage, lane, p.y, p.ldy, row0, p.M, gcol, p.N, true, false);
          __syncwarp();
          stage_row(stage, lane, u, 1.f);
          __syncwarp();
          write_block<true>(stage, lane, p.y, p.ldy, row0, p.M, gcol + kHalf, p.N, true, false);
          __syncwarp();
        }
        float hv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) hv[j] = swiglu_fwd_f(g[j], u[j]);
        stage_row(stage, lane, hv, 1.f);
        __syncwarp();
        write_block<true>(stage, lane, p.h, p.ldh, row0, p.M, icol, inter, true, false);
        __syncwarp();
      } else {
        stage_block_bf16(stage, lane, dnext);
        if (cc + 1 < (group + 1) * nch)
          load_block_bf16(dnext, lane, p.h, p.ldh, row0, p.M, icol + 32);
        __syncwarp();
        float d[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 x = *reinterpret_cast<const float4*>(stage + stage_off(lane, q));
          d[4 * q] = x.x;
          d[4 * q + 1] = x.y;
          d[4 * q + 2] = x.z;
          d[4 * q + 3] = x.w;
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float dg, du;
          swiglu_bwd_f(d[j], g[j], u[j], dg, du);
          g[j] = dg;
          u[j] = du;
        }
        stage_row(stage, lane, g, 1.f);
        __syncwarp();
        write_block<true>(stage, lane, p.y, p.ldy, row0, p.M, gcol, p.N, true, false);
        __syncwarp();
        stage_row(stage, lane, u, 1.f);
        __syncwarp();
        write_block<true>(stage, lane, p.y, p.ldy, row0, p.M, gcol + kHalf, p.N, true, false);
        __syncwarp();
      }
    }
  }
};

// SwiGLU backward in the epilogue of the down projection's input-gradient GEMM:
// the accumulator is dh [M, N] (N = the intermediate size), which is rounded to
// bf16 as a plain GEMM output would be; with g and u read from y in the
// interleaved layout of EpiSwiGLU (intermediate column c: g at column
// 256 (c / 128) + c % 128 of y, u 128 further), dg and du overwrite g and u in y.
// Every (row, column) pair is read and written by one lane, so the update is in
// place. Results equal the unfused GEMM + SwiGLU backward kernels bit for bit.
template <int BN>
struct EpiDSwiGLU {
  struct Params {
    bf16* y;  // [M, 2N]: [g | u] in, [dg | du] out
    int64_t ldy;
    int M, N;
  };
  // A warp owns 32 accumulator rows (its TMEM lane quarter) x its group's columns,
  // which lie in one interleave block of 128. Rows are handled in two halves of
  // 16: dh of the half goes through the warp's staging block as bf16 (16 rows x
  // 128 columns = 4 KB), then each lane takes 8 consecutive columns of a row, so
  // every load / store instruction covers 2 rows x 256 contiguous bytes of g, u,
  // dg and du (long DRAM bursts; the same rows' g and u are 128 columns apart).
  static constexpr int kPass = 4;  // passes (2 rows each) whose loads are issued together
  static __device__ __forceinline__ int gcol_of(int icol) { return (icol >> 7) * 256 + (icol & 127); }
  static __device__ __forceinline__ void tile(const Params& p, const CUtensorMap* tmc, int row_base, int nt,
                                              int ks, int quarter, int lane, uint32_t taddr,
                                              uint8_t* stage, int group, int ngroups) {
    const int nch = BN / 32 / ngroups;   // 32-column chunks of this warp (4 with 8 warps)
    const int c0 = group * nch;
    const int icol0 = nt * BN + c0 * 32;  // first intermediate column of the warp
    if (icol0 >= p.N) {
      for (int cc = c0; cc < c0 + nch; ++cc) {  // the accumulator is read in every case
        float d[32];
        tmem_ld32(taddr + cc * 32, d);
      }
      return;
    }
    const int width = nch * 32;          // <= 128, within one interleave block
    const int gc0 = gcol_of(icol0);
    const int row0 = row_base + quarter * 32;
    uint16_t* sh = reinterpret_cast<uint16_t*>(stage);  // [16][width] bf16
#pragma unroll 1
    for (int hr = 0; hr < 2; ++hr) {
#pragma unroll 1
      for (int cc = 0; cc < nch; ++cc) {
        float d[32];
        tmem_ld32(taddr + (c0 + cc) * 32, d);
        if ((lane >> 4) == hr) {
          uint32_t wv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) wv[j] = pack_bf16x2(d[2 * j], d[2 * j + 1]);
          uint4* dst = reinterpret_cast<uint4*>(sh + (lane & 15) * width + cc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
        }
      }
      __syncwarp();
      const int lpr = width / 8;            // lanes per row (16 for 128 columns)
      const int rpp = 32 / lpr;             // rows per pass
      const int npass = 16 / rpp;
      const int cl = lane % lpr, rl = lane / lpr;
#pragma unroll 1
      for (int p0 = 0; p0 < npass; p0 += kPass) {
        uint4 gv[kPass], uv[kPass];
#pragma unroll
        for (int k = 0; k < kPass; ++k) {
          const int r = (p0 + k) * rpp + rl;  // row within the half
          const int grow = row0 + hr * 16 + r;
          if (p0 + k < npass && grow < p.M) {
            const bf16* src = p.y + (int64_t)grow * p.ldy + gc0 + 8 * cl;
            gv[k] = *reinterpret_cast<const uint4*>(src);
            uv[k] = *reinterpret_cast<const uint4*>(src + 128);
          }
        }
#pragma unroll
        for (int k = 0; k < kPass; ++k) {
          const int r = (p0 + k) * rpp + rl;
          const int grow = row0 + hr * 16 + r;
          if (p0 + k >= npass || grow >= p.M) continue;
          const uint4 dv4 = *reinterpret_cast<const uint4*>(sh + r * width + 8 * cl);
          const __nv_bfloat162* dh2 = reinterpret_cast<const __nv_bfloat162*>(&dv4);
          const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv[k]);
          const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv[k]);
          uint32_t og[4], ou[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 dd = __bfloat1622float2(dh2[q]), gg = __bfloat1622float2(g2[q]),
                         uu = __bfloat1622float2(u2[q]);
            float dg0, du0, dg1, du1;
            swiglu_bwd_f(dd.x, gg.x, uu.x, dg0, du0);
            swiglu_bwd_f(dd.y, gg.y, uu.y, dg1, du1);
            og[q] = pack_bf16x2(dg0, dg1);
            ou[q] = pack_bf16x2(du0, du1);
          }
          bf16* dst = p.y + (int64_t)grow * p.ldy + gc0 + 8 * cl;
          *reinterpret_cast<uint4*>(dst) = make_uint4(og[0], og[1], og[2], og[3]);
          *reinterpret_cast<uint4*>(dst + 128) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
        }
      }
      __syncwarp();  // the staging block is rewritten by the next half
    }
  }
};

// Logits epilogue of the CE forward: online-softmax state per (row, tile),
// target logit capture, bf16 logits store.
// Shifted exponentials. With `shift` set, the tile stores E = exp(z - c_row)
// in bf16 instead of the logit z. The
// gradient of the row is then dL = s_row * E with one entry corrected for the
// target, s_row = exp(c_row - lse_row) / denominator, so the dX and dW GEMMs
// read E directly and no pass rewrites the logits buffer. bf16 has the fp32
// exponent range: with c within a few tens of the row maximum, E neither
// overflows nor loses any entry of relative size above e^-50.
constexpr float kShiftMargin = 32.f;  // c = (target or column-0 logit) + margin
constexpr float kShiftGap = 40.f;     // a tile maximum above c + gap raises the flag

template <int BN>
struct EpiCE {
  struct Params {
    const int64_t* targets;
    float4* partials;  // [n_tiles * ngroups][M]: (max, sum exp, sum z*exp, argmax bits)
    float* zt;         // [M] target logit (written by the tile holding it)
    bf16* logits;      // [M][ld_logits] or nullptr
    int64_t ld_logits;
    int64_t vocab_offset;  // first vocabulary row of this weight shard (0 unsharded)
    int M, N;
    int tma;  // logits stored through tma_c
    const float* shift;  // [M] or nullptr (store the logits themselves)
    int* flag;           // set to 1 when a row's maximum exceeds shift + kShiftGap
    int onehot;          // shift = lse: store E - 1 at the target column (= p - 1)
    int has_ignore;      // rows whose target is ignore_index store E = 0 (statistics kept)
    int64_t ignore_index;
  };
  static __device__ __forceinline__ void store(const Params& p, const CUtensorMap* tmc,
                                               uint8_t* stage, int lane, int& nstore,
                                               const float (&v)[32], int col0, int row0) {
    if (p.tma) {
      tma_store_block_bf16(tmc, stage, lane, nstore, v, 1.f, col0, row0, p.M);
    } else {
      stage_row(stage, lane, v, 1.f);
      __syncwarp();
      write_block<true>(stage, lane, p.logits, p.ld_logits, row0, p.M, col0, p.N, true, false);
      __syncwarp();
    }
  }
  // Shifted mode: the sums run against a fixed reference, the row's shift c:
  // S = sum exp(z - c), W = sum z exp(z - c), whose terms are the stored E
  // themselves, on packed fp32 pairs; the record is rescaled to the tile
  // maximum once at the end. A chunk maximum more than kRebase above the
  // reference (possible only on a row that also raises the overflow flag,
  // kRebase > kShiftGap) moves the reference up so the sums stay finite; the
  // values then stored for that row are rewritten by the fallback GEMM.
  static constexpr float kRebase = 60.f;
  static __device__ __forceinline__ void tile_shifted(const Params& p, const CUtensorMap* tmc,
                                                      int row0, int nt, int lane, uint32_t taddr,
                                                      uint8_t* stage, int group, int ngroups) {
    const int row = row0 + lane;
    const int nch = BN / 32 / ngroups;
    const bool row_ok = row < p.M;
    const int64_t t = row_ok ? p.targets[row] - p.vocab_offset : -1;
    // rows past M: any finite reference (nothing of theirs is stored or recorded)
    const float c = row_ok ? p.shift[row] : 0.f;
    // an ignored row's gradient is 0: store zeros, which also keeps the dX / dW
    // operands sparse (zero operands draw less tensor-core power)
    const bool zero_row = p.has_ignore && row_ok && p.targets[row] == p.ignore_index;
    float ref = c;
    float m = -INFINITY;
    int bidx = 0x7fffffff;
    float ztv = 0.f;
    bool found = false, over = false;
    int nstore = 0;
    uint64_t S2 = f2_pack(0.f, 0.f), W2 = f2_pack(0.f, 0.f);
    const uint64_t L2 = f2_pack(kLog2e, kLog2e);
#pragma unroll 1
    for (int cc = group * nch; cc < (group + 1) * nch; ++cc) {
      float v[32];
      tmem_ld32(taddr + cc * 32, v);
      const int col0 = nt * BN + cc * 32;
      const int nvalid = p.N - col0;
      if (nvalid <= 0) continue;
      if (nvalid < 32) {  // finite fill: exp gives 0 and 0 * fill stays 0
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j >= nvalid) v[j] = -1e30f;
      }
      float cm = v[0];
#pragma unroll
      for (int j = 1; j < 32; ++j) cm = fmaxf(cm, v[j]);
      if (cm > m) {  // new maximum: its first index in the chunk
        int ci = 0;
#pragma unroll
        for (int j = 31; j >= 0; --j)
          if (v[j] == cm) ci = j;
        m = cm;
        bidx = col0 + ci;
      }
      const bool has_t = t >= col0 && t < col0 + 32 && t < p.N;
      const int tj = static_cast<int>(t - col0);
      if (has_t) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j == tj) ztv = v[j];
        found = true;
      }
      over |= cm - c > kShiftGap;
      if (cm - ref > kRebase) {
        const float f = fast_exp2((ref - cm) * kLog2e);
        const uint64_t f2 = f2_pack(f, f);
        S2 = f2_mul(S2, f2);
        W2 = f2_mul(W2, f2);
        ref = cm;
      }
      const float rb = ref * kLog2e;
      const uint64_t NR = f2_pack(-rb, -rb);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint64_t z = f2_pack(v[2 * i], v[2 * i + 1]);
        float a0, a1;
        f2_unpack(f2_fma(z, L2, NR), a0, a1);
        const float e0 = fast_exp2(a0), e1 = fast_exp2(a1);  // 0 for padded columns
        const uint64_t e = f2_pack(e0, e1);
        S2 = f2_add(S2, e);
        W2 = f2_fma(z, e, W2);
        v[2 * i] = e0;
        v[2 * i + 1] = e1;
      }
      if (p.onehot && has_t) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j == tj) v[j] -= 1.f;
      }
      if (zero_row) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      store(p, tmc, stage, lane, nstore, v, col0, row0);
    }
    if (row_ok) {
      float s0, s1, w0, w1;
      f2_unpack(S2, s0, s1);
      f2_unpack(W2, w0, w1);
      // relative to the tile maximum; a tile more than 80 below the reference
      // holds probabilities below e^-48 of the row (the reference is at most
      // 32 above the logit of one of the row's columns) and counts as empty
      float sr = 0.f, wr = 0.f;
      if (m != -INFINITY && ref - m <= 80.f) {
        const float g = fast_exp2((ref - m) * kLog2e);
        sr = (s0 + s1) * g;
        wr = (w0 + w1) * g;
      }
      p.partials[(int64_t)(nt * ngroups + group) * p.M + row] = make_float4(m, sr, wr, __int_as_float(bidx));
      if (found) p.zt[row] = ztv;
      if (over) *p.flag = 1;
    }
  }
  static __device__ __forceinline__ void tile(const Params& p, const CUtensorMap* tmc, int row_base, int nt, int ks,
                                              int quarter, int lane, uint32_t taddr, uint8_t* stage,
                                              int group, int ngroups) {
    const int row0 = row_base + quarter * 32;
    if (p.logits && p.shift) {
      tile_shifted(p, tmc, row0, nt, lane, taddr, stage, group, ngroups);
      return;
    }
    // raw mode: the logits themselves (or nothing) stored, running-maximum sums
    const int row = row0 + lane;
    const int nch = BN / 32 / ngroups;
    const bool row_ok = row < p.M;
    const int64_t t = row_ok ? p.targets[row] - p.vocab_offset : -1;
    float m = -INFINITY, s = 0.f, w = 0.f;
    int bidx = 0x7fffffff;
    float ztv = 0.f;
    bool found = false;
    int nstore = 0;
#pragma unroll 1
    for (int cc = group * nch; cc < (group + 1) * nch; ++cc) {
      float v[32];
      tmem_ld32(taddr + cc * 32, v);
      const int col0 = nt * BN + cc * 32;
      const int nvalid = p.N - col0;
      if (nvalid <= 0) continue;
      if (nvalid < 32) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j >= nvalid) v[j] = -1e30f;
      }
      if (p.logits) store(p, tmc, stage, lane, nstore, v, col0, row0);
      // chunk maximum with its first index
      float cm = v[0];
      int ci = 0;
#pragma unroll
      for (int j = 1; j < 32; ++j)
        if (v[j] > cm) {
          cm = v[j];
          ci = j;
        }
      if (cm > m) {
        const float f = fast_exp2((m - cm) * kLog2e);  // 0 when m = -inf
        s *= f;
        w *= f;
        m = cm;
        bidx = col0 + ci;
      }
      if (t >= col0 && t < col0 + 32 && t < p.N) {
        const int tj = static_cast<int>(t - col0);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j == tj) ztv = v[j];
        found = true;
      }
      const float mb = m * kLog2e;
      if (nvalid >= 32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float e = fast_exp2(fmaf(v[j], kLog2e, -mb));
          s += e;
          w = fmaf(v[j], e, w);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j < nvalid) {
            const float e = fast_exp2(fmaf(v[j], kLog2e, -mb));
            s += e;
            w = fmaf(v[j], e, w);
          }
        }
      }
    }
    if (row_ok) {
      p.partials[(int64_t)(nt * ngroups + group) * p.M + row] = make_float4(m, s, w, __int_as_float(bidx));
      if (found) p.zt[row] = ztv;
    }
  }
};

// ------------------------------------------------------- tensor maps -------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D map of a 16-bit type (bf16 by default, or fp16) over a row-major matrix
// [outer, inner] with row stride ld (elements), box {64, box_outer}, 128-byte
// swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                    uint32_t box_outer,
                    CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return SOUP_ERR_CUDA;
  }
  if (int rc = bind_context()) return rc;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[160];
    snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu ld=%llu",
             static_cast<int>(r), (unsigned long long)inner, (unsigned long long)outer,
             (unsigned long long)ld);
    set_last_error(msg);
    return SOUP_ERR_UNSUPPORTED;
  }
  return SOUP_OK;
}

// Output map for the epilogues' TMA stores: bf16 [outer, inner] with row
// stride ld (elements), box {32, 32}, 64-byte swizzle (the staging layout of
// tma_store_block_bf16).
static int make_store_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer,
                          uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return SOUP_ERR_CUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed for an output map");
    return SOUP_ERR_UNSUPPORTED;
  }
  return SOUP_OK;
}

// Operand map: K-major operand stored [rows, K]: box {64 (K), rows_box};
// MN-major operand stored [K, rows]: box {64 (MN), 64 (K)}.
static int make_operand_map(CUtensorMap* map, const void* ptr, bool mn_major, int64_t rows, int64_t k,
                            int64_t ld, int rows_box, bool f16 = false) {
  const CUtensorMapDataType dt =
      f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (mn_major) return make_map(map, ptr, rows, k, ld, 64, dt);
  return make_map(map, ptr, k, rows, ld, rows_box, dt);
}

static bool tma_ok(const void* p, int64_t ld) {
  return aligned16(p) && ((ld * 2) % 16 == 0) && ld > 0;
}

constexpr int kBN = 256;
constexpr int kStages = 4;

// Epilogue warps of every GEMM launch (two per TMEM lane quarter).
constexpr int kEpiWarps = 8;

// CTA-pair tiles (256 rows over two SMs, cta_group::2) are the default;
// SOUP_GEMM_PAIRS=0 in the environment selects single-CTA 128-row tiles.
static bool use_pairs() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SOUP_GEMM_PAIRS");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}
// rows of one output tile, and the row box of a K-major B operand map
static int tile_m() { return use_pairs() ? 2 * BM : BM; }
static int b_box_rows() { return use_pairs() ? kBN / 2 : kBN; }
static int m_tiles(int64_t m) { return static_cast<int>((m + tile_m() - 1) / tile_m()); }

constexpr int kPairStages = 6;

template <bool A_MN, bool B_MN, class Epi>
static int launch_gemm_single(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ma2,
                              const CUtensorMap& mb2, const CUtensorMap& mc, Sched sched,
                              const typename Epi::Params& ep, cudaStream_t stream, int* err) {
  using L = SmemLayout<kBN, kStages, kEpiWarps>;
  auto kern = gemm_kernel<kBN, kStages, A_MN, B_MN, Epi, kEpiWarps>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(cache_mutex());
    if (!attr_set[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
      if (e != cudaSuccess) return cuda_status(e);
      attr_set[dev] = true;
    }
  }
  const int units = sched.m_tiles * sched.n_tiles * sched.splits;
  const int grid = units < num_sms() ? units : num_sms();
  kern<<<grid, gemm_threads(kEpiWarps), L::kBytes, stream>>>(ma, mb, ma2, mb2, mc, sched, ep, err);
  return launch_status();
}

// ---- stream-K scratch, one per device (soup_gemm_set_stream_k_workspace) ----
// Layout, fixed for a device: ready flags [slots][kSlotFlags] int (zero
// between launches), padded to 256 bytes, then the fp32 partial slots
// [slots][kSlotFloats], slots = half the SM count (one per CTA pair). Every
// launch uses the same offsets, so no launch's partials land where another
// launch's flags live.
using SkL = SkLayout<kBN, kEpiWarps>;
// A stream-K tail has on average at most this many k parts per tile.
constexpr int kSkMaxParts = 3;
struct SkWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
static SkWorkspace g_sk_ws[64];

static size_t sk_flag_bytes(int slots) {
  return ((size_t)slots * SkL::kSlotFlags * sizeof(int) + 255) & ~(size_t)255;
}
static size_t sk_bytes(int slots) {
  return sk_flag_bytes(slots) + (size_t)slots * SkL::kSlotFloats * sizeof(float);
}

// k blocks a stream-K tail must save over a whole tile
// (soup_gemm_set_stream_k_min_saved)
constexpr int kSkMinSavedDefault = 24;
static std::atomic<int> g_sk_min_saved{kSkMinSavedDefault};
static int sk_min_saved() { return g_sk_min_saved.load(std::memory_order_relaxed); }

// Fills in sched's stream-K fields when the current device has a workspace,
// the launch has one k split and is no diagnostic, and the tiles do not fill
// whole waves of `max_cl` clusters; returns the number of clusters to launch.
static int plan_stream_k(Sched& sched, int max_cl, int dev) {
  const int tiles = sched.m_tiles * sched.n_tiles;
  const int whole = tiles < max_cl ? tiles : max_cl;
  if (sched.splits != 1 || sched.withhold >= 0 || tiles % max_cl == 0) return whole;
  SkWorkspace ws;
  {
    std::lock_guard<std::mutex> lock(cache_mutex());
    ws = g_sk_ws[dev];
  }
  if (!ws.ptr) return whole;
  const int sk = tiles > max_cl ? tiles % max_cl : tiles;
  const long long iters = (long long)sk * sched.kb_total;
  long long skc = max_cl;
  if (skc > (long long)sk * kSkMaxParts) skc = (long long)sk * kSkMaxParts;
  if (skc > iters) skc = iters;
  const int slots = num_sms() / 2;
  // the kernel computes segment bounds in 32-bit integers
  if (skc <= sk || skc > slots || sk_bytes(slots) > ws.bytes || (iters + 1) * (skc + 1) >= (1ll << 31))
    return whole;
  // worth it only if a segment is much shorter than a tile: a finishing pair
  // waits for the partials and adds them after its last MMA (measured at 5-7 us
  // per launch on B200, the time of ~20 k blocks of a 256 x 256 tile)
  if ((iters + skc - 1) / skc + sk_min_saved() > sched.kb_total) return whole;
  sched.sk_tiles = sk;
  sched.sk_clusters = (int)skc;
  sched.sk_flag = static_cast<int*>(ws.ptr);
  sched.sk_part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws.ptr) + sk_flag_bytes(slots));
  return tiles > max_cl ? max_cl : (int)skc;
}

template <bool A_MN, bool B_MN, class Epi>
static int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ma2,
                            const CUtensorMap& mb2, const CUtensorMap& mc, Sched sched,
                            const typename Epi::Params& ep, cudaStream_t stream, int* err) {
  using L = SmemLayout<kBN / 2, kPairStages, kEpiWarps>;
  static_assert(L::kBytes <= 232448, "pair GEMM shared memory exceeds 227 KB");
  auto kern = gemm_pair_kernel<kBN, kPairStages, A_MN, B_MN, Epi, kEpiWarps>;
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cuda_status(cudaErrorInvalidDevice);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch: the prologue (barriers, TMEM allocation)
  // overlaps the previous kernel's tail; the kernel waits (griddepcontrol.wait)
  // before any global memory access
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(gemm_threads(kEpiWarps));
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const int sms = num_sms();
  int max_cl = 0;
  {
    std::lock_guard<std::mutex> lock(cache_mutex());
    if (max_clusters[dev] == 0) {
      cudaError_t e =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
      if (e != cudaSuccess) return cuda_status(e);
      int n = 0;
      cfg.gridDim = dim3(2 * (sms / 2));
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return cuda_status(e);
      if (n <= 0) {
        set_last_error("pair GEMM: no cluster of two CTAs fits on this device");
        return SOUP_ERR_UNSUPPORTED;
      }
      max_clusters[dev] = n;
    }
    max_cl = max_clusters[dev];
  }
  const int units = sched.m_tiles * sched.n_tiles * sched.splits;
  const int clusters = sched.splits == 1 ? plan_stream_k(sched, max_cl, dev)
                                         : (units < max_cl ? units : max_cl);
  cfg.gridDim = dim3(2 * clusters);
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ma, mb, ma2, mb2, mc, sched, ep, err));
}

// sched.m_tiles counts tile_m() rows. ma2 / mb2 are read for the last
// sched.kb2 k-blocks (the second K segment); mc is the output map of an
// epilogue that stores through TMA (any valid map otherwise).
template <bool A_MN, bool B_MN, class Epi>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ma2,
                       const CUtensorMap& mb2, const CUtensorMap& mc, Sched sched,
                       const typename Epi::Params& ep, cudaStream_t stream) {
  const int units = sched.m_tiles * sched.n_tiles * sched.splits;
  if (units <= 0) return SOUP_OK;
  int* err = device_err_ptr();
  if (!err) {
    set_last_error("device error word unavailable");
    return SOUP_ERR_CUDA;
  }
  if (sched.wait_ns == 0) sched.wait_ns = wait_limit_ns();
  if (use_pairs())
    return launch_gemm_pair<A_MN, B_MN, Epi>(ma, mb, ma2, mb2, mc, sched, ep, stream, err);
  return launch_gemm_single<A_MN, B_MN, Epi>(ma, mb, ma2, mb2, mc, sched, ep, stream, err);
}

// One K segment (sched.kb2 must be 0).
template <bool A_MN, bool B_MN, class Epi>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                       Sched sched, const typename Epi::Params& ep, cudaStream_t stream) {
  sched.kb2 = 0;
  return launch_gemm<A_MN, B_MN, Epi>(ma, mb, ma, mb, mc, sched, ep, stream);
}

// ------------------------------------------------------ CE row kernels -----
// Per row, before the logits GEMM: the shift c of the shifted exponentials,
// the logit of the row's target (targets[row] - vocab_offset on a vocabulary
// shard) plus kShiftMargin, or of column 0 when the target is outside the
// vocabulary (shard) or the row is ignored: ignored rows still record their
// entropy, and their gradient factor is 0 later. Any finite value not far
// below the row maximum works; the logit of one column is a lower bound of
// that maximum. One warp per row; also clears the overflow flag of this call.
// Rows are 16-byte aligned with dim % 8 == 0. T: the operands' type (bf16 or
// fp16, as the logits GEMM reads them).
template <typename T>
__global__ void __launch_bounds__(256) ce_shift_kernel(const T* __restrict__ H, int64_t h_ld,
                                                       const T* __restrict__ W, int64_t w_ld,
                                                       const int64_t* __restrict__ targets,
                                                       int rows, int vocab, int dim,
                                                       int64_t vocab_offset, float* __restrict__ shift,
                                                       int* __restrict__ flag) {
  if (blockIdx.x == 0 && threadIdx.x == 0) *flag = 0;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t tg = targets[row];
  const int64_t t = tg - vocab_offset;
  const int64_t j = (t >= 0 && t < vocab) ? t : 0;
  const T* h = H + (int64_t)row * h_ld;
  const T* w = W + j * w_ld;
  float acc = 0.f;
  for (int k = lane * 8; k < dim; k += 256) {
    const Vec16<T> a = ld16(h + k), b = ld16(w + k);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(Cvt<T>::to_f(a.v[i]), Cvt<T>::to_f(b.v[i]), acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) shift[row] = acc + kShiftMargin;
}

// After the logits GEMM, per row: merge the tile records (metrics), then the
// gradient factors of the shifted exponentials:
//   s = exp(c - lse) / denominator (0 for ignored rows), E[t] = (p_t - 1) exp(lse - c)
// so that s * E is the row of dlogits. When the GEMM raised the overflow
// flag every row takes c = lse (s = 1 / denominator) and the gated second
// logits GEMM rewrites E, the target entries included. With hs set, also
// hs[row] = s * hidden[row] (the dW GEMM's scaled operand).
// 8 rows per block of 512 threads: thread (warp w, lane l) merges records
// j = g, g + 64, ... of row r0 + (l & 7), g = 4 w + (l >> 3), ten loads in
// flight at a time, so each load instruction of a warp reads four runs of 8
// consecutive records (128 B) of the [record][row] layout; the 64 partial
// states of a row are then merged in a fixed order (8 x 8). The block's
// hidden rows (for hs) are copied to shared memory by cp.async before the
// records are read, so their latency overlaps the merge without holding
// registers (the kernel stays at two blocks per SM).
constexpr int kStatRows = 8;
constexpr int kStatBatch = 10;
constexpr int kStatHidMax = 2048;  // dim up to which the hidden rows are staged in shared memory
template <typename T>  // the hidden rows' type (bf16 or fp16); hs is bf16
__global__ void __launch_bounds__(512, 2) ce_stats_kernel(
    const float4* __restrict__ partials, int n_tiles, const float* __restrict__ zt,
    const int64_t* __restrict__ targets, int rows, int vocab, float inv_den, int64_t ignore_index,
    float* __restrict__ losses, float* __restrict__ entropies, int32_t* __restrict__ correct,
    bf16* __restrict__ E, int64_t ld_e, float* __restrict__ shift, float* __restrict__ rscale,
    const int* __restrict__ flag, const T* __restrict__ hidden, int64_t h_ld,
    bf16* __restrict__ hs, int dim) {
  constexpr int kGroups = 512 / kStatRows;
  __shared__ SoftmaxState part[kGroups][kStatRows + 1];
  __shared__ SoftmaxState part2[8][kStatRows + 1];
  __shared__ float s_scale[kStatRows];
  __shared__ __align__(16) T hid[kStatRows * kStatHidMax];
  const int r0 = blockIdx.x * kStatRows;
  const int lr = threadIdx.x % kStatRows, g = threadIdx.x / kStatRows;
  const int nvec = dim / 8;
  const bool hid_smem = hs && dim <= kStatHidMax;
  // the finalizing threads' row inputs, loaded before the records
  int64_t pre_t = 0;
  float pre_z = 0.f, pre_c = 0.f;
  int pre_flag = 0;
  if (threadIdx.x < kStatRows && r0 + (int)threadIdx.x < rows) {
    const int row = r0 + threadIdx.x;
    pre_t = targets[row];
    pre_z = zt[row];  // meaningful only when the target is in range
    if (E) {
      pre_c = shift[row];
      pre_flag = *flag;
    }
  }
  if (hid_smem) {
    for (int i = threadIdx.x; i < kStatRows * nvec; i += blockDim.x) {
      const int rr = i / nvec;
      if (r0 + rr >= rows) break;  // i only grows
      const int k = (i - rr * nvec) * 8;
      const T* src = hidden + (int64_t)(r0 + rr) * h_ld + k;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(hid + rr * dim + k)),
                   "l"(src)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  {
    const int row = r0 + lr;
    SoftmaxState st = sm_init();
    if (row < rows) {
      for (int j0 = g; j0 < n_tiles; j0 += kStatBatch * kGroups) {
        float4 p[kStatBatch];
#pragma unroll
        for (int i = 0; i < kStatBatch; ++i) {
          const int j = j0 + i * kGroups;
          p[i] = j < n_tiles ? partials[(int64_t)j * rows + row]
                             : make_float4(-INFINITY, 0.f, 0.f, __int_as_float(0x7fffffff));
        }
#pragma unroll
        for (int i = 0; i < kStatBatch; ++i)
          st = sm_merge(st, SoftmaxState{p[i].x, p[i].y, p[i].z, __float_as_int(p[i].w)});
      }
    }
    part[g][lr] = st;
  }
  __syncthreads();
  if (threadIdx.x < 8 * kStatRows) {
    const int sub = threadIdx.x / kStatRows;
    SoftmaxState st = part[sub * (kGroups / 8)][lr];
    for (int i = 1; i < kGroups / 8; ++i) st = sm_merge(st, part[sub * (kGroups / 8) + i][lr]);
    part2[sub][lr] = st;
  }
  __syncthreads();
  if (threadIdx.x < kStatRows && r0 + (int)threadIdx.x < rows) {
    const int row = r0 + threadIdx.x;
    SoftmaxState r = part2[0][threadIdx.x];
    for (int i = 1; i < 8; ++i) r = sm_merge(r, part2[i][threadIdx.x]);
    const int64_t t = pre_t;
    const bool ignored = (t == ignore_index);
    const float safe_s = fmaxf(r.s, 1e-12f);
    const float lse = r.m + logf(safe_s);
    const bool in_range = (t >= 0 && t < vocab);
    const float z_t = in_range ? pre_z : 0.f;
    float loss = ignored ? 0.f : (lse - z_t);
    float ent = fmaxf(0.f, lse - r.w / safe_s);
    if (!isfinite(loss)) loss = 0.f;
    if (!isfinite(ent)) ent = 0.f;
    losses[row] = loss;
    entropies[row] = ent;
    correct[row] = (!ignored && in_range && r.idx == static_cast<int>(t)) ? 1 : 0;
    if (E) {
      float sc = 0.f;
      if (pre_flag) shift[row] = lse;  // every row: the fallback GEMM reads it
      if (!ignored) {
        if (pre_flag) {
          sc = inv_den;
        } else {
          const float c = pre_c;
          sc = fast_exp2((c - lse) * kLog2e) * inv_den;
          if (in_range) {
            const float q = fast_exp2((z_t - lse) * kLog2e) - 1.f;
            E[(int64_t)row * ld_e + t] = __float2bfloat16_rn(q * fast_exp2((lse - c) * kLog2e));
          }
        }
      }
      rscale[row] = sc;
      s_scale[threadIdx.x] = sc;
    }
  }
  if (!hs) return;  // block-uniform
  if (hid_smem) asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  for (int i = threadIdx.x; i < kStatRows * nvec; i += blockDim.x) {
    const int rr = i / nvec;
    const int row = r0 + rr;
    if (row >= rows) break;  // i only grows
    const int k = (i - rr * nvec) * 8;
    const float sc = s_scale[rr];
    const Vec16<T> a = hid_smem ? *reinterpret_cast<const Vec16<T>*>(hid + rr * dim + k)
                                : ld16(hidden + (int64_t)row * h_ld + k);
    Vec16<bf16> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.v[e] = __float2bfloat16_rn(sc * Cvt<T>::to_f(a.v[e]));
    st16(hs + (int64_t)row * dim + k, o);
  }
}

// hs[row] = rscale[row] * hidden[row] (bf16; hidden bf16 or fp16), one block per row.
template <typename T>
__global__ void __launch_bounds__(256) ce_scale_rows_kernel(const T* __restrict__ hidden,
                                                            int64_t h_ld,
                                                            const float* __restrict__ rscale,
                                                            int dim, bf16* __restrict__ hs) {
  const int row = blockIdx.x;
  const float sc = rscale[row];
  const T* hrow = hidden + (int64_t)row * h_ld;
  bf16* orow = hs + (int64_t)row * dim;
  for (int k = threadIdx.x * 8; k < dim; k += blockDim.x * 8) {
    const Vec16<T> a = ld16(hrow + k);
    Vec16<bf16> o;
#pragma unroll
    for (int i = 0; i < 8; ++i) o.v[i] = __float2bfloat16_rn(sc * Cvt<T>::to_f(a.v[i]));
    st16(orow + k, o);
  }
}

// sums[0] = sum of losses, sums[1] = number of hits; one block, fixed order.
__global__ void __launch_bounds__(1024) ce_sums_kernel(const float* __restrict__ losses,
                                                       const int32_t* __restrict__ correct,
                                                       int rows, float* __restrict__ sums) {
  __shared__ float sl[32], sc[32];
  float a = 0.f, b = 0.f;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    a += losses[i];
    b += static_cast<float>(correct[i]);
  }
  a = warp_sum(a);
  b = warp_sum(b);
  if ((threadIdx.x & 31) == 0) {
    sl[threadIdx.x >> 5] = a;
    sc[threadIdx.x >> 5] = b;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ta = 0.f, tb = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
      ta += sl[i];
      tb += sc[i];
    }
    sums[0] = ta;
    sums[1] = tb;
  }
}

// out[m, n] = row_scale[m] * sum_s ws[s][m][n] (fixed order over s; no
// row_scale: 1), stored as OutT. cols % 4 == 0.
template <typename OutT>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t slice,
                                     int rows, int cols, OutT* __restrict__ out, int64_t ldo,
                                     const float* __restrict__ row_scale) {
  const int64_t n4 = (int64_t)rows * cols / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 4;
    float4 acc = *reinterpret_cast<const float4*>(ws + e);
    for (int s = 1; s < splits; ++s) {
      float4 v = *reinterpret_cast<const float4*>(ws + s * slice + e);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const int64_t r = e / cols, c = e % cols;
    if (row_scale) {
      const float k = row_scale[r];
      acc.x *= k;
      acc.y *= k;
      acc.z *= k;
      acc.w *= k;
    }
    OutT* o = out + r * ldo + c;
    o[0] = Cvt<OutT>::from_f(acc.x);
    o[1] = Cvt<OutT>::from_f(acc.y);
    o[2] = Cvt<OutT>::from_f(acc.z);
    o[3] = Cvt<OutT>::from_f(acc.w);
  }
}

// ------------------------------------------------- vocab-parallel kernels ---
// Per row (one warp each): merge this shard's tile states into one record
// {max, sum exp, sum z*exp, global argmax (int bits), target logit or 0}.
__global__ void __launch_bounds__(256) ce_shard_state_kernel(
    const float4* __restrict__ partials, int n_tiles, const float* __restrict__ zt,
    const int64_t* __restrict__ targets, int rows, int vocab_shard, int64_t vocab_offset,
    float* __restrict__ states) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  SoftmaxState st = sm_init();
  for (int j = lane; j < n_tiles; j += 32) {
    float4 p = partials[(int64_t)j * rows + row];
    st = sm_merge(st, SoftmaxState{p.x, p.y, p.z, __float_as_int(p.w)});
  }
  st = sm_warp_reduce(st);
  if (lane == 0) {
    const int64_t t = targets[row] - vocab_offset;
    float* o = states + (int64_t)row * 5;
    o[0] = st.m;
    o[1] = st.s;
    o[2] = st.w;
    o[3] = __int_as_float(static_cast<int>(st.idx + vocab_offset));
    o[4] = (t >= 0 && t < vocab_shard) ? zt[row] : 0.f;
  }
}

// Per row (one thread each): merge the ranks' records in rank order (ties keep
// the smaller global index), then the row metrics and the global lse.
__global__ void __launch_bounds__(256) ce_combine_kernel(
    const float* __restrict__ states, int nranks, int64_t rank_stride,
    const int64_t* __restrict__ targets, int rows, int64_t vocab_total, int64_t ignore_index,
    float* __restrict__ losses, float* __restrict__ entropies, int32_t* __restrict__ correct,
    float* __restrict__ lse_out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  SoftmaxState st = sm_init();
  float z_t = 0.f;
  for (int r = 0; r < nranks; ++r) {
    const float* o = states + r * rank_stride + (int64_t)row * 5;
    st = sm_merge(st, SoftmaxState{o[0], o[1], o[2], __float_as_int(o[3])});
    z_t += o[4];
  }
  const int64_t t = targets[row];
  const bool ignored = t == ignore_index;
  const bool in_range = t >= 0 && t < vocab_total;
  const float safe_s = fmaxf(st.s, 1e-12f);
  const float lse = st.m + logf(safe_s);
  float loss = ignored ? 0.f : lse - (in_range ? z_t : 0.f);
  float ent = fmaxf(0.f, lse - st.w / safe_s);
  if (!isfinite(loss)) loss = 0.f;
  if (!isfinite(ent)) ent = 0.f;
  losses[row] = loss;
  entropies[row] = ent;
  correct[row] = (!ignored && in_range && st.idx == static_cast<int>(t)) ? 1 : 0;
  lse_out[row] = lse;
}

// Gradient factors of one shard's shifted exponentials from the global lse,
// one warp per row: s = exp(c - lse) / denominator (0 for ignored rows),
// E[t] = (p_t - 1) exp(lse - c) when the target is in the shard, and with hs
// set hs[row] = s * hidden[row]. When the shard's logits GEMM raised the
// overflow flag every row takes c = lse and the gated second GEMM rewrites E.
// T: the hidden rows' type (bf16 or fp16); hs is bf16.
template <typename T>
__global__ void __launch_bounds__(256) ce_vp_grad_kernel(
    const float* __restrict__ lse, const float* __restrict__ zt, const int64_t* __restrict__ targets,
    int rows, int vocab_shard, int64_t vocab_offset, float inv_den, int64_t ignore_index,
    bf16* __restrict__ E, int64_t ld_e, float* __restrict__ shift, float* __restrict__ rscale,
    const int* __restrict__ flag, const T* __restrict__ hidden, int64_t h_ld,
    bf16* __restrict__ hs, int dim) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float sc = 0.f;
  if (lane == 0) {
    const int64_t tg = targets[row];
    const float l = lse[row];
    const bool flagged = *flag != 0;
    if (flagged) shift[row] = l;  // every row: the fallback GEMM reads it
    if (tg != ignore_index) {
      if (flagged) {
        sc = inv_den;
      } else {
        const float c = shift[row];
        sc = fast_exp2((c - l) * kLog2e) * inv_den;
        const int64_t t = tg - vocab_offset;
        if (t >= 0 && t < vocab_shard) {
          const float q = fast_exp2((zt[row] - l) * kLog2e) - 1.f;
          E[(int64_t)row * ld_e + t] = __float2bfloat16_rn(q * fast_exp2((l - c) * kLog2e));
        }
      }
    }
    rscale[row] = sc;
  }
  if (!hs) return;
  sc = __shfl_sync(0xffffffffu, sc, 0);
  const T* hrow = hidden + (int64_t)row * h_ld;
  bf16* orow = hs + (int64_t)row * dim;
  for (int k = lane * 8; k < dim; k += 256) {
    const Vec16<T> a = ld16(hrow + k);
    Vec16<bf16> o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.v[e] = __float2bfloat16_rn(sc * Cvt<T>::to_f(a.v[e]));
    st16(orow + k, o);
  }
}

// ------------------------------------------------------- stage events ------
static thread_local cudaEvent_t g_stage_events[8];
static thread_local int g_n_stage_events = 0;

static void mark_stage(int i, cudaStream_t s) {
  if (i < g_n_stage_events && g_stage_events[i]) cudaEventRecord(g_stage_events[i], s);
}

// ---------------------------------------------------- workspace layout -----
struct CEWorkspace {
  int64_t ld_logits;
  int n_vtiles;
  int n_parts;  // online-softmax records per row (vocab tiles x epilogue column groups)
  int splits;  // dX vocabulary splits
  size_t off_logits, off_partials, off_zt, off_splitk;
  size_t off_shift, off_rscale, off_flag, off_hs;  // shifted-exponential gradient state
  size_t total;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Vocabulary splits of the dX GEMM (1..16, >= 16 k-blocks per unit). Units
// are (m tile, n tile, split); the estimated time of a split count is
//   waves x k-blocks per unit           (one k-block of a tile ~ 512 tensor
//                                        cycles ~ 0.28 us on every worker)
//   + fp32 partial bytes re-read by the reduce, at HBM speed
// (0.28 us of HBM ~ 1.8 MB), and the cheapest count wins.
static int choose_splits(int64_t rows, int64_t dim, int64_t vocab, int sms) {
  const int64_t tiles = m_tiles(rows) * ((dim + kBN - 1) / kBN);
  const int64_t workers = use_pairs() ? sms / 2 : sms;
  const int64_t kb = (vocab + BK - 1) / BK;
  int64_t s_max = kb / 16;
  if (s_max > 16) s_max = 16;
  if (s_max < 1) s_max = 1;
  constexpr double kBytesPerKBlock = 1.8e6;
  int best = 1;
  double best_cost = 0.0;
  for (int64_t s = 1; s <= s_max; ++s) {
    const int64_t units = tiles * s;
    const int64_t waves = (units + workers - 1) / workers;
    double cost = static_cast<double>(waves * ((kb + s - 1) / s));
    if (s > 1) cost += static_cast<double>(s * rows * dim * 4) / kBytesPerKBlock;
    if (s == 1 || cost < best_cost) {
      best_cost = cost;
      best = static_cast<int>(s);
    }
  }
  return best;
}

static CEWorkspace ce_layout(int64_t rows, int64_t vocab, int64_t dim) {
  CEWorkspace w;
  w.ld_logits = (vocab + 7) / 8 * 8;
  w.n_vtiles = static_cast<int>((vocab + kBN - 1) / kBN);
  w.n_parts = w.n_vtiles * (kEpiWarps / 4);
  w.splits = choose_splits(rows, dim, vocab, num_sms());
  size_t off = 0;
  w.off_logits = off;
  off = align_up(off + (size_t)rows * w.ld_logits * 2, 256);
  w.off_partials = off;
  off = align_up(off + (size_t)w.n_parts * rows * 16, 256);
  w.off_zt = off;
  off = align_up(off + (size_t)rows * 4, 256);
  w.off_splitk = off;
  off = align_up(off + (size_t)w.splits * rows * dim * 4, 256);
  w.off_shift = off;
  off = align_up(off + (size_t)rows * 4, 256);
  w.off_rscale = off;
  off = align_up(off + (size_t)rows * 4, 256);
  w.off_flag = off;
  off = align_up(off + 4, 256);
  w.off_hs = off;
  off = align_up(off + (size_t)rows * dim * 2, 256);
  w.total = off;
  return w;
}

// dH[M, D] = diag(row_scale) dL W: A = dlogits (or shifted exponentials)
// K-major, B = W MN-major. With `splits` > 1 the vocabulary is split into
// fp32 slices reduced in a fixed order (the row scale applied there);
// otherwise the GEMM epilogue writes dH directly. dh_dtype: SOUP_BF16 or SOUP_F32.
static int dx_gemm(const bf16* L, int64_t ld_logits, const void* weight, int64_t w_ld, int M, int V,
                   int D, int splits, float* splitk, void* dh, int dh_dtype, cudaStream_t stream,
                   int gemm_stage = -1, const float* row_scale = nullptr) {
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_operand_map(&ma, L, false, M, V, ld_logits, BM))) return rc;
  if ((rc = make_operand_map(&mb, weight, true, D, V, w_ld, 64))) return rc;
  Sched sc{m_tiles(M), (D + kBN - 1) / kBN, splits, (V + BK - 1) / BK, 1};
  // last vocabulary split first: the logits GEMM (which runs over the vocab in
  // order) leaves the end of dL / E and of W in L2; the last split run is then
  // the vocab's start, where the dW GEMM begins
  sc.rev_split = 1;
  const bool bf = dh_dtype == SOUP_BF16;
  if (splits == 1) {
    const int vec = (aligned16(dh) && (D * (bf ? 2 : 4)) % 16 == 0) ? 1 : 0;
    CUtensorMap mc = ma;
    const int tma = (bf && vec && make_store_map(&mc, dh, D, M, D) == SOUP_OK) ? 1 : 0;
    EpiStore<kBN>::Params ep{dh, D, 0, nullptr, 1.f, bf ? 1 : 0, 0, vec, M, D, nullptr, tma,
                             row_scale};
    rc = launch_gemm<false, true, EpiStore<kBN>>(ma, mb, mc, sc, ep, stream);
    if (!rc && gemm_stage >= 0) mark_stage(gemm_stage, stream);
    return rc;
  }
  EpiStore<kBN>::Params ep{splitk, D, (int64_t)M * D, nullptr, 1.f, 0, 0, 1, M, D};
  if ((rc = launch_gemm<false, true, EpiStore<kBN>>(ma, mb, ma, sc, ep, stream))) return rc;
  if (gemm_stage >= 0) mark_stage(gemm_stage, stream);
  const int64_t n4 = (int64_t)M * D / 4;
  int blocks = static_cast<int>((n4 + 255) / 256);
  if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
  if (bf)
    splitk_reduce_kernel<bf16><<<blocks, 256, 0, stream>>>(splitk, splits, (int64_t)M * D, M, D,
                                                          static_cast<bf16*>(dh), D, row_scale);
  else
    splitk_reduce_kernel<float><<<blocks, 256, 0, stream>>>(splitk, splits, (int64_t)M * D, M, D,
                                                           static_cast<float*>(dh), D, row_scale);
  return launch_status();
}

// dW[V, D] (+)= scale * dL^T H: A = dlogits (or shifted exponentials, with H
// already scaled by the row factors) read MN-major, B = hidden MN-major.
static int dweight_gemm(const bf16* L, int64_t ld_logits, const void* hidden, int64_t h_ld, int M,
                        int V, int D, const float* scale, void* dweight, int dw_dtype,
                        int accumulate, cudaStream_t stream) {
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_operand_map(&ma, L, true, V, M, ld_logits, 64))) return rc;
  if ((rc = make_operand_map(&mb, hidden, true, D, M, h_ld, 64))) return rc;
  Sched sc{m_tiles(V), (D + kBN - 1) / kBN, 1, (M + BK - 1) / BK, 1};
  const int es = dw_dtype == SOUP_BF16 ? 2 : 4;
  const int vec = (aligned16(dweight) && (D * es) % 16 == 0) ? 1 : 0;
  CUtensorMap mc = ma;
  const int tma = (dw_dtype == SOUP_BF16 && !accumulate && vec &&
                   make_store_map(&mc, dweight, D, V, D) == SOUP_OK) ? 1 : 0;
  EpiStore<kBN>::Params ep{dweight, D, 0, scale, 1.f, dw_dtype == SOUP_BF16 ? 1 : 0,
                           accumulate ? 1 : 0, vec, V, D, nullptr, tma};
  return launch_gemm<true, true, EpiStore<kBN>>(ma, mb, mc, sc, ep, stream);
}

// Launch helpers shared by the entry points below (operand type T of the
// hidden rows and the weight: bf16 or fp16).
template <typename T>
static int launch_shift(const void* hidden, int64_t h_ld, const void* weight, int64_t w_ld,
                        const int64_t* targets, int M, int V, int D, int64_t vocab_offset,
                        float* shift, int* flag, cudaStream_t stream) {
  ce_shift_kernel<T><<<(M + 7) / 8, 256, 0, stream>>>(
      static_cast<const T*>(hidden), h_ld, static_cast<const T*>(weight), w_ld, targets, M, V, D,
      vocab_offset, shift, flag);
  return launch_status();
}

static int check_in_dtype(const char* fn, int in_dtype, const void* weight_bwd, bool need_dx) {
  if (in_dtype != SOUP_BF16 && in_dtype != SOUP_F16) {
    char msg[160];
    snprintf(msg, sizeof(msg), "%s: in_dtype must be BF16 or F16", fn);
    set_last_error(msg);
    return SOUP_ERR_INVALID;
  }
  if (in_dtype == SOUP_F16 && need_dx && !weight_bwd) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "%s: fp16 operands need weight_bwd, a bf16 copy of the weight for the dX GEMM", fn);
    set_last_error(msg);
    return SOUP_ERR_INVALID;
  }
  return SOUP_OK;
}

}  // namespace tc
}  // namespace soup

using namespace soup;
using namespace soup::tc;

extern "C" {

size_t soup_ce_linear_workspace_bytes(int64_t rows, int64_t vocab, int64_t dim) {
  if (rows <= 0 || vocab <= 0 || dim <= 0) return 0;
  return ce_layout(rows, vocab, dim).total;
}

int soup_ce_linear(const void* hidden, int64_t h_ld, const void* weight, int64_t w_ld, int in_dtype,
                   const void* weight_bwd, int64_t wb_ld, const int64_t* targets, int64_t rows,
                   int64_t vocab, int64_t dim, float denominator, int64_t ignore_index,
                   float* losses, float* entropies, int32_t* correct, float* sums, void* dhidden,
                   int dh_dtype, void* dweight, int dw_dtype, int accumulate_dw, void* workspace,
                   size_t workspace_bytes, void* stream_) {
  if (!hidden || !weight || !targets || !losses || !entropies || !correct || !workspace) {
    set_last_error("soup_ce_linear: null pointer argument");
    return SOUP_ERR_INVALID;
  }
  if (rows <= 0 || vocab <= 0 || dim <= 0 || rows > (1 << 30) || vocab > (1 << 30) ||
      h_ld < dim || w_ld < dim || (weight_bwd && wb_ld < dim)) {
    set_last_error("soup_ce_linear: bad sizes");
    return SOUP_ERR_INVALID;
  }
  if ((dweight && dw_dtype != SOUP_F32 && dw_dtype != SOUP_BF16) ||
      (dhidden && dh_dtype != SOUP_F32 && dh_dtype != SOUP_BF16)) {
    set_last_error("soup_ce_linear: dhidden / dweight dtypes must be F32 or BF16");
    return SOUP_ERR_INVALID;
  }
  int rc = check_in_dtype("soup_ce_linear", in_dtype, weight_bwd, dhidden != nullptr);
  if (rc) return rc;
  const bool f16 = in_dtype == SOUP_F16;
  // the dX GEMM multiplies the bf16 exponentials by a bf16 weight
  const void* wb = f16 ? weight_bwd : weight;
  const int64_t wbl = f16 ? wb_ld : w_ld;
  if (!tma_ok(hidden, h_ld) || !tma_ok(weight, w_ld) || (dhidden && !tma_ok(wb, wbl)) ||
      (dim % 8) != 0) {
    set_last_error("soup_ce_linear: hidden/weight need 16-byte aligned rows and dim % 8 == 0");
    return SOUP_ERR_UNSUPPORTED;
  }
  CEWorkspace w = ce_layout(rows, vocab, dim);
  if (workspace_bytes < w.total || !aligned16(workspace)) {
    set_last_error("soup_ce_linear: workspace too small or misaligned");
    return SOUP_ERR_WORKSPACE;
  }
  cudaStream_t stream = as_stream(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  bf16* L = reinterpret_cast<bf16*>(ws + w.off_logits);
  float4* partials = reinterpret_cast<float4*>(ws + w.off_partials);
  float* zt = reinterpret_cast<float*>(ws + w.off_zt);
  float* splitk = reinterpret_cast<float*>(ws + w.off_splitk);
  float* shift = reinterpret_cast<float*>(ws + w.off_shift);
  float* rscale = reinterpret_cast<float*>(ws + w.off_rscale);
  int* flag = reinterpret_cast<int*>(ws + w.off_flag);
  bf16* hs = reinterpret_cast<bf16*>(ws + w.off_hs);
  const bool need_grad = dhidden || dweight;
  const int M = static_cast<int>(rows), V = static_cast<int>(vocab), D = static_cast<int>(dim);
  const float inv_den = 1.f / (denominator > 0.f ? denominator : 1.f);

  // 0. row shifts of the stored exponentials (gradient only)
  if (need_grad) {
    rc = f16 ? launch_shift<__half>(hidden, h_ld, weight, w_ld, targets, M, V, D, 0, shift, flag,
                                    stream)
             : launch_shift<bf16>(hidden, h_ld, weight, w_ld, targets, M, V, D, 0, shift, flag,
                                  stream);
    if (rc) return rc;
  }
  // 1. logits GEMM + online-softmax epilogue (+ E = exp(z - shift) stored)
  CUtensorMap ma, mb, mc;
  Sched sc{m_tiles(M), w.n_vtiles, 1, (D + BK - 1) / BK, 0};
  sc.ab_f16 = f16 ? 1 : 0;
  EpiCE<kBN>::Params ep{targets, partials, zt, need_grad ? L : nullptr, w.ld_logits, 0, M, V, 0,
                        need_grad ? shift : nullptr, flag, 0, 1, ignore_index};
  {
    if ((rc = make_operand_map(&ma, hidden, false, rows, dim, h_ld, BM, f16))) return rc;
    if ((rc = make_operand_map(&mb, weight, false, vocab, dim, w_ld, b_box_rows(), f16))) return rc;
    mc = ma;
    ep.tma = (need_grad && make_store_map(&mc, L, V, M, w.ld_logits) == SOUP_OK) ? 1 : 0;
    if ((rc = launch_gemm<false, false, EpiCE<kBN>>(ma, mb, mc, sc, ep, stream))) return rc;
    mark_stage(0, stream);
  }
  // 2. metrics, gradient row factors and target entries (+ hs for dW)
  {
    const unsigned blocks = (M + kStatRows - 1) / kStatRows;
    if (f16)
      ce_stats_kernel<__half><<<blocks, 512, 0, stream>>>(
          partials, w.n_parts, zt, targets, M, V, inv_den, ignore_index, losses, entropies, correct,
          need_grad ? L : nullptr, w.ld_logits, shift, rscale, flag,
          static_cast<const __half*>(hidden), h_ld, dweight ? hs : nullptr, D);
    else
      ce_stats_kernel<bf16><<<blocks, 512, 0, stream>>>(
          partials, w.n_parts, zt, targets, M, V, inv_den, ignore_index, losses, entropies, correct,
          need_grad ? L : nullptr, w.ld_logits, shift, rscale, flag,
          static_cast<const bf16*>(hidden), h_ld, dweight ? hs : nullptr, D);
    if ((rc = launch_status())) return rc;
    if (need_grad) {
      // overflow fallback: the same GEMM with shift = lse, run only when the
      // flag is set (otherwise every CTA returns at entry)
      Sched sc2 = sc;
      sc2.gate = flag;
      EpiCE<kBN>::Params ep2 = ep;
      ep2.onehot = 1;
      if ((rc = launch_gemm<false, false, EpiCE<kBN>>(ma, mb, mc, sc2, ep2, stream))) return rc;
    }
    mark_stage(1, stream);
  }
  if (sums) {
    ce_sums_kernel<<<1, 1024, 0, stream>>>(losses, correct, M, sums);
    if ((rc = launch_status())) return rc;
    mark_stage(2, stream);
  }
  // 4. dH = diag(s) E W  (split along the vocab)
  if (dhidden) {
    if ((rc = dx_gemm(L, w.ld_logits, wb, wbl, M, V, D, w.splits, splitk, dhidden, dh_dtype,
                      stream, 3, rscale)))
      return rc;
    mark_stage(4, stream);
  }
  // 5. dW = E^T diag(s) H
  if (dweight) {
    if ((rc = dweight_gemm(L, w.ld_logits, hs, D, M, V, D, nullptr, dweight, dw_dtype,
                           accumulate_dw, stream)))
      return rc;
    mark_stage(5, stream);
  }
  return SOUP_OK;
}

int soup_ce_linear_dweight(void* workspace, size_t workspace_bytes, const void* hidden,
                           int64_t h_ld, int in_dtype, int64_t rows, int64_t vocab, int64_t dim,
                           const float* grad_scale, void* dweight, int dw_dtype, int accumulate_dw,
                           void* stream) {
  if (!workspace || !hidden || !dweight || rows <= 0 || vocab <= 0 || dim <= 0 ||
      rows > (1 << 30) || vocab > (1 << 30) || h_ld < dim) {
    set_last_error("soup_ce_linear_dweight: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (dw_dtype != SOUP_F32 && dw_dtype != SOUP_BF16) {
    set_last_error("soup_ce_linear_dweight: dweight dtype must be F32 or BF16");
    return SOUP_ERR_INVALID;
  }
  int rc = check_in_dtype("soup_ce_linear_dweight", in_dtype, nullptr, false);
  if (rc) return rc;
  if (!tma_ok(hidden, h_ld) || (dim % 8) != 0) {
    set_last_error("soup_ce_linear_dweight: hidden needs 16-byte aligned rows and dim % 8 == 0");
    return SOUP_ERR_UNSUPPORTED;
  }
  CEWorkspace w = ce_layout(rows, vocab, dim);
  if (workspace_bytes < w.total || !aligned16(workspace)) {
    set_last_error("soup_ce_linear_dweight: workspace too small or misaligned");
    return SOUP_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const bf16* L = reinterpret_cast<const bf16*>(ws + w.off_logits);
  const float* rscale = reinterpret_cast<const float*>(ws + w.off_rscale);
  bf16* hs = reinterpret_cast<bf16*>(ws + w.off_hs);
  cudaStream_t st = as_stream(stream);
  if (in_dtype == SOUP_F16)
    ce_scale_rows_kernel<__half><<<static_cast<unsigned>(rows), 256, 0, st>>>(
        static_cast<const __half*>(hidden), h_ld, rscale, static_cast<int>(dim), hs);
  else
    ce_scale_rows_kernel<bf16><<<static_cast<unsigned>(rows), 256, 0, st>>>(
        static_cast<const bf16*>(hidden), h_ld, rscale, static_cast<int>(dim), hs);
  rc = launch_status();
  if (rc) return rc;
  return dweight_gemm(L, w.ld_logits, hs, dim, static_cast<int>(rows), static_cast<int>(vocab),
                      static_cast<int>(dim), grad_scale, dweight, dw_dtype, accumulate_dw, st);
}

// ------------------------------------------------------ vocab-parallel CE --
size_t soup_ce_vp_workspace_bytes(int64_t rows, int64_t vocab_shard, int64_t dim) {
  if (rows <= 0 || vocab_shard <= 0 || dim <= 0) return 0;
  return ce_layout(rows, vocab_shard, dim).total;
}

int soup_ce_vp_forward(const void* hidden, int64_t h_ld, const void* weight_shard, int64_t w_ld,
                       int in_dtype, const int64_t* targets, int64_t rows, int64_t vocab_shard,
                       int64_t vocab_offset, int64_t dim, float* states, void* workspace,
                       size_t workspace_bytes, void* stream_) {
  if (!hidden || !weight_shard || !targets || !states || !workspace || rows <= 0 ||
      vocab_shard <= 0 || dim <= 0 || rows > (1 << 30) || vocab_shard > (1 << 30) ||
      vocab_offset < 0 || h_ld < dim || w_ld < dim) {
    set_last_error("soup_ce_vp_forward: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (int rc0 = check_in_dtype("soup_ce_vp_forward", in_dtype, nullptr, false)) return rc0;
  const bool f16 = in_dtype == SOUP_F16;
  if (!tma_ok(hidden, h_ld) || !tma_ok(weight_shard, w_ld) || (dim % 8) != 0) {
    set_last_error("soup_ce_vp_forward: hidden/weight need 16-byte aligned rows and dim % 8 == 0");
    return SOUP_ERR_UNSUPPORTED;
  }
  CEWorkspace w = ce_layout(rows, vocab_shard, dim);
  if (workspace_bytes < w.total || !aligned16(workspace)) {
    set_last_error("soup_ce_vp_forward: workspace too small or misaligned");
    return SOUP_ERR_WORKSPACE;
  }
  cudaStream_t stream = as_stream(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  bf16* L = reinterpret_cast<bf16*>(ws + w.off_logits);
  float4* partials = reinterpret_cast<float4*>(ws + w.off_partials);
  float* zt = reinterpret_cast<float*>(ws + w.off_zt);
  float* shift = reinterpret_cast<float*>(ws + w.off_shift);
  int* flag = reinterpret_cast<int*>(ws + w.off_flag);
  const int M = static_cast<int>(rows), V = static_cast<int>(vocab_shard), D = static_cast<int>(dim);
  int rc;
  // row shifts from the shard's own columns
  rc = f16 ? launch_shift<__half>(hidden, h_ld, weight_shard, w_ld, targets, M, V, D, vocab_offset,
                                  shift, flag, stream)
           : launch_shift<bf16>(hidden, h_ld, weight_shard, w_ld, targets, M, V, D, vocab_offset,
                                shift, flag, stream);
  if (rc) return rc;
  CUtensorMap ma, mb;
  if ((rc = make_operand_map(&ma, hidden, false, rows, dim, h_ld, BM, f16))) return rc;
  if ((rc = make_operand_map(&mb, weight_shard, false, vocab_shard, dim, w_ld, b_box_rows(), f16)))
    return rc;
  Sched sc{m_tiles(M), w.n_vtiles, 1, (D + BK - 1) / BK, 0};
  sc.ab_f16 = f16 ? 1 : 0;
  CUtensorMap mc = ma;
  const int tma = make_store_map(&mc, L, V, M, w.ld_logits) == SOUP_OK ? 1 : 0;
  EpiCE<kBN>::Params ep{targets, partials, zt, L, w.ld_logits, vocab_offset, M, V, tma, shift, flag, 0};
  if ((rc = launch_gemm<false, false, EpiCE<kBN>>(ma, mb, mc, sc, ep, stream))) return rc;
  ce_shard_state_kernel<<<(M + 7) / 8, 256, 0, stream>>>(partials, w.n_parts, zt, targets, M, V,
                                                         vocab_offset, states);
  return launch_status();
}

int soup_ce_vp_combine(const float* states_all, int nranks, const int64_t* targets, int64_t rows,
                       int64_t vocab_total, int64_t ignore_index, float* losses, float* entropies,
                       int32_t* correct, float* lse, float* sums, void* stream_) {
  if (!states_all || nranks <= 0 || !targets || !losses || !entropies || !correct || !lse ||
      rows <= 0 || rows > (1 << 30) || vocab_total <= 0) {
    set_last_error("soup_ce_vp_combine: bad arguments");
    return SOUP_ERR_INVALID;
  }
  cudaStream_t stream = as_stream(stream_);
  const int M = static_cast<int>(rows);
  ce_combine_kernel<<<(M + 255) / 256, 256, 0, stream>>>(states_all, nranks, (int64_t)M * 5, targets,
                                                         M, vocab_total, ignore_index, losses,
                                                         entropies, correct, lse);
  int rc = launch_status();
  if (rc || !sums) return rc;
  ce_sums_kernel<<<1, 1024, 0, stream>>>(losses, correct, M, sums);
  return launch_status();
}

int soup_ce_vp_backward(void* workspace, size_t workspace_bytes, const void* hidden, int64_t h_ld,
                        const void* weight_shard, int64_t w_ld, int in_dtype,
                        const void* weight_shard_bwd, int64_t wb_ld, const int64_t* targets,
                        int64_t rows, int64_t vocab_shard, int64_t vocab_offset, int64_t dim,
                        const float* lse, float denominator, int64_t ignore_index,
                        void* dhidden_partial, int dh_dtype, void* dweight_shard, int dw_dtype,
                        int accumulate_dw, void* stream_) {
  if (!workspace || !hidden || !weight_shard || !targets || !lse || rows <= 0 ||
      vocab_shard <= 0 || dim <= 0 || rows > (1 << 30) || vocab_shard > (1 << 30) ||
      h_ld < dim || w_ld < dim || (weight_shard_bwd && wb_ld < dim)) {
    set_last_error("soup_ce_vp_backward: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (int rc0 = check_in_dtype("soup_ce_vp_backward", in_dtype, weight_shard_bwd,
                               dhidden_partial != nullptr))
    return rc0;
  const bool f16 = in_dtype == SOUP_F16;
  const void* wb = f16 ? weight_shard_bwd : weight_shard;
  const int64_t wbl = f16 ? wb_ld : w_ld;
  if ((dhidden_partial && dh_dtype != SOUP_F32 && dh_dtype != SOUP_BF16) ||
      (dweight_shard && dw_dtype != SOUP_F32 && dw_dtype != SOUP_BF16)) {
    set_last_error("soup_ce_vp_backward: gradient dtypes must be F32 or BF16");
    return SOUP_ERR_INVALID;
  }
  if (!tma_ok(hidden, h_ld) || !tma_ok(weight_shard, w_ld) ||
      (dhidden_partial && !tma_ok(wb, wbl)) || (dim % 8) != 0) {
    set_last_error("soup_ce_vp_backward: hidden/weight need 16-byte aligned rows and dim % 8 == 0");
    return SOUP_ERR_UNSUPPORTED;
  }
  CEWorkspace w = ce_layout(rows, vocab_shard, dim);
  if (workspace_bytes < w.total || !aligned16(workspace)) {
    set_last_error("soup_ce_vp_backward: workspace too small or misaligned");
    return SOUP_ERR_WORKSPACE;
  }
  cudaStream_t stream = as_stream(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  bf16* L = reinterpret_cast<bf16*>(ws + w.off_logits);
  float4* partials = reinterpret_cast<float4*>(ws + w.off_partials);
  float* zt = reinterpret_cast<float*>(ws + w.off_zt);
  float* splitk = reinterpret_cast<float*>(ws + w.off_splitk);
  float* shift = reinterpret_cast<float*>(ws + w.off_shift);
  float* rscale = reinterpret_cast<float*>(ws + w.off_rscale);
  int* flag = reinterpret_cast<int*>(ws + w.off_flag);
  bf16* hs = reinterpret_cast<bf16*>(ws + w.off_hs);
  const int M = static_cast<int>(rows), V = static_cast<int>(vocab_shard), D = static_cast<int>(dim);
  const float den = denominator > 0.f ? denominator : 1.f;
  int rc;
  // gradient factors from the global lse (+ s * H for dW)
  if (f16)
    ce_vp_grad_kernel<__half><<<(M + 7) / 8, 256, 0, stream>>>(
        lse, zt, targets, M, V, vocab_offset, 1.f / den, ignore_index, L, w.ld_logits, shift,
        rscale, flag, static_cast<const __half*>(hidden), h_ld, dweight_shard ? hs : nullptr, D);
  else
    ce_vp_grad_kernel<bf16><<<(M + 7) / 8, 256, 0, stream>>>(
        lse, zt, targets, M, V, vocab_offset, 1.f / den, ignore_index, L, w.ld_logits, shift,
        rscale, flag, static_cast<const bf16*>(hidden), h_ld, dweight_shard ? hs : nullptr, D);
  if ((rc = launch_status())) return rc;
  // overflow fallback: the shard's logits GEMM again with shift = lse, only when flagged
  {
    CUtensorMap ma, mb;
    if ((rc = make_operand_map(&ma, hidden, false, rows, dim, h_ld, BM, f16))) return rc;
    if ((rc = make_operand_map(&mb, weight_shard, false, vocab_shard, dim, w_ld, b_box_rows(), f16)))
      return rc;
    Sched sc{m_tiles(M), w.n_vtiles, 1, (D + BK - 1) / BK, 0};
    sc.ab_f16 = f16 ? 1 : 0;
    sc.gate = flag;
    CUtensorMap mc = ma;
    const int tma = make_store_map(&mc, L, V, M, w.ld_logits) == SOUP_OK ? 1 : 0;
    EpiCE<kBN>::Params ep{targets, partials, zt, L, w.ld_logits, vocab_offset, M, V, tma,
                          shift, flag, 1};
    if ((rc = launch_gemm<false, false, EpiCE<kBN>>(ma, mb, mc, sc, ep, stream))) return rc;
  }
  if (dhidden_partial &&
      (rc = dx_gemm(L, w.ld_logits, wb, wbl, M, V, D, w.splits, splitk, dhidden_partial,
                    dh_dtype, stream, -1, rscale)))
    return rc;
  if (dweight_shard)
    return dweight_gemm(L, w.ld_logits, hs, D, M, V, D, nullptr, dweight_shard, dw_dtype,
                        accumulate_dw, stream);
  return SOUP_OK;
}

int soup_set_stage_events(void** events, int n) {
  if (n < 0 || n > 8 || (n > 0 && !events)) {
    set_last_error("soup_set_stage_events: n must be 0..8");
    return SOUP_ERR_INVALID;
  }
  for (int i = 0; i < 8; ++i) g_stage_events[i] = (i < n) ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_n_stage_events = n;
  return SOUP_OK;
}

size_t soup_gemm_stream_k_workspace_bytes(void) {
  const int sms = num_sms();
  return sms >= 2 ? sk_bytes(sms / 2) : 0;
}

int soup_gemm_set_stream_k_workspace(void* ws, size_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64 || (ws && reinterpret_cast<uintptr_t>(ws) % 256 != 0)) {
    set_last_error("soup_gemm_set_stream_k_workspace: workspace must be 256-byte aligned");
    return SOUP_ERR_INVALID;
  }
  if (ws && bytes < soup_gemm_stream_k_workspace_bytes()) {
    set_last_error("soup_gemm_set_stream_k_workspace: smaller than soup_gemm_stream_k_workspace_bytes()");
    return SOUP_ERR_WORKSPACE;
  }
  std::lock_guard<std::mutex> lock(cache_mutex());
  g_sk_ws[dev].ptr = ws;
  g_sk_ws[dev].bytes = ws ? bytes : 0;
  return SOUP_OK;
}

int soup_gemm_set_stream_k_min_saved(int kblocks) {
  if (kblocks < 0) kblocks = kSkMinSavedDefault;
  g_sk_min_saved.store(kblocks, std::memory_order_relaxed);
  return SOUP_OK;
}

int soup_gemm_bf16(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                   int b_mn_major, void* c, int64_t ldc, int c_dtype, int64_t m, int64_t n,
                   int64_t k, float alpha, int accumulate, void* stream_) {
  return soup_gemm_bf16_lora(a, lda, a_mn_major, b, ldb, b_mn_major, nullptr, 0, nullptr, 0, 0,
                             nullptr, c, ldc, c_dtype, m, n, k, alpha, accumulate, stream_);
}

int soup_gemm_bf16_lora(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                        int b_mn_major, const void* a2, int64_t lda2, const void* b2, int64_t ldb2,
                        int64_t r, const void* bias, void* c, int64_t ldc, int c_dtype, int64_t m,
                        int64_t n, int64_t k, float alpha, int accumulate, void* stream_) {
  if (!a || !b || !c || m <= 0 || n <= 0 || k <= 0 || m > (1 << 30) || n > (1 << 30) ||
      k > (1 << 30) || r < 0 || r > 4096 || (r > 0 && (!a2 || !b2))) {
    set_last_error("soup_gemm_bf16: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (c_dtype != SOUP_F32 && c_dtype != SOUP_BF16) {
    set_last_error("soup_gemm_bf16: C dtype must be F32 or BF16");
    return SOUP_ERR_INVALID;
  }
  if ((a_mn_major ? lda < m : lda < k) || (b_mn_major ? ldb < n : ldb < k) || ldc < n ||
      (r > 0 && ((a_mn_major ? lda2 < m : lda2 < r) || (b_mn_major ? ldb2 < n : ldb2 < r)))) {
    set_last_error("soup_gemm_bf16: leading dimension too small");
    return SOUP_ERR_INVALID;
  }
  if (!tma_ok(a, lda) || !tma_ok(b, ldb) || (r > 0 && (!tma_ok(a2, lda2) || !tma_ok(b2, ldb2)))) {
    set_last_error("soup_gemm_bf16: operands need 16-byte aligned rows");
    return SOUP_ERR_UNSUPPORTED;
  }
  CUtensorMap ma, mb, ma2, mb2;
  int rc;
  if ((rc = make_operand_map(&ma, a, a_mn_major != 0, m, k, lda, BM))) return rc;
  if ((rc = make_operand_map(&mb, b, b_mn_major != 0, n, k, ldb, b_box_rows()))) return rc;
  if (r > 0) {
    // the rank-r segment: boxes are 64 deep along K; TMA fills the columns
    // (K-major) or rows (MN-major) beyond r with zeros
    if ((rc = make_operand_map(&ma2, a2, a_mn_major != 0, m, r, lda2, BM))) return rc;
    if ((rc = make_operand_map(&mb2, b2, b_mn_major != 0, n, r, ldb2, b_box_rows()))) return rc;
  } else {
    ma2 = ma;
    mb2 = mb;
  }
  const int es = c_dtype == SOUP_BF16 ? 2 : 4;
  const int vec = (aligned16(c) && (ldc * es) % 16 == 0) ? 1 : 0;
  CUtensorMap mc = ma;
  const int tma = (c_dtype == SOUP_BF16 && !accumulate && vec &&
                   make_store_map(&mc, c, n, m, ldc) == SOUP_OK) ? 1 : 0;
  EpiStore<kBN>::Params ep{c, ldc, 0, nullptr, alpha, c_dtype == SOUP_BF16 ? 1 : 0, accumulate ? 1 : 0,
                           vec, (int)m, (int)n, static_cast<const bf16*>(bias), tma};
  const int mt = m_tiles(m), nt = (int)((n + kBN - 1) / kBN);
  const int kb1 = (int)((k + BK - 1) / BK), kb2 = (int)((r + BK - 1) / BK);
  Sched sc{mt, nt, 1, kb1 + kb2, nt > mt ? 0 : 1, kb2};
  cudaStream_t stream = as_stream(stream_);
  using E = EpiStore<kBN>;
  if (!a_mn_major && !b_mn_major) return launch_gemm<false, false, E>(ma, mb, ma2, mb2, mc, sc, ep, stream);
  if (!a_mn_major && b_mn_major) return launch_gemm<false, true, E>(ma, mb, ma2, mb2, mc, sc, ep, stream);
  if (a_mn_major && !b_mn_major) return launch_gemm<true, false, E>(ma, mb, ma2, mb2, mc, sc, ep, stream);
  return launch_gemm<true, true, E>(ma, mb, ma2, mb2, mc, sc, ep, stream);
}

int soup_gemm_bf16_lora_dswiglu(const void* a, int64_t lda, const void* b, int64_t ldb,
                                const void* a2, int64_t lda2, const void* b2, int64_t ldb2,
                                int64_t r, void* y, int64_t ldy, int64_t m, int64_t inter,
                                int64_t k, void* stream_) {
  if (!a || !b || !y || m <= 0 || inter <= 0 || k <= 0 || m > (1 << 30) || inter > (1 << 29) ||
      k > (1 << 30) || r < 0 || r > 4096 || (r > 0 && (!a2 || !b2))) {
    set_last_error("soup_gemm_bf16_lora_dswiglu: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (inter % (kBN / 2) != 0) {
    set_last_error("soup_gemm_bf16_lora_dswiglu: the intermediate size must be a multiple of 128");
    return SOUP_ERR_UNSUPPORTED;
  }
  if (lda < k || ldb < inter || ldy < 2 * inter || (r > 0 && (lda2 < r || ldb2 < inter))) {
    set_last_error("soup_gemm_bf16_lora_dswiglu: leading dimension too small");
    return SOUP_ERR_INVALID;
  }
  if (!tma_ok(a, lda) || !tma_ok(b, ldb) || (r > 0 && (!tma_ok(a2, lda2) || !tma_ok(b2, ldb2))) ||
      !aligned16(y) || (ldy * 2) % 16 != 0) {
    set_last_error("soup_gemm_bf16_lora_dswiglu: operands need 16-byte aligned rows");
    return SOUP_ERR_UNSUPPORTED;
  }
  CUtensorMap ma, mb, ma2, mb2;
  int rc;
  // dh = a [m, k] b [k, inter] (+ a2 [m, r] b2 [r, inter]): B operands MN-major
  if ((rc = make_operand_map(&ma, a, false, m, k, lda, BM))) return rc;
  if ((rc = make_operand_map(&mb, b, true, inter, k, ldb, b_box_rows()))) return rc;
  if (r > 0) {
    if ((rc = make_operand_map(&ma2, a2, false, m, r, lda2, BM))) return rc;
    if ((rc = make_operand_map(&mb2, b2, true, inter, r, ldb2, b_box_rows()))) return rc;
  } else {
    ma2 = ma;
    mb2 = mb;
  }
  EpiDSwiGLU<kBN>::Params ep{static_cast<bf16*>(y), ldy, (int)m, (int)inter};
  const int mt = m_tiles(m), nt = (int)((inter + kBN - 1) / kBN);
  const int kb1 = (int)((k + BK - 1) / BK), kb2 = (int)((r + BK - 1) / BK);
  Sched sc{mt, nt, 1, kb1 + kb2, nt > mt ? 0 : 1, kb2};
  return launch_gemm<false, true, EpiDSwiGLU<kBN>>(ma, mb, ma2, mb2, ma, sc, ep, as_stream(stream_));
}

int soup_gemm_wait_expiry_check(const void* a, const void* b, void* c, int64_t m, int64_t n,
                                int64_t k, uint64_t wait_ns, void* stream_) {
  if (!a || !b || !c || m <= 0 || n <= 0 || k < 2 * BK || m > (1 << 20) || n > (1 << 20) ||
      k > (1 << 20) || wait_ns < 1000000ull || wait_ns > kWaitNs) {
    set_last_error("soup_gemm_wait_expiry_check: bad arguments (k >= 128, 1 ms <= wait <= 2 s)");
    return SOUP_ERR_INVALID;
  }
  if (!tma_ok(a, k) || !tma_ok(b, k) || !aligned16(c) || (n * 2) % 16 != 0) {
    set_last_error("soup_gemm_wait_expiry_check: operands need 16-byte aligned rows");
    return SOUP_ERR_UNSUPPORTED;
  }
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_operand_map(&ma, a, false, m, k, k, BM))) return rc;
  if ((rc = make_operand_map(&mb, b, false, n, k, k, b_box_rows()))) return rc;
  EpiStore<kBN>::Params ep{c, n, 0, nullptr, 1.f, 1, 0, 1, (int)m, (int)n};
  const int mt = m_tiles(m), nt = (int)((n + kBN - 1) / kBN);
  Sched sc{mt, nt, 1, (int)((k + BK - 1) / BK), nt > mt ? 0 : 1, 0};
  sc.wait_ns = wait_ns;
  sc.withhold = 1;  // the second k-block of every worker's first tile
  return launch_gemm<false, false, EpiStore<kBN>>(ma, mb, ma, mb, ma, sc, ep, as_stream(stream_));
}

int soup_gemm_bf16_lora_swiglu(const void* a, int64_t lda, const void* b, int64_t ldb,
                               const void* a2, int64_t lda2, const void* b2, int64_t ldb2, int64_t r,
                               const void* bias, int mode, void* h, int64_t ldh, void* y, int64_t ldy,
                               int64_t m, int64_t inter, int64_t k, void* stream_) {
  const int64_t n = 2 * inter;
  if (!a || !b || !h || m <= 0 || inter <= 0 || k <= 0 || m > (1 << 30) || n > (1 << 30) ||
      k > (1 << 30) || r < 0 || r > 4096 || (r > 0 && (!a2 || !b2)) || (mode != 0 && mode != 1) ||
      (mode == 1 && !y)) {
    set_last_error("soup_gemm_bf16_lora_swiglu: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (inter % (kBN / 2) != 0) {
    set_last_error("soup_gemm_bf16_lora_swiglu: the intermediate size must be a multiple of 128");
    return SOUP_ERR_UNSUPPORTED;
  }
  if (lda < k || ldb < k || ldh < inter || (y && ldy < n) || (r > 0 && (lda2 < r || ldb2 < r))) {
    set_last_error("soup_gemm_bf16_lora_swiglu: leading dimension too small");
    return SOUP_ERR_INVALID;
  }
  if (!tma_ok(a, lda) || !tma_ok(b, ldb) || (r > 0 && (!tma_ok(a2, lda2) || !tma_ok(b2, ldb2))) ||
      !aligned16(h) || (ldh * 2) % 16 != 0 || (y && (!aligned16(y) || (ldy * 2) % 16 != 0))) {
    set_last_error("soup_gemm_bf16_lora_swiglu: operands need 16-byte aligned rows");
    return SOUP_ERR_UNSUPPORTED;
  }
  CUtensorMap ma, mb, ma2, mb2;
  int rc;
  if ((rc = make_operand_map(&ma, a, false, m, k, lda, BM))) return rc;
  if ((rc = make_operand_map(&mb, b, false, n, k, ldb, b_box_rows()))) return rc;
  if (r > 0) {
    if ((rc = make_operand_map(&ma2, a2, false, m, r, lda2, BM))) return rc;
    if ((rc = make_operand_map(&mb2, b2, false, n, r, ldb2, b_box_rows()))) return rc;
  } else {
    ma2 = ma;
    mb2 = mb;
  }
  EpiSwiGLU<kBN>::Params ep{mode, static_cast<bf16*>(h), ldh, static_cast<bf16*>(y), ldy,
                            static_cast<const bf16*>(bias), (int)m, (int)n};
  const int mt = m_tiles(m), nt = (int)(n / kBN);
  const int kb1 = (int)((k + BK - 1) / BK), kb2 = (int)((r + BK - 1) / BK);
  Sched sc{mt, nt, 1, kb1 + kb2, nt > mt ? 0 : 1, kb2};
  return launch_gemm<false, false, EpiSwiGLU<kBN>>(ma, mb, ma2, mb2, ma, sc, ep, as_stream(stream_));
}

}  // extern "C"
