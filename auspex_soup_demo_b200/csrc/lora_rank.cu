// Rank-r products of the LoRA path on the 5th-generation tensor cores.
//
//   C[m, n] = sum_k A(m, k) * B(n, k),   n <= 64 (a LoRA rank, or the stacked
//                                         rank of a projection group)
//
// The products of a LoRA linear besides its base GEMM are all of this shape:
//   xa  = x  As^T    A = x  [T, in]   (K-major), B = As  [r, in]
//   dxa = dy B       A = dy [T, out]  (K-major), B = B^T [r, out]
//   gA  = s dxa^T x  computed as C = x^T dxa:  A = x  stored [T, in]  (MN-major),
//                                              B = dxa^T [r, T], written transposed
//   gB  = dy^T xa    A = dy stored [T, out] (MN-major), B = xa^T [r, T]
// They move one large operand (the activations or their gradient, 25-300 MB
// at 8192 tokens) against a few KB of factors, so they are HBM-bound: what
// matters is how many bytes each SM keeps in flight. A 128-row tile of A
// streams through a 4-stage TMA ring (16 KB per stage, 128-byte swizzle;
// three CTAs per SM overlap one another's start and end)
// into one tcgen05.mma per 16-deep slice (M = 128, N = n rounded up to 16)
// accumulating in TMEM. When the tiles of A are fewer than the SMs, the K
// range is split over a cluster of up to 16 CTAs; every CTA leaves its fp32
// partial tile in its shared memory and, after a cluster barrier, CTA p sums
// rows [128 p / ks, 128 (p + 1) / ks) of all partials through
// distributed shared memory in rank order (fixed order: bitwise reproducible)
// and writes them: bf16 C and/or its transpose, or an fp32 accumulation into
// gradient buffers (+= alpha * C, optionally transposed, optionally split by
// row blocks into the members of a projection group).
//
//   warp 0     TMA producer (one lane)
//   warp 1     TMEM allocator + MMA issuer (one lane)
//   warps 2-5  epilogue: tcgen05.ld of lane quarter (warp % 4), partial tile,
//              reduction over the cluster, stores
//
// Every mbarrier wait is bounded (soup_set_wait_limit_ns); on expiry the code
// goes to the device error word, the CTA stops issuing, drains what it issued,
// still takes part in both cluster barriers (so no peer waits for it), skips
// its stores and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "soup_common.cuh"
#include "tc_gemm.cuh"

namespace soup {
namespace {

using bf16 = __nv_bfloat16;
using namespace tc;

constexpr int kRankStages = 4;
constexpr int kRankThreads = 192;
constexpr int kRankMaxN = 64;
constexpr int kRankMaxMembers = 4;
constexpr int kErrRankProducer = 0x121;
constexpr int kErrRankMma = 0x122;
constexpr int kErrRankEpilogue = 0x123;
constexpr int kErrRankSmem = 0x124;

template <int NP>
struct RankSmem {
  static constexpr int kABytes = 128 * 64 * 2;  // 128 rows x 64 k, bf16
  static constexpr int kBBytes = NP * 64 * 2;   // NP rows x 64 k (a multiple of 1 KB)
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int kPartStride = NP + 4;  // floats per partial row (16-byte rows, no bank conflicts)
  // the partial tile reuses the stages: written only after every MMA (the
  // last reader of the stages) has completed
  static constexpr int kPart = 0;
  static_assert(128 * kPartStride * 4 <= kRankStages * kStage, "partial tile exceeds the stages");
  static constexpr int kBar = kRankStages * kStage;
  static constexpr int kNumBars = 2 * kRankStages + 1;  // full[S], empty[S], acc_full
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  static constexpr int kBytes = kUsed + 1024;  // + alignment slack
};

struct RankArgs {
  int m, n, k;
  int kb_total;  // 64-deep k-blocks
  int ks;        // CTAs of a cluster, each one part of the K range
  uint64_t wait_ns;
  float alpha;
  // outputs (any combination; g and the member table are exclusive)
  bf16* c;           // C [m, n] bf16, row stride ldc
  int64_t ldc;
  bf16* ct;          // C^T [n, m] bf16, row stride ldct
  int64_t ldct;
  float* g;          // fp32: g[row * ldg + col] += alpha * C (g_trans: g[col * ldg + row])
  int64_t ldg;
  int g_trans;
  // projection-group gradients: rows of C are the members' rows (consecutive
  // blocks, or interleaved blocks of 128: tile t -> member t % nmem); member j
  // takes columns [col_off[j], col_off[j+1]) into gm[j][local row * ldgm[j] + col - col_off[j]]
  int nmem;
  int interleaved;
  int row_off[kRankMaxMembers + 1];
  int col_off[kRankMaxMembers + 1];
  float* gm[kRankMaxMembers];
  int64_t ldgm[kRankMaxMembers];
};

__device__ __forceinline__ uint32_t rank_dynamic_smem() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// 32 lanes x 16 consecutive fp32 columns (no wait; tcgen05.wait::ld follows).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Writes the four columns [col, col + 4) of row `row` of C (fp32 sums s).
__device__ __forceinline__ void rank_emit(const RankArgs& a, int mt, int row, int col, float4 s) {
  const float v[4] = {s.x * a.alpha, s.y * a.alpha, s.z * a.alpha, s.w * a.alpha};
  if (row >= a.m) return;
  if (a.c) {
    bf16* p = a.c + (int64_t)row * a.ldc + col;
    if (col + 4 <= a.n && ((reinterpret_cast<uintptr_t>(p) & 7) == 0)) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]);
      __nv_bfloat162 hi = __floats2bfloat162_rn(v[2], v[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&lo);
      u.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(p) = u;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col + j < a.n) p[j] = __float2bfloat16_rn(v[j]);
    }
  }
  if (a.ct) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < a.n) a.ct[(int64_t)(col + j) * a.ldct + row] = __float2bfloat16_rn(v[j]);
  }
  if (a.g) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (col + j >= a.n) continue;
      float* p = a.g_trans ? a.g + (int64_t)(col + j) * a.ldg + row : a.g + (int64_t)row * a.ldg + col + j;
      *p += v[j];
    }
  }
  if (a.nmem > 0) {
    int j = 0, lrow = 0;
    if (a.interleaved) {
      j = mt % a.nmem;
      lrow = (mt / a.nmem) * 128 + (row - mt * 128);
    } else {
      while (j + 1 < a.nmem && row >= a.row_off[j + 1]) ++j;
      lrow = row - a.row_off[j];
    }
    float* gj = a.gm[j];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int cc = col + q;
      if (cc >= a.col_off[j] && cc < a.col_off[j + 1] && cc < a.n)
        gj[(int64_t)lrow * a.ldgm[j] + (cc - a.col_off[j])] += v[q];
    }
  }
}

// Grid: (m tiles) x ks CTAs, clusters of ks consecutive CTAs along x (one m
// tile per cluster, rank p taking k-blocks [kb_total * p / ks, kb_total * (p+1) / ks)).
// A K-major: map {K, M}, box {64, 128}; A MN-major: map {M, K}, box {64, 64};
// B: map {K, N}, box {64, NP}; all with the 128-byte swizzle.
template <bool A_MN, int NP>
__global__ void __launch_bounds__(kRankThreads, 3)
    rank_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const RankArgs a, int* err) {
  using L = RankSmem<NP>;
  constexpr uint32_t kCols = NP <= 32 ? 32 : 64;
  constexpr uint32_t kIdesc = idesc_bf16(NP, A_MN, false, 128);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if ((uint32_t)(smem - smem_raw) + L::kUsed > rank_dynamic_smem()) {  // grid-uniform
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrRankSmem);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kRankStages + s); };
  const uint32_t acc_bar = bar0 + 8u * (2 * kRankStages);
  float* part = reinterpret_cast<float*>(smem + L::kPart);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = a.ks;
  const int rank = ks > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int mt = blockIdx.x / ks;
  const int kb0 = static_cast<int>((int64_t)a.kb_total * rank / ks);
  const int kb1 = static_cast<int>((int64_t)a.kb_total * (rank + 1) / ks);
  const uint64_t wait_ns = a.wait_ns ? a.wait_ns : kWaitNs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) mbar_init(bar0 + 8u * i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % kRankStages;
        const uint32_t ph = (it / kRankStages) & 1u;
        if (!bounded_wait(empty_bar(s), ph ^ 1u, abort_flag, err, kErrRankProducer, wait_ns)) break;
        const uint32_t a_dst = sbase + s * L::kStage;
        const uint32_t b_dst = a_dst + L::kABytes;
        mbar_arrive_expect_tx(full_bar(s), L::kStage);
        if (A_MN) {
          tma_load_2d(a_dst, &tma_a, full_bar(s), mt * 128, kb * 64);
          tma_load_2d(a_dst + 8192, &tma_a, full_bar(s), mt * 128 + 64, kb * 64);
        } else {
          tma_load_2d(a_dst, &tma_a, full_bar(s), kb * 64, mt * 128);
        }
        tma_load_2d(b_dst, &tma_b, full_bar(s), kb * 64, 0);
      }
      // let the copies still in flight land before the CTA may leave (bounded)
      const int n_wait = it < kRankStages ? it : kRankStages;
      for (int i = 1; i <= n_wait; ++i) {
        const int j = it - i;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(full_bar(j % kRankStages), (j / kRankStages) & 1u) &&
               globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------- MMA issuer ----
      int it = 0;
      bool issued = false;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % kRankStages;
        const uint32_t ph = (it / kRankStages) & 1u;
        if (!bounded_wait(full_bar(s), ph, abort_flag, err, kErrRankMma, wait_ns)) break;
        tc_fence_after();
        const uint32_t a_addr = sbase + s * L::kStage;
        const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                   : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
          tc_mma_bf16(tmem, ad, bd, kIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        issued = true;
        tc_commit(empty_bar(s));
      }
      // the accumulator (or nothing, for an empty K range) is complete
      if (issued) {
        tc_commit(acc_bar);
        // the MMAs are done before TMEM can be freed, also when the epilogue
        // stopped waiting for them (bounded)
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(acc_bar, 0) && globaltimer() - t0 < wait_ns) {
        }
      } else {
        mbar_arrive(acc_bar);
      }
    }
  } else {
    // ------------------------------------------------------ epilogue ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    bool ok = true;
    if (lane == 0) ok = bounded_wait(acc_bar, 0, abort_flag, err, kErrRankEpilogue, wait_ns);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    tc_fence_after();
    float v[NP];
    if (ok && kb1 > kb0) {
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      __syncwarp();
#pragma unroll
      for (int c = 0; c < NP; c += 16) tmem_ld16_nowait(taddr + c, v + c);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    } else {
#pragma unroll
      for (int c = 0; c < NP; ++c) v[c] = 0.f;
    }
    float* prow = part + row * L::kPartStride;
#pragma unroll
    for (int c = 0; c < NP; c += 4)
      *reinterpret_cast<float4*>(prow + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
  }

  // every thread of every CTA of the cluster: the partial tiles are complete
  __syncwarp();
  if (ks > 1) cluster_sync_all();
  else __syncthreads();

  if (warp >= 2 && !*abort_flag) {
    const int t = threadIdx.x - 64;
    const int r0 = 128 * rank / ks, rs = 128 * (rank + 1) / ks - r0;  // rows this CTA reduces and writes
    const int items = rs * (NP / 4);
    const uint32_t part_addr = smem_u32(part);
    for (int item = t; item < items; item += 128) {
      const int rl = item % rs, cg = item / rs;
      const int r = r0 + rl, col = cg * 4;
      const uint32_t off = static_cast<uint32_t>((r * L::kPartStride + col) * 4);
      // eight partials' loads in flight at a time, then added in rank order
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p0 = 0; p0 < ks; p0 += 8) {
        float4 q[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int p = p0 + u;
          q[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (p < ks)
            q[u] = (p == rank) ? *reinterpret_cast<const float4*>(part + r * L::kPartStride + col)
                               : ld_cluster_f4(cluster_addr(part_addr + off, p));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (p0 + u < ks) {
            s.x += q[u].x;
            s.y += q[u].y;
            s.z += q[u].z;
            s.w += q[u].w;
          }
        }
      }
      if (col < a.n) rank_emit(a, mt, mt * 128 + r, col, s);
    }
  }

  // peers may still read this CTA's partial tile until here
  tc_fence_before();
  if (ks > 1) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Both rank products of one output gradient in one pass over it:
//   dxa = dy Bt^T   [m, r]   (dy K-major, Bt [r, n])
//   G   = dy^T Xt^T [n, r]   (dy MN-major, Xt = xa^T [r, m])
// A CTA owns rt x ct tiles of 128 x 128 of dy (rows x columns). Each
// tile is loaded once (two TMA boxes of 128 rows x 64 columns, 128-byte
// swizzle) and feeds two MMAs: as the K-major A of its row tile's dxa
// accumulator (K = its 128 columns) and, the same bytes read as an MN-major
// operand, as the A of its column tile's G accumulator (M = its 128 columns,
// K = its 128 rows). The rt + ct accumulators (NP fp32 columns each) share
// the 512 TMEM columns; the launcher picks rt and ct for the shape. The CTA leaves its fp32 partials in a workspace,
// dxa per column block and G per row block, and dual_reduce_kernel sums them
// in block order (bitwise reproducible).
template <int NP>
struct DualSmem {
  static constexpr int kMaxAcc = 512 / NP;          // rt + ct accumulators fit in TMEM
  static constexpr int kDyBytes = 128 * 128 * 2;    // one 128 x 128 tile of dy
  static constexpr int kFacBytes = NP * 64 * 2;     // one box of a factor: NP rows x 64
  static constexpr int kStage = kDyBytes + 4 * kFacBytes;  // dy, Bt (2 boxes), Xt (2 boxes)
  static constexpr int kStages = 4 * kStage + 2048 <= 232448 ? 4 : 3;
  static constexpr int kBar = kStages * kStage;
  static constexpr int kNumBars = 2 * kStages + 1;  // full[S], empty[S], acc_full
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  static constexpr int kBytes = kUsed + 1024;  // + alignment slack
};

struct DualArgs {
  int m, n;           // dy [m, n]
  int mt, nt;         // 128-row and 128-column tiles of dy
  int rt, ct;         // row and column tiles per CTA (rt + ct <= 512 / NP)
  int rb, cb;         // CTA blocks along rows and columns (grid = rb * cb)
  uint64_t wait_ns;
  float* ws_dxa;      // [cb][m][NP]: dxa partial of each column block
  float* ws_g;        // [rb][n][NP]: G partial of each row block
};

template <int NP>
__global__ void __launch_bounds__(kRankThreads, 1)
    dual_rank_kernel(const __grid_constant__ CUtensorMap tma_d, const __grid_constant__ CUtensorMap tma_bt,
                     const __grid_constant__ CUtensorMap tma_xt, const DualArgs a, int* err) {
  using L = DualSmem<NP>;
  const int RT = a.rt, CT = a.ct;
  constexpr int S = L::kStages;
  constexpr uint32_t kIdescK = idesc_bf16(NP, false, false, 128);
  constexpr uint32_t kIdescMN = idesc_bf16(NP, true, false, 128);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if ((uint32_t)(smem - smem_raw) + L::kUsed > rank_dynamic_smem()) {  // grid-uniform
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrRankSmem);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t acc_bar = bar0 + 8u * (2 * S);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bi = blockIdx.x / a.cb, bj = blockIdx.x - (blockIdx.x / a.cb) * a.cb;
  const int i_n = min(RT, a.mt - bi * RT), j_n = min(CT, a.nt - bj * CT);  // tiles inside dy
  const uint64_t wait_ns = a.wait_ns ? a.wait_ns : kWaitNs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) mbar_init(bar0 + 8u * i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tma_d);
    tma_prefetch_desc(&tma_bt);
    tma_prefetch_desc(&tma_xt);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      int it = 0;
      bool ok = true;
      for (int j = 0; j < j_n && ok; ++j) {
        for (int i = 0; i < i_n; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!bounded_wait(empty_bar(s), ph ^ 1u, abort_flag, err, kErrRankProducer, wait_ns)) {
            ok = false;
            break;
          }
          const uint32_t d_dst = sbase + s * L::kStage;
          const uint32_t bt_dst = d_dst + L::kDyBytes;
          const uint32_t xt_dst = bt_dst + 2 * L::kFacBytes;
          const int r0 = (bi * RT + i) * 128, c0 = (bj * CT + j) * 128;
          mbar_arrive_expect_tx(full_bar(s), L::kStage);
          tma_load_2d(d_dst, &tma_d, full_bar(s), c0, r0);
          tma_load_2d(d_dst + 16384, &tma_d, full_bar(s), c0 + 64, r0);
          tma_load_2d(bt_dst, &tma_bt, full_bar(s), c0, 0);
          tma_load_2d(bt_dst + L::kFacBytes, &tma_bt, full_bar(s), c0 + 64, 0);
          tma_load_2d(xt_dst, &tma_xt, full_bar(s), r0, 0);
          tma_load_2d(xt_dst + L::kFacBytes, &tma_xt, full_bar(s), r0 + 64, 0);
        }
      }
      // let the copies still in flight land before the CTA may leave (bounded)
      const int n_wait = it < S ? it : S;
      for (int q = 1; q <= n_wait; ++q) {
        const int jj = it - q;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(full_bar(jj % S), (jj / S) & 1u) && globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------- MMA issuer ----
      int it = 0;
      bool ok = true, issued = false;
      for (int j = 0; j < j_n && ok; ++j) {
        for (int i = 0; i < i_n; ++i, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!bounded_wait(full_bar(s), ph, abort_flag, err, kErrRankMma, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_addr = sbase + s * L::kStage;
          const uint32_t bt_addr = d_addr + L::kDyBytes;
          const uint32_t xt_addr = bt_addr + 2 * L::kFacBytes;
          // dxa(row tile i) += dy tile . Bt^T over the tile's 128 columns
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc_sw128(d_addr + h * 16384 + kk * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(bt_addr + h * L::kFacBytes + kk * 32, 16, 1024);
              tc_mma_bf16(tmem + i * NP, ad, bd, kIdescK, (j > 0 || h > 0 || kk > 0) ? 1u : 0u);
            }
          }
          // G(column tile j) += dy tile^T . Xt^T over the tile's 128 rows: the
          // same bytes as an MN-major operand (64-column boxes 16 KB apart)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = smem_desc_sw128(d_addr + kk * 2048, 16384, 1024);
            const uint64_t bd = smem_desc_sw128(xt_addr + (kk >> 2) * L::kFacBytes + (kk & 3) * 32, 16, 1024);
            tc_mma_bf16(tmem + (RT + j) * NP, ad, bd, kIdescMN, (i > 0 || kk > 0) ? 1u : 0u);
          }
          issued = true;
          tc_commit(empty_bar(s));
        }
      }
      if (issued) {
        tc_commit(acc_bar);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(acc_bar, 0) && globaltimer() - t0 < wait_ns) {
        }
      } else {
        mbar_arrive(acc_bar);
      }
    }
  } else {
    // ------------------------------------------------------ epilogue ----
    const int quarter = warp & 3;
    bool ok = true;
    if (lane == 0) ok = bounded_wait(acc_bar, 0, abort_flag, err, kErrRankEpilogue, wait_ns);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    tc_fence_after();
    if (ok && !*abort_flag) {
      const uint32_t tl = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
      for (int t = 0; t < i_n + j_n; ++t) {
        const bool is_dxa = t < i_n;
        const int tile = is_dxa ? t : t - i_n;
        float v[NP];
        __syncwarp();
#pragma unroll
        for (int c = 0; c < NP; c += 16)
          tmem_ld16_nowait(tl + (is_dxa ? tile : RT + tile) * NP + c, v + c);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int row = ((is_dxa ? bi * RT : bj * CT) + tile) * 128 + quarter * 32 + lane;
        if (row >= (is_dxa ? a.m : a.n)) continue;
        float* dst = is_dxa ? a.ws_dxa + ((int64_t)bj * a.m + row) * NP
                            : a.ws_g + ((int64_t)bi * a.n + row) * NP;
#pragma unroll
        for (int c = 0; c < NP; c += 4)
          *reinterpret_cast<float4*>(dst + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// dxa[m, :r] (bf16) = sum over the column blocks of ws_dxa; G[n, :r] (fp32) =
// sum over the row blocks of ws_g; block order, four columns per thread.
__global__ void __launch_bounds__(256) dual_reduce_kernel(const float* __restrict__ ws_dxa,
                                                          const float* __restrict__ ws_g, int m, int n, int r,
                                                          int np, int rb, int cb, bf16* __restrict__ dxa,
                                                          int64_t lddxa, float* __restrict__ g, int64_t ldg) {
  pdl_wait();
  const int q = np / 4;
  const int64_t n1 = (int64_t)m * q, total = n1 + (int64_t)n * q;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const bool is_dxa = idx < n1;
    const int64_t e = is_dxa ? idx : idx - n1;
    const int64_t row = e / q;
    const int col = static_cast<int>(e - row * q) * 4;
    if (col >= r) continue;
    const int blocks = is_dxa ? cb : rb;
    const int rows = is_dxa ? m : n;
    const float* src = (is_dxa ? ws_dxa : ws_g) + row * np + col;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b < blocks; ++b) {
      const float4 p = *reinterpret_cast<const float4*>(src + (int64_t)b * rows * np);
      s.x += p.x;
      s.y += p.y;
      s.z += p.z;
      s.w += p.w;
    }
    const float v[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (col + c >= r) break;
      if (is_dxa) dxa[row * lddxa + col + c] = __float2bfloat16_rn(v[c]);
      else g[row * ldg + col + c] = v[c];
    }
  }
  pdl_trigger();
}

}  // namespace
}  // namespace soup

// ------------------------------------------------------------------- host --
namespace soup {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 rank_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lock(cache_mutex());
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// bf16 matrix [outer, inner] with row stride ld (elements): box {64, box_outer},
// 128-byte swizzle, zero fill out of bounds.
int rank_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
             uint32_t box_outer) {
  auto fn = rank_encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return SOUP_ERR_CUDA;
  }
  if (int rc = bind_context()) return rc;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed for a rank-product operand");
    return SOUP_ERR_UNSUPPORTED;
  }
  return SOUP_OK;
}

bool rank_tma_ok(const void* p, int64_t ld) { return aligned16(p) && ld > 0 && (ld * 2) % 16 == 0; }

// ks = CTAs per cluster (1..16): as many as one wave of resident CTAs allows
// (2-3 per SM, by the kernel's shared memory), at least four k-blocks per CTA,
// and a cluster size the device can hold with this kernel's shared memory.
template <bool A_MN, int NP>
int rank_launch(const CUtensorMap& ma, const CUtensorMap& mb, RankArgs args, int m_tiles, cudaStream_t stream) {
  using L = RankSmem<NP>;
  static_assert(L::kBytes <= 232448, "rank product shared memory exceeds 227 KB");
  auto kern = rank_gemm_kernel<A_MN, NP>;
  static bool attr_done[64] = {false};
  static int per_sm[64] = {0};           // resident CTAs per SM
  static int max_clusters[64][17] = {};  // by cluster size; -1: none fits
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cuda_status(cudaErrorInvalidDevice);
  int* err = device_err_ptr();
  if (!err) {
    set_last_error("device error word unavailable");
    return SOUP_ERR_CUDA;
  }
  const int sms = num_sms();

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kRankThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  {
    std::lock_guard<std::mutex> lock(cache_mutex());
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
      if (e != cudaSuccess) return cuda_status(e);
      // clusters of up to 16 CTAs (the occupancy query below says which fit)
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        cudaGetLastError();
      // by shared memory (228 KB per SM, 1 KB of it reserved per CTA), at most 3
      int smem_sm = 0;
      if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess) {
        cudaGetLastError();
        smem_sm = L::kBytes;
      }
      const int n = smem_sm / (L::kBytes + 1024);
      per_sm[dev] = n < 1 ? 1 : n > 3 ? 3 : n;
      attr_done[dev] = true;
    }
  }
  // one wave of resident CTAs (2-3 per SM, by this kernel's shared memory), at
  // least four k-blocks per CTA, clusters of up to 16 where the device can hold
  // one of that size with this kernel
  int ks = per_sm[dev] * sms / (m_tiles > 0 ? m_tiles : 1);
  if (ks > 16) ks = 16;
  if (ks > args.kb_total / 4) ks = args.kb_total / 4;
  if (ks < 1) ks = 1;
  for (; ks > 1; --ks) {
    std::lock_guard<std::mutex> lock(cache_mutex());
    if (max_clusters[dev][ks] == 0) {
      int n = 0;
      attr[0].val.clusterDim.x = ks;
      cfg.gridDim = dim3(ks * (sms / ks));
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      max_clusters[dev][ks] = n > 0 ? n : -1;
    }
    if (max_clusters[dev][ks] > 0) break;
  }
  args.ks = ks;
  attr[0].val.clusterDim.x = ks;
  cfg.gridDim = dim3(m_tiles * ks);
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ma, mb, args, err));
}

template <bool A_MN>
int rank_dispatch(const CUtensorMap& ma, const CUtensorMap& mb, const RankArgs& args, int m_tiles,
                  cudaStream_t stream) {
  if (args.n <= 16) return rank_launch<A_MN, 16>(ma, mb, args, m_tiles, stream);
  if (args.n <= 32) return rank_launch<A_MN, 32>(ma, mb, args, m_tiles, stream);
  if (args.n <= 48) return rank_launch<A_MN, 48>(ma, mb, args, m_tiles, stream);
  return rank_launch<A_MN, 64>(ma, mb, args, m_tiles, stream);
}

int np_of(int64_t n) { return n <= 16 ? 16 : n <= 32 ? 32 : n <= 48 ? 48 : 64; }

// Shared checks and set-up of both entry points; fills maps and the size fields.
int rank_prepare(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int64_t m, int64_t n,
                 int64_t k, CUtensorMap* ma, CUtensorMap* mb, RankArgs* args, const char* name) {
  char msg[160];
  if (!a || !b || m <= 0 || k <= 0 || n <= 0 || n > kRankMaxN || m > (1 << 30) || k > (1 << 30)) {
    snprintf(msg, sizeof(msg), "%s: bad arguments (n must be 1..%d)", name, kRankMaxN);
    set_last_error(msg);
    return SOUP_ERR_INVALID;
  }
  if ((a_mn_major ? lda < m : lda < k) || ldb < k) {
    snprintf(msg, sizeof(msg), "%s: leading dimension too small", name);
    set_last_error(msg);
    return SOUP_ERR_INVALID;
  }
  if (!rank_tma_ok(a, lda) || !rank_tma_ok(b, ldb)) {
    snprintf(msg, sizeof(msg), "%s: operands need 16-byte aligned rows", name);
    set_last_error(msg);
    return SOUP_ERR_UNSUPPORTED;
  }
  int rc;
  if (a_mn_major) rc = rank_map(ma, a, (uint64_t)m, (uint64_t)k, (uint64_t)lda, 64);
  else rc = rank_map(ma, a, (uint64_t)k, (uint64_t)m, (uint64_t)lda, 128);
  if (rc) return rc;
  if ((rc = rank_map(mb, b, (uint64_t)k, (uint64_t)n, (uint64_t)ldb, (uint32_t)np_of(n)))) return rc;
  *args = RankArgs{};
  args->m = (int)m;
  args->n = (int)n;
  args->k = (int)k;
  args->kb_total = (int)((k + 63) / 64);
  args->ks = 1;
  args->wait_ns = wait_limit_ns();
  return SOUP_OK;
}

template <int NP>
int dual_launch(const CUtensorMap& md, const CUtensorMap& mbt, const CUtensorMap& mxt, DualArgs args, int r,
                bf16* dxa, int64_t lddxa, float* g, int64_t ldg, cudaStream_t stream) {
  using L = DualSmem<NP>;
  static_assert(L::kBytes <= 232448, "dual rank product shared memory exceeds 227 KB");
  auto kern = dual_rank_kernel<NP>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cuda_status(cudaErrorInvalidDevice);
  int* err = device_err_ptr();
  if (!err) {
    set_last_error("device error word unavailable");
    return SOUP_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> lock(cache_mutex());
    if (!attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
      if (e != cudaSuccess) return cuda_status(e);
      attr_done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(kRankThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(args.rb * args.cb);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, md, mbt, mxt, args, err);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t items = ((int64_t)args.m + args.n) * (NP / 4);
  int64_t blocks = (items + 255) / 256;
  const int64_t cap = 4ll * num_sms();
  if (blocks > cap) blocks = cap;
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, dual_reduce_kernel, static_cast<const float*>(args.ws_dxa),
                                        static_cast<const float*>(args.ws_g), args.m, args.n, r, NP, args.rb,
                                        args.cb, dxa, lddxa, g, ldg));
}

// accumulator width of the dual kernel: 16, 32 or 64 columns (TMEM offsets
// i * NP stay multiples of NP)
int dual_np(int64_t r) { return r <= 16 ? 16 : r <= 32 ? 32 : 64; }

// Row and column tiles per CTA (rt + ct <= 512 / np accumulators): the
// estimate is the slowest SM's share of dy (whole waves of CTAs, each
// streaming rt x ct tiles at ~40 GB/s) plus the partials' HBM round trip.
void dual_blocking(int64_t m, int64_t n, int np, int sms, int* rt, int* ct) {
  const int64_t mt = (m + 127) / 128, nt = (n + 127) / 128;
  double best = 1e30;
  *rt = *ct = 1;
  for (int a = 1; a < 512 / np; ++a) {
    for (int b = 1; a + b <= 512 / np; ++b) {
      if (a > mt || b > nt) continue;
      const int64_t rb = (mt + a - 1) / a, cb = (nt + b - 1) / b;
      const int64_t waves = (rb * cb + sms - 1) / sms;
      const double t = waves * (double)a * b * 32768.0 / 40e9 + (double)(cb * m + rb * n) * np * 8.0 / 6e12;
      if (t < best) {
        best = t;
        *rt = a;
        *ct = b;
      }
    }
  }
}

}  // namespace
}  // namespace soup

extern "C" {

size_t soup_lora_rank_dual_workspace_bytes(int64_t m, int64_t n, int64_t r) {
  using namespace soup;
  if (m <= 0 || n <= 0 || r <= 0 || r > kRankMaxN || m > (1 << 30) || n > (1 << 30)) return 0;
  int rt, ct;
  dual_blocking(m, n, dual_np(r), num_sms(), &rt, &ct);
  const int64_t rb = ((m + 127) / 128 + rt - 1) / rt, cb = ((n + 127) / 128 + ct - 1) / ct;
  return (size_t)((cb * m + rb * n) * dual_np(r) * 4);
}

int soup_lora_rank_dual(const void* dy, int64_t lddy, const void* bt, int64_t ldbt, const void* xt,
                        int64_t ldxt, int64_t m, int64_t n, int64_t r, void* dxa, int64_t lddxa, float* g,
                        int64_t ldg, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace soup;
  if (!dy || !bt || !xt || !dxa || !g || m <= 0 || n <= 0 || r <= 0 || r > kRankMaxN || m > (1 << 30) ||
      n > (1 << 30)) {
    set_last_error("soup_lora_rank_dual: bad arguments (r must be 1..64)");
    return SOUP_ERR_INVALID;
  }
  if (lddy < n || ldbt < n || ldxt < m || lddxa < r || ldg < r) {
    set_last_error("soup_lora_rank_dual: leading dimension too small");
    return SOUP_ERR_INVALID;
  }
  if (!rank_tma_ok(dy, lddy) || !rank_tma_ok(bt, ldbt) || !rank_tma_ok(xt, ldxt)) {
    set_last_error("soup_lora_rank_dual: operands need 16-byte aligned rows");
    return SOUP_ERR_UNSUPPORTED;
  }
  const size_t need = soup_lora_rank_dual_workspace_bytes(m, n, r);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_last_error("soup_lora_rank_dual: workspace missing, unaligned or smaller than "
                   "soup_lora_rank_dual_workspace_bytes()");
    return SOUP_ERR_WORKSPACE;
  }
  const int np = dual_np(r);
  CUtensorMap md, mbt, mxt;
  int rc;
  if ((rc = rank_map(&md, dy, (uint64_t)n, (uint64_t)m, (uint64_t)lddy, 128))) return rc;
  if ((rc = rank_map(&mbt, bt, (uint64_t)n, (uint64_t)r, (uint64_t)ldbt, (uint32_t)np))) return rc;
  if ((rc = rank_map(&mxt, xt, (uint64_t)m, (uint64_t)r, (uint64_t)ldxt, (uint32_t)np))) return rc;
  DualArgs args{};
  dual_blocking(m, n, np, num_sms(), &args.rt, &args.ct);
  args.m = (int)m;
  args.n = (int)n;
  args.mt = (int)((m + 127) / 128);
  args.nt = (int)((n + 127) / 128);
  args.rb = (args.mt + args.rt - 1) / args.rt;
  args.cb = (args.nt + args.ct - 1) / args.ct;
  args.wait_ns = wait_limit_ns();
  args.ws_dxa = static_cast<float*>(workspace);
  args.ws_g = args.ws_dxa + (int64_t)args.cb * m * np;
  bf16* d = static_cast<bf16*>(dxa);
  cudaStream_t st = as_stream(stream);
  switch (np) {
    case 16: return dual_launch<16>(md, mbt, mxt, args, (int)r, d, lddxa, g, ldg, st);
    case 32: return dual_launch<32>(md, mbt, mxt, args, (int)r, d, lddxa, g, ldg, st);
    default: return dual_launch<64>(md, mbt, mxt, args, (int)r, d, lddxa, g, ldg, st);
  }
}


int soup_lora_rank_gemm(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int64_t m,
                        int64_t n, int64_t k, void* c, int64_t ldc, void* ct, int64_t ldct, float* g,
                        int64_t ldg, int g_transposed, float alpha, void* stream) {
  using namespace soup;
  if (!c && !ct && !g) {
    set_last_error("soup_lora_rank_gemm: no output");
    return SOUP_ERR_INVALID;
  }
  if ((c && ldc < n) || (ct && ldct < m) || (g && ldg < (g_transposed ? m : n))) {
    set_last_error("soup_lora_rank_gemm: output leading dimension too small");
    return SOUP_ERR_INVALID;
  }
  CUtensorMap ma, mb;
  RankArgs args;
  if (int rc = rank_prepare(a, lda, a_mn_major, b, ldb, m, n, k, &ma, &mb, &args, "soup_lora_rank_gemm"))
    return rc;
  args.alpha = alpha;
  args.c = static_cast<bf16*>(c);
  args.ldc = ldc;
  args.ct = static_cast<bf16*>(ct);
  args.ldct = ldct;
  args.g = g;
  args.ldg = ldg;
  args.g_trans = g_transposed ? 1 : 0;
  const int m_tiles = (int)((m + 127) / 128);
  if (a_mn_major) return rank_dispatch<true>(ma, mb, args, m_tiles, as_stream(stream));
  return rank_dispatch<false>(ma, mb, args, m_tiles, as_stream(stream));
}

int soup_lora_rank_grad_group(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                              int64_t k, int nmem, int interleaved, const int64_t* row_off,
                              const int64_t* col_off, float* const* g, const int64_t* ldg, float alpha,
                              void* stream) {
  using namespace soup;
  if (nmem < 1 || nmem > kRankMaxMembers || !row_off || !col_off || !g || !ldg) {
    set_last_error("soup_lora_rank_grad_group: bad member table");
    return SOUP_ERR_INVALID;
  }
  if (row_off[0] != 0 || row_off[nmem] != m || col_off[0] < 0 || col_off[nmem] > n) {
    set_last_error("soup_lora_rank_grad_group: member offsets must cover [0, m) and lie within [0, n]");
    return SOUP_ERR_INVALID;
  }
  for (int j = 0; j < nmem; ++j) {
    const int64_t rows = row_off[j + 1] - row_off[j], cols = col_off[j + 1] - col_off[j];
    if (rows <= 0 || cols <= 0 || !g[j] || ldg[j] < cols) {
      set_last_error("soup_lora_rank_grad_group: empty member or bad gradient buffer");
      return SOUP_ERR_INVALID;
    }
    if (interleaved && (rows != m / nmem || rows % 128)) {
      set_last_error("soup_lora_rank_grad_group: interleaved members need equal row counts, multiples of 128");
      return SOUP_ERR_INVALID;
    }
  }
  CUtensorMap ma, mb;
  RankArgs args;
  if (int rc = rank_prepare(a, lda, 1, b, ldb, m, n, k, &ma, &mb, &args, "soup_lora_rank_grad_group"))
    return rc;
  args.alpha = alpha;
  args.nmem = nmem;
  args.interleaved = interleaved ? 1 : 0;
  for (int j = 0; j <= nmem; ++j) {
    args.row_off[j] = (int)row_off[j];
    args.col_off[j] = (int)col_off[j];
  }
  for (int j = 0; j < nmem; ++j) {
    args.gm[j] = g[j];
    args.ldgm[j] = ldg[j];
  }
  const int m_tiles = (int)((m + 127) / 128);
  return rank_dispatch<true>(ma, mb, args, m_tiles, as_stream(stream));
}

}  // extern "C"
