// Causal grouped-query flash attention for sm_100a on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA), head dim 128,
// bf16 in / fp32 accumulate. Replaces the SDPA call of transformers' Qwen2
// attention (modeling_qwen2.py: Qwen2Attention.forward -> sdpa_attention_forward)
// in the QLoRA step; the reference runs it through torch SDPA.
//
// Forward (one CTA per (batch, query head, 128-query tile); heavy tiles first):
//   warp 0      TMA producer: the Q tile once, then K / V tiles of 128 keys into
//               a 2-stage ring (4-D tensor maps over [B, H, S, D] with any
//               b / h / s strides, so HF's transposed [B, S, H, D] views are read
//               in place)
//   warp 1      TMEM allocator + MMA issuer (lane 0): S = Q K^T into one of two
//               TMEM buffers (the next tile's S overlaps this tile's softmax),
//               then O += P V with P from shared memory
//   warps 2..5  softmax: one query row per thread (TMEM lane quarter = warp % 4),
//               online softmax in base 2 with a lazily updated row maximum (O and
//               the row sum are rescaled only when the maximum grows by more than
//               2^8, so most tiles skip the TMEM read-modify-write of O), P written
//               as bf16 into the MMA's 128-byte-swizzled K-major layout; at the end
//               O / l in bf16 to [B, S, H, D] and the row log-sum-exp (natural
//               units) for the backward.
// Backward: dK / dV per (batch, KV head, 128-key tile) looping over the query
// heads of its group and the causal query tiles (S^T, dP^T, dV += P^T dO, dK +=
// dS^T Q; all four accumulators in TMEM), and dQ per (batch, query head, query
// tile) looping over key tiles (S, dP, dQ += dS K). Both recompute P from the
// saved log-sum-exp; no atomics, results are bitwise reproducible.
//
// Every mbarrier wait is bounded as in the GEMM kernels (tc_gemm.cuh): on expiry
// the role records a code in the device error word, raises the CTA's abort
// flag, the producer waits (bounded) for its copies, the MMA warp drains its
// MMAs, and the CTA frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "soup_common.cuh"
#include "tc_gemm.cuh"

namespace soup {
namespace attn {

using bf16 = __nv_bfloat16;
using tc::bounded_wait;
using tc::mbar_arrive;
using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_try_wait;
using tc::smem_desc_sw128;
using tc::smem_u32;
using tc::tc_commit;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tc_mma_bf16;
using tc::tmem_ld32;

constexpr int kHeadDim = 128;
constexpr int kTile = 128;             // query rows per CTA and keys per tile
constexpr int kBox = kTile * 128;      // one [128 rows x 64 cols] bf16 box: 16 KB
constexpr int kTileBytes = 2 * kBox;   // a 128 x 128 bf16 tile (two 64-column boxes)
constexpr int kStages = 2;             // K / V ring depth

constexpr int kErrAttnProducer = 0x111;
constexpr int kErrAttnMma = 0x112;
constexpr int kErrAttnSoftmax = 0x113;
constexpr int kErrAttnSmem = 0x114;  // dynamic shared memory too small after 1 KB alignment

// 4-D TMA tile load (coordinates innermost first) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 32 lanes x 32 consecutive fp32 columns from registers into TMEM (the
// inverse of tmem_ld32); the caller waits with tmem_st_wait.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 fp32 columns from TMEM without waiting: several loads are
// issued back to back and completed by one tmem_ld_wait (the registers may
// not be read before it).
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// K-major operand tile of 128 rows x 128 bf16 columns in shared memory: two
// 16 KB boxes (columns 0-63, 64-127), rows of 128 B, 128-byte swizzle. The
// descriptor of k-step kk (16 columns) for tcgen05.mma.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int kk) {
  return smem_desc_sw128(base + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024);
}
// The same bytes read as an MN-major operand whose MN dimension is the tile's
// 128 columns and whose K dimension is its 128 rows: k-step kk covers rows
// [16 kk, 16 kk + 16); the two 64-column boxes are the MN atoms (LBO 16 KB).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int kk) {
  return smem_desc_sw128(base + kk * 2048, kBox, 1024);
}

// Byte offset of the 16-byte chunk c (columns 8c..8c+7 of a 64-column box) of
// row r in a 128-byte-swizzled box: the layout TMA writes and the descriptors read.
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// Instruction descriptors (fp32 accumulate, bf16 operands, M = N = 128).
constexpr uint32_t kIdescKK = tc::idesc_bf16(128, false, false, 128);  // A, B K-major
constexpr uint32_t kIdescKM = tc::idesc_bf16(128, false, true, 128);   // B MN-major

struct AttnArgs {
  int B, H, Hk, S;       // batch, query heads, KV heads, sequence length
  float scale_log2;      // softmax scale * log2(e)
  int causal;
  bf16* out;             // [B, S, H, D] contiguous (row of one token: H * D)
  float* lse;            // [B, H, S_pad] natural-log log-sum-exp of scale * q.k, rows
                         // padded to S_pad = S rounded up to 128 (padding not written)
  uint64_t wait_ns;
};

// ------------------------------------------------------------- forward ----
// Shared memory: Q (32 KB), K ring (2 x 32 KB), V ring (2 x 32 KB), P (32 KB),
// barriers. TMEM: S buffers at columns 0 and 128, O at 256 (512 allocated).
struct FwdSmem {
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTileBytes;
  static constexpr int kV = kK + kStages * kTileBytes;
  static constexpr int kP = kV + kStages * kTileBytes;
  static constexpr int kBar = kP + kTileBytes;
  // q_full, k_full[2], v_full[2], kv_empty[2], s_full[2], s_empty[2], p_full, pv_done, drain
  static constexpr int kNumBars = 1 + 2 * kStages + kStages + 2 + 2 + 3;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16 + 1024;
};
static_assert(FwdSmem::kBytes <= 232448, "attention forward shared memory exceeds 227 KB");

constexpr int kSoftmaxWarps = 4;
constexpr int kFwdThreads = 64 + 32 * kSoftmaxWarps;

// Q, K, V maps: 4-D {D, S, heads, B} with box {64, 128, 1, 1}; coordinates
// (d0, s0, head, b).
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                    const __grid_constant__ CUtensorMap tma_v, AttnArgs a, int* err) {
  using L = FwdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + kStages + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + 2 * kStages + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (1 + 3 * kStages + b); };
  auto s_empty = [&](int b) { return bar0 + 8u * (3 + 3 * kStages + b); };
  const uint32_t p_full = bar0 + 8u * (5 + 3 * kStages);
  const uint32_t pv_done = bar0 + 8u * (6 + 3 * kStages);
  const uint32_t drain_bar = bar0 + 8u * (7 + 3 * kStages);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (a.S + kTile - 1) / kTile;
  const int bh = blockIdx.x % (a.B * a.H);
  const int qt = nq - 1 - blockIdx.x / (a.B * a.H);  // heavy (late) query tiles first
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  const int q0 = qt * kTile;
  const int nkv = a.causal ? qt + 1 : nq;
  const uint64_t wait_ns = a.wait_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      // the softmax warps arrive once each on s_empty and p_full
      const bool per_warp = bar == s_empty(0) || bar == s_empty(1) || bar == p_full;
      mbar_init(bar, per_warp ? kSoftmaxWarps : 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::tma_prefetch_desc(&tma_q);
    tc::tma_prefetch_desc(&tma_k);
    tc::tma_prefetch_desc(&tma_v);
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

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sbase + L::kQ, &tma_q, q_full, 0, q0, h, b);
      tma_load_4d(sbase + L::kQ + kBox, &tma_q, q_full, 64, q0, h, b);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kStages;
        if (!bounded_wait(kv_empty(st), ((j / kStages) & 1) ^ 1, abort_flag, err, kErrAttnProducer,
                          wait_ns))
          break;
        const uint32_t kd = sbase + L::kK + st * kTileBytes;
        const uint32_t vd = sbase + L::kV + st * kTileBytes;
        mbar_arrive_expect_tx(k_full(st), kTileBytes);
        tma_load_4d(kd, &tma_k, k_full(st), 0, j * kTile, hk, b);
        tma_load_4d(kd + kBox, &tma_k, k_full(st), 64, j * kTile, hk, b);
        mbar_arrive_expect_tx(v_full(st), kTileBytes);
        tma_load_4d(vd, &tma_v, v_full(st), 0, j * kTile, hk, b);
        tma_load_4d(vd + kBox, &tma_v, v_full(st), 64, j * kTile, hk, b);
        ++issued;
      }
      // let every issued copy land before the CTA may leave (bounded)
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(q_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        t0 = tc::globaltimer();
        while (!mbar_try_wait(k_full(st), ph) && tc::globaltimer() - t0 < wait_ns) {
        }
        t0 = tc::globaltimer();
        while (!mbar_try_wait(v_full(st), ph) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(q_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      auto issue_s = [&](int j) -> bool {
        const int st = j % kStages, sb = j & 1;
        if (!bounded_wait(k_full(st), (j / kStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (!bounded_wait(s_empty(sb), ((j >> 1) & 1) ^ 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        tc_fence_after();
        const uint32_t qa = sbase + L::kQ, kb = sbase + L::kK + st * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)
          tc_mma_bf16(tmem + sb * 128, desc_kmajor(qa, kk), desc_kmajor(kb, kk), kIdescKK,
                      kk > 0 ? 1u : 0u);
        tc_commit(s_full(sb));
        issued = true;
        return true;
      };
      if (ok && nkv > 0) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !(ok = issue_s(j + 1))) break;
        const int st = j % kStages;
        if (!(ok = bounded_wait(v_full(st), (j / kStages) & 1, abort_flag, err, kErrAttnMma,
                                wait_ns)))
          break;
        if (!(ok = bounded_wait(p_full, j & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
        const uint32_t pa = sbase + L::kP, vb = sbase + L::kV + st * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          tc_mma_bf16(tmem + 256, desc_kmajor(pa, kk), desc_mnmajor(vb, kk), kIdescKM,
                      (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(kv_empty(st));
        tc_commit(pv_done);
      }
      if (!ok && issued) {
        tc_commit(drain_bar);
        uint64_t t0 = tc::globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else {
    // ------------------------------------------------------- softmax ----
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;   // query row of this thread within the tile
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* pbuf = smem + L::kP;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1;
      bool w = true;
      if (lane == 0) w = bounded_wait(s_full(sb), (j >> 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                      wait_ns);
      ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      float s[kTile];
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c)
        tmem_ld32_async(tmem + sb * 128 + c * 32 + lane_off,
                        *reinterpret_cast<float(*)[32]>(s + c * 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty(sb));
      // masks: keys beyond the sequence, and (causal) keys after the query
      const int k0 = j * kTile;
      const bool edge = (k0 + kTile > a.S) || (a.causal && j == qt);
      if (edge) {
#pragma unroll
        for (int i = 0; i < kTile; ++i) {
          const int key = k0 + i;
          if (key >= a.S || (a.causal && key > q)) s[i] = -INFINITY;
        }
      }
      // row maximum of the raw logits (the scale is positive), eight chains
      float mx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx[u] = s[u];
#pragma unroll
      for (int i = 8; i < kTile; i += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = fmaxf(mx[u], s[i + u]);
      }
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * a.scale_log2;
      bool rescale = false;
      float alpha = 1.f;
      if (mt > m_used + 8.f) {  // also when m_used is still -inf
        alpha = fast_exp2(m_used - mt);
        m_used = mt;
        rescale = true;
      }
      float sm[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < kTile; i += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          s[i + u] = fast_exp2(fmaf(s[i + u], a.scale_log2, -m_used));
          sm[u] += s[i + u];
        }
      }
      const float sum = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      l = rescale ? l * alpha + sum : l + sum;
      // P V of the previous tile must be done: the P buffer and O are reused
      if (j > 0) {
        if (lane == 0) w = bounded_wait(pv_done, (j - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
        if (!ok) break;
        tc_fence_after();
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
        // rescales when any of its rows needs it (alpha = 1 for the others)
        if (__any_sync(0xffffffffu, rescale)) {
          float o[kHeadDim];
#pragma unroll
          for (int c = 0; c < kHeadDim / 32; ++c)
            tmem_ld32_async(tmem + 256 + c * 32 + lane_off,
                            *reinterpret_cast<float(*)[32]>(o + c * 32));
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < kHeadDim; ++i) o[i] *= alpha;
#pragma unroll
          for (int c = 0; c < kHeadDim / 32; ++c)
            tmem_st32(tmem + 256 + c * 32 + lane_off, *reinterpret_cast<float(*)[32]>(o + c * 32));
          tmem_st_wait();
        }
      }
      // P (bf16) into the K-major swizzled layout: keys 0-63 in box 0, 64-127 in box 1
#pragma unroll
      for (int c = 0; c < kTile / 8; ++c) {
        const uint4 u = make_uint4(pack_bf16(s[8 * c], s[8 * c + 1]), pack_bf16(s[8 * c + 2], s[8 * c + 3]),
                                   pack_bf16(s[8 * c + 4], s[8 * c + 5]),
                                   pack_bf16(s[8 * c + 6], s[8 * c + 7]));
        *reinterpret_cast<uint4*>(pbuf + (c >> 3) * kBox + swz_off(r, c & 7)) = u;
      }
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && nkv > 0) {
      bool w = true;
      if (lane == 0) w = bounded_wait(pv_done, (nkv - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                      wait_ns);
      ok = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
    }
    if (ok && nkv > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = a.out + ((int64_t)b * a.S + q) * (int64_t)(a.H * kHeadDim) + h * kHeadDim;
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + 256 + c * 32 + lane_off, o);
        if (q < a.S) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint4 u = make_uint4(pack_bf16(o[8 * g] * inv, o[8 * g + 1] * inv),
                                       pack_bf16(o[8 * g + 2] * inv, o[8 * g + 3] * inv),
                                       pack_bf16(o[8 * g + 4] * inv, o[8 * g + 5] * inv),
                                       pack_bf16(o[8 * g + 6] * inv, o[8 * g + 7] * inv));
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * g) = u;
          }
        }
      }
      if (q < a.S)
        a.lse[((int64_t)b * a.H + h) * ((int64_t)nq * kTile) + q] = (m_used + __log2f(l)) * kLn2;
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

// ------------------------------------------------------------ backward ----
// D[b, h, q] = sum_d dO[b, q, h, d] * O[b, q, h, d] (fp32), one warp per row;
// D rows padded like lse ([B, H, S_pad]). dO and O are [B, S, H, D] contiguous.
__global__ void __launch_bounds__(256) attn_bwd_dot_kernel(const bf16* __restrict__ dO,
                                                           const bf16* __restrict__ O, int B, int H,
                                                           int S, float* __restrict__ Dv) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);  // (b, q, h) row-major
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * S * H) return;
  const uint2 a = *reinterpret_cast<const uint2*>(dO + row * kHeadDim + lane * 4);
  const uint2 c = *reinterpret_cast<const uint2*>(O + row * kHeadDim + lane * 4);
  const __nv_bfloat162* ap = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* cp = reinterpret_cast<const __nv_bfloat162*>(&c);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 x = __bfloat1622float2(ap[i]), y = __bfloat1622float2(cp[i]);
    acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int h = (int)(row % H);
    const int64_t bq = row / H;
    const int q = (int)(bq % S), b = (int)(bq / S);
    const int64_t s_pad = (int64_t)(S + kTile - 1) / kTile * kTile;
    Dv[((int64_t)b * H + h) * s_pad + q] = acc;
  }
}

struct BwdArgs {
  int B, H, Hk, S;
  float scale;        // softmax scale (applied to dK, dQ in fp32)
  float scale_log2;   // scale * log2(e)
  int causal;
  const float* lse;   // [B, H, S_pad] from the forward (S_pad = S rounded up to 128)
  const float* Dv;    // [B, H, S_pad] from attn_bwd_dot_kernel
  float* dk_part;     // dK/dV kernel: fp32 [B, H, S, D] per query head
  float* dv_part;
  bf16* dq;           // dQ kernel: [B, S, H, D]
  uint64_t wait_ns;
};

// dK / dV partials of one query head for one 128-key tile: TMEM columns S^T 0,
// dP^T 128, dV 256, dK 384. Shared memory: K, V (32 KB each, loaded once), two
// stages of (Q, dO) (64 KB each), one P / dS buffer (32 KB).
struct DkvSmem {
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTileBytes;
  static constexpr int kQD = kV + kTileBytes;          // stage s: Q at +0, dO at +kTileBytes
  static constexpr int kPS = kQD + 2 * 2 * kTileBytes;  // P^T, then dS^T
  static constexpr int kVec = kPS + kTileBytes;         // stage s: lse, D of its query tile (2 x 512 B)
  static constexpr int kBar = kVec + 2 * 2 * kTile * 4;
  // kv_full, qdo_full[2], qdo_empty[2], st_full, st_empty, p_full, pv_done, ds_full,
  // buf_free, acc_done, drain
  static constexpr int kNumBars = 13;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  // alignment slack up to the 227 KB limit: the kernel checks at entry that the
  // padding to the 1024-byte boundary of its dynamic shared memory fits
  static constexpr int kBytes = kUsed + 1024 <= 232448 ? kUsed + 1024 : 232448;
};
static_assert(DkvSmem::kUsed + 128 <= 232448, "attention dK/dV shared memory exceeds 227 KB");

constexpr int kBwdThreads = 64 + 32 * kSoftmaxWarps;

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing on an mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint32_t dynamic_smem_bytes() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}

// One bool from lane 0 to the warp.
__device__ __forceinline__ bool warp_ok(bool v) { return __shfl_sync(0xffffffffu, v ? 1 : 0, 0) != 0; }

// Rows of a packed bf16 tile (64 words = 128 values of this thread's row) into
// the K-major swizzled layout of a 128 x 128 operand tile.
__device__ __forceinline__ void store_row_tile(uint8_t* tile, int r, const uint32_t (&w)[64]) {
#pragma unroll
  for (int c = 0; c < 16; ++c)
    *reinterpret_cast<uint4*>(tile + (c >> 3) * kBox + swz_off(r, c & 7)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Maps: Q over [B, H, S, D], K / V over [B, Hk, S, D], dO over [B, S, H, D]
// viewed as [B, H, S, D] (strides S*H*D, D, H*D).
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tma_q,
                         const __grid_constant__ CUtensorMap tma_k,
                         const __grid_constant__ CUtensorMap tma_v,
                         const __grid_constant__ CUtensorMap tma_do, BwdArgs a, int* err) {
  using L = DkvSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if ((uint32_t)(smem - smem_raw) + L::kUsed > dynamic_smem_bytes()) {  // grid-uniform
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrAttnSmem);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  const uint32_t kv_full = bar0;
  auto qdo_full = [&](int st) { return bar0 + 8u * (1 + st); };
  auto qdo_empty = [&](int st) { return bar0 + 8u * (3 + st); };
  const uint32_t st_full = bar0 + 8u * 5, st_empty = bar0 + 8u * 6, p_full = bar0 + 8u * 7;
  const uint32_t pv_done = bar0 + 8u * 8, ds_full = bar0 + 8u * 9, buf_free = bar0 + 8u * 10;
  const uint32_t acc_done = bar0 + 8u * 11, drain_bar = bar0 + 8u * 12;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (a.S + kTile - 1) / kTile;
  const int bh = blockIdx.x % (a.B * a.H);
  const int kt = blockIdx.x / (a.B * a.H);  // causal: early key tiles have the most queries
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  const int k0 = kt * kTile;
  const int qt_first = a.causal ? kt : 0;
  const int n = nq - qt_first;
  const int64_t s_pad = (int64_t)nq * kTile;
  const uint64_t wait_ns = a.wait_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      const bool per_warp = bar == st_empty || bar == p_full || bar == ds_full;
      mbar_init(bar, per_warp ? kSoftmaxWarps : 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::tma_prefetch_desc(&tma_q);
    tc::tma_prefetch_desc(&tma_k);
    tc::tma_prefetch_desc(&tma_v);
    tc::tma_prefetch_desc(&tma_do);
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

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
      tma_load_4d(sbase + L::kK, &tma_k, kv_full, 0, k0, hk, b);
      tma_load_4d(sbase + L::kK + kBox, &tma_k, kv_full, 64, k0, hk, b);
      tma_load_4d(sbase + L::kV, &tma_v, kv_full, 0, k0, hk, b);
      tma_load_4d(sbase + L::kV + kBox, &tma_v, kv_full, 64, k0, hk, b);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int st = i & 1;
        if (!bounded_wait(qdo_empty(st), ((i >> 1) & 1) ^ 1, abort_flag, err, kErrAttnProducer,
                          wait_ns))
          break;
        const int q0 = (qt_first + i) * kTile;
        const uint32_t qd = sbase + L::kQD + st * 2 * kTileBytes;
        const int64_t vrow = ((int64_t)b * a.H + h) * s_pad + q0;
        const uint32_t vd = sbase + L::kVec + st * 2 * kTile * 4;
        mbar_arrive_expect_tx(qdo_full(st), 2 * kTileBytes + 2 * kTile * 4);
        tma_load_4d(qd, &tma_q, qdo_full(st), 0, q0, h, b);
        tma_load_4d(qd + kBox, &tma_q, qdo_full(st), 64, q0, h, b);
        tma_load_4d(qd + kTileBytes, &tma_do, qdo_full(st), 0, q0, h, b);
        tma_load_4d(qd + kTileBytes + kBox, &tma_do, qdo_full(st), 64, q0, h, b);
        bulk_load(vd, a.lse + vrow, kTile * 4, qdo_full(st));
        bulk_load(vd + kTile * 4, a.Dv + vrow, kTile * 4, qdo_full(st));
        ++issued;
      }
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(kv_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int i = issued > 2 ? issued - 2 : 0; i < issued; ++i) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(qdo_full(i & 1), (i >> 1) & 1) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(kv_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      const uint32_t ka = sbase + L::kK, va = sbase + L::kV, ps = sbase + L::kPS;
      auto issue_sd = [&](int i) -> bool {
        const int st = i & 1;
        if (!bounded_wait(qdo_full(st), (i >> 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (i > 0 &&
            !bounded_wait(st_empty, (i - 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        tc_fence_after();
        const uint32_t qd = sbase + L::kQD + st * 2 * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // S^T = K Q^T
          tc_mma_bf16(tmem, desc_kmajor(ka, kk), desc_kmajor(qd, kk), kIdescKK, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // dP^T = V dO^T
          tc_mma_bf16(tmem + 128, desc_kmajor(va, kk), desc_kmajor(qd + kTileBytes, kk), kIdescKK,
                      kk > 0 ? 1u : 0u);
        tc_commit(st_full);
        issued = true;
        return true;
      };
      if (ok && n > 0) ok = issue_sd(0);
      for (int i = 0; i < n && ok; ++i) {
        const int st = i & 1;
        const uint32_t qd = sbase + L::kQD + st * 2 * kTileBytes;
        if (i + 1 < n && !(ok = issue_sd(i + 1))) break;
        if (!(ok = bounded_wait(p_full, i & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dV += P^T dO
          tc_mma_bf16(tmem + 256, desc_kmajor(ps, kk), desc_mnmajor(qd + kTileBytes, kk), kIdescKM,
                      (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pv_done);
        if (!(ok = bounded_wait(ds_full, i & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dK += dS^T Q
          tc_mma_bf16(tmem + 384, desc_kmajor(ps, kk), desc_mnmajor(qd, kk), kIdescKM,
                      (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(buf_free);
        tc_commit(qdo_empty(st));
      }
      if (ok && n > 0) tc_commit(acc_done);
      if (!ok && issued) {
        tc_commit(drain_bar);
        uint64_t t0 = tc::globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else {
    // ------------------------------------------------------- compute ----
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row of this thread
    const int key = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* ps = smem + L::kPS;
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int qt = qt_first + i;
      const int q0 = qt * kTile;
      bool w = true;
      // S^T / dP^T of this tile are issued after its Q / dO / lse / D landed
      if (lane == 0) w = bounded_wait(st_full, i & 1, abort_flag, err, kErrAttnSoftmax, wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      const float* vlse = reinterpret_cast<const float*>(smem + L::kVec + (i & 1) * 2 * kTile * 4);
      const float* vD = vlse + kTile;
      const bool edge = (q0 + kTile > a.S) || (a.causal && qt == kt);
      uint32_t pw[64], dw[64];
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld32_async(tmem + c * 32 + lane_off, sv);
        tmem_ld32_async(tmem + 128 + c * 32 + lane_off, dp);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p2[2], d2[2];
          const float2 l2 = *reinterpret_cast<const float2*>(vlse + c * 32 + e);
          const float2 dd = *reinterpret_cast<const float2*>(vD + c * 32 + e);
          const float lv[2] = {l2.x, l2.y}, dvv[2] = {dd.x, dd.y};
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int qi = c * 32 + e + u;
            float pv = fast_exp2(fmaf(sv[e + u], a.scale_log2, -lv[u] * 1.4426950408889634f));
            float dv = pv * (dp[e + u] - dvv[u]);
            if (edge) {  // padding rows of lse / D may hold anything: select, do not scale
              const int q = q0 + qi;
              if (q >= a.S || (a.causal && q < key)) pv = dv = 0.f;
            }
            p2[u] = pv;
            d2[u] = dv;
          }
          pw[(c * 32 + e) >> 1] = pack_bf16(p2[0], p2[1]);
          dw[(c * 32 + e) >> 1] = pack_bf16(d2[0], d2[1]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(st_empty);
      if (i > 0) {  // the previous tile's dK product has read the P / dS buffer
        if (lane == 0) w = bounded_wait(buf_free, (i - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
      }
      store_row_tile(ps, r, pw);
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (lane == 0) w = bounded_wait(pv_done, i & 1, abort_flag, err, kErrAttnSoftmax, wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      store_row_tile(ps, r, dw);
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && n > 0) {
      bool w = true;
      if (lane == 0) w = bounded_wait(acc_done, 0, abort_flag, err, kErrAttnSoftmax, wait_ns);
      ok = warp_ok(w);
    }
    if (ok && n > 0) {
      tc_fence_after();
      const int64_t row = (((int64_t)b * a.H + h) * a.S + key) * kHeadDim;
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        float v[32], g[32];
        tmem_ld32(tmem + 256 + c * 32 + lane_off, v);
        tmem_ld32(tmem + 384 + c * 32 + lane_off, g);
        if (key < a.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            *reinterpret_cast<float4*>(a.dv_part + row + c * 32 + e) =
                make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            *reinterpret_cast<float4*>(a.dk_part + row + c * 32 + e) =
                make_float4(g[e] * a.scale, g[e + 1] * a.scale, g[e + 2] * a.scale,
                            g[e + 3] * a.scale);
          }
        }
      }
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

// dQ of one query tile: TMEM columns S 0, dP 128, dQ 256. Shared memory: Q and
// dO (32 KB each, loaded once), two stages of (K, V) (64 KB each), dS (32 KB).
struct DqSmem {
  static constexpr int kQ = 0;
  static constexpr int kDO = kQ + kTileBytes;
  static constexpr int kKV = kDO + kTileBytes;          // stage s: K at +0, V at +kTileBytes
  static constexpr int kDS = kKV + 2 * 2 * kTileBytes;
  static constexpr int kBar = kDS + kTileBytes;
  // qdo_full, kv_full[2], kv_empty[2], st_full, st_empty, ds_full, buf_free, acc_done, drain
  static constexpr int kNumBars = 11;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  static constexpr int kBytes = kUsed + 1024 <= 232448 ? kUsed + 1024 : 232448;
};
static_assert(DqSmem::kUsed + 128 <= 232448, "attention dQ shared memory exceeds 227 KB");

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tma_q,
                       const __grid_constant__ CUtensorMap tma_k,
                       const __grid_constant__ CUtensorMap tma_v,
                       const __grid_constant__ CUtensorMap tma_do, BwdArgs a, int* err) {
  using L = DqSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if ((uint32_t)(smem - smem_raw) + L::kUsed > dynamic_smem_bytes()) {  // grid-uniform
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrAttnSmem);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  const uint32_t qdo_full = bar0;
  auto kv_full = [&](int st) { return bar0 + 8u * (1 + st); };
  auto kv_empty = [&](int st) { return bar0 + 8u * (3 + st); };
  const uint32_t st_full = bar0 + 8u * 5, st_empty = bar0 + 8u * 6, ds_full = bar0 + 8u * 7;
  const uint32_t buf_free = bar0 + 8u * 8, acc_done = bar0 + 8u * 9, drain_bar = bar0 + 8u * 10;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (a.S + kTile - 1) / kTile;
  const int bh = blockIdx.x % (a.B * a.H);
  const int qt = nq - 1 - blockIdx.x / (a.B * a.H);  // heavy (late) query tiles first
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  const int q0 = qt * kTile;
  const int n = a.causal ? qt + 1 : nq;
  const uint64_t wait_ns = a.wait_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      const bool per_warp = bar == st_empty || bar == ds_full;
      mbar_init(bar, per_warp ? kSoftmaxWarps : 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::tma_prefetch_desc(&tma_q);
    tc::tma_prefetch_desc(&tma_k);
    tc::tma_prefetch_desc(&tma_v);
    tc::tma_prefetch_desc(&tma_do);
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

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      mbar_arrive_expect_tx(qdo_full, 2 * kTileBytes);
      tma_load_4d(sbase + L::kQ, &tma_q, qdo_full, 0, q0, h, b);
      tma_load_4d(sbase + L::kQ + kBox, &tma_q, qdo_full, 64, q0, h, b);
      tma_load_4d(sbase + L::kDO, &tma_do, qdo_full, 0, q0, h, b);
      tma_load_4d(sbase + L::kDO + kBox, &tma_do, qdo_full, 64, q0, h, b);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j & 1;
        if (!bounded_wait(kv_empty(st), ((j >> 1) & 1) ^ 1, abort_flag, err, kErrAttnProducer,
                          wait_ns))
          break;
        const uint32_t kv = sbase + L::kKV + st * 2 * kTileBytes;
        mbar_arrive_expect_tx(kv_full(st), 2 * kTileBytes);
        tma_load_4d(kv, &tma_k, kv_full(st), 0, j * kTile, hk, b);
        tma_load_4d(kv + kBox, &tma_k, kv_full(st), 64, j * kTile, hk, b);
        tma_load_4d(kv + kTileBytes, &tma_v, kv_full(st), 0, j * kTile, hk, b);
        tma_load_4d(kv + kTileBytes + kBox, &tma_v, kv_full(st), 64, j * kTile, hk, b);
        ++issued;
      }
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(qdo_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(kv_full(j & 1), (j >> 1) & 1) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(qdo_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      const uint32_t qa = sbase + L::kQ, da = sbase + L::kDO, ds = sbase + L::kDS;
      auto issue_sd = [&](int j) -> bool {
        const int st = j & 1;
        if (!bounded_wait(kv_full(st), (j >> 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (j > 0 && !bounded_wait(st_empty, (j - 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        tc_fence_after();
        const uint32_t kv = sbase + L::kKV + st * 2 * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // S = Q K^T
          tc_mma_bf16(tmem, desc_kmajor(qa, kk), desc_kmajor(kv, kk), kIdescKK, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // dP = dO V^T
          tc_mma_bf16(tmem + 128, desc_kmajor(da, kk), desc_kmajor(kv + kTileBytes, kk), kIdescKK,
                      kk > 0 ? 1u : 0u);
        tc_commit(st_full);
        issued = true;
        return true;
      };
      if (ok && n > 0) ok = issue_sd(0);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j & 1;
        const uint32_t kv = sbase + L::kKV + st * 2 * kTileBytes;
        if (j + 1 < n && !(ok = issue_sd(j + 1))) break;
        if (!(ok = bounded_wait(ds_full, j & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dQ += dS K
          tc_mma_bf16(tmem + 256, desc_kmajor(ds, kk), desc_mnmajor(kv, kk), kIdescKM,
                      (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(buf_free);
        tc_commit(kv_empty(st));
      }
      if (ok && n > 0) tc_commit(acc_done);
      if (!ok && issued) {
        tc_commit(drain_bar);
        uint64_t t0 = tc::globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else {
    // ------------------------------------------------------- compute ----
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of this thread
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t vidx = ((int64_t)b * a.H + h) * ((int64_t)nq * kTile) + q;
    const float lse2 = q < a.S ? a.lse[vidx] * 1.4426950408889634f : 0.f;
    const float dq_d = q < a.S ? a.Dv[vidx] : 0.f;
    uint8_t* dsb = smem + L::kDS;
    bool ok = true;
    for (int j = 0; j < n && ok; ++j) {
      bool w = true;
      if (lane == 0) w = bounded_wait(st_full, j & 1, abort_flag, err, kErrAttnSoftmax, wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      const int k0 = j * kTile;
      const bool edge = (k0 + kTile > a.S) || (a.causal && j == qt);
      uint32_t dw[64];
#pragma unroll
      for (int c = 0; c < kTile / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld32_async(tmem + c * 32 + lane_off, sv);
        tmem_ld32_async(tmem + 128 + c * 32 + lane_off, dp);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float d2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float pv = fast_exp2(sv[e + u] * a.scale_log2 - lse2);
            float dv = pv * (dp[e + u] - dq_d);
            if (edge) {
              const int key = k0 + c * 32 + e + u;
              if (key >= a.S || (a.causal && key > q)) dv = 0.f;
            }
            d2[u] = dv;
          }
          dw[(c * 32 + e) >> 1] = pack_bf16(d2[0], d2[1]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(st_empty);
      if (j > 0) {  // the previous tile's dQ product has read the dS buffer
        if (lane == 0) w = bounded_wait(buf_free, (j - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
      }
      store_row_tile(dsb, r, dw);
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && n > 0) {
      bool w = true;
      if (lane == 0) w = bounded_wait(acc_done, 0, abort_flag, err, kErrAttnSoftmax, wait_ns);
      ok = warp_ok(w);
    }
    if (ok && n > 0) {
      tc_fence_after();
      bf16* orow = a.dq + ((int64_t)b * a.S + q) * (int64_t)(a.H * kHeadDim) + h * kHeadDim;
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + 256 + c * 32 + lane_off, o);
        if (q < a.S) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const float sc = a.scale;
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * g) =
                make_uint4(pack_bf16(o[8 * g] * sc, o[8 * g + 1] * sc),
                           pack_bf16(o[8 * g + 2] * sc, o[8 * g + 3] * sc),
                           pack_bf16(o[8 * g + 4] * sc, o[8 * g + 5] * sc),
                           pack_bf16(o[8 * g + 6] * sc, o[8 * g + 7] * sc));
          }
        }
      }
    }
  }

  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

// dK, dV [B, S, Hk, D] bf16 = sums of the fp32 per-query-head partials
// [B, H, S, D] over each KV head's group (fixed head order), 4 elements per thread.
__global__ void __launch_bounds__(256) attn_bwd_group_sum_kernel(const float* __restrict__ dk_part,
                                                                 const float* __restrict__ dv_part,
                                                                 int B, int H, int Hk, int S,
                                                                 bf16* __restrict__ dk,
                                                                 bf16* __restrict__ dv) {
  pdl_wait();
  pdl_trigger();
  const int rep = H / Hk;
  const int64_t n4 = (int64_t)B * S * Hk * (kHeadDim / 4);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d4 = (int)(i % (kHeadDim / 4));
    int64_t t = i / (kHeadDim / 4);
    const int hk = (int)(t % Hk);
    t /= Hk;
    const int s = (int)(t % S);
    const int b = (int)(t / S);
    float4 ak = make_float4(0.f, 0.f, 0.f, 0.f), av = ak;
    for (int g = 0; g < rep; ++g) {
      const int64_t src = (((int64_t)b * H + hk * rep + g) * S + s) * kHeadDim + d4 * 4;
      const float4 x = *reinterpret_cast<const float4*>(dk_part + src);
      const float4 y = *reinterpret_cast<const float4*>(dv_part + src);
      ak.x += x.x; ak.y += x.y; ak.z += x.z; ak.w += x.w;
      av.x += y.x; av.y += y.y; av.z += y.z; av.w += y.w;
    }
    const int64_t dst = (((int64_t)b * S + s) * Hk + hk) * kHeadDim + d4 * 4;
    *reinterpret_cast<uint2*>(dk + dst) = make_uint2(pack_bf16(ak.x, ak.y), pack_bf16(ak.z, ak.w));
    *reinterpret_cast<uint2*>(dv + dst) = make_uint2(pack_bf16(av.x, av.y), pack_bf16(av.z, av.w));
  }
}

// ----------------------------------------------------------------- host ----
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::lock_guard<std::mutex> lock(cache_mutex());
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

// 4-D map over a bf16 [B, heads, S, D] tensor with element strides (b, h, s)
// and a contiguous last dimension: dims {D, S, heads, B}, box {64, 128, 1, 1},
// 128-byte swizzle, zero fill outside.
static int make_bhsd_map(CUtensorMap* map, const void* ptr, const int64_t* strides, int64_t B,
                         int64_t heads, int64_t S, const char* what) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return SOUP_ERR_CUDA;
  }
  if (int rc = bind_context()) return rc;
  cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)S, (cuuint64_t)heads, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2,
                        (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)kTile, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, gstr, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[200];
    snprintf(msg, sizeof(msg), "attention: cuTensorMapEncodeTiled failed (%d) for %s", (int)r, what);
    set_last_error(msg);
    return SOUP_ERR_UNSUPPORTED;
  }
  return SOUP_OK;
}

// Strides of a [B, heads, S, 128] bf16 operand usable by TMA: 16-byte aligned
// base, every stride a multiple of 8 elements.
static bool bhsd_ok(const void* p, const int64_t* st) {
  return p && aligned16(p) && st && st[0] > 0 && st[1] > 0 && st[2] > 0 && st[0] % 8 == 0 &&
         st[1] % 8 == 0 && st[2] % 8 == 0;
}

template <typename K>
static int set_smem(K kern, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cuda_status(cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lock(cache_mutex());
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return cuda_status(e);
    done[dev] = true;
  }
  return SOUP_OK;
}

}  // namespace attn
}  // namespace soup

using namespace soup;
using namespace soup::attn;

extern "C" {

int soup_attention_fwd(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq,
                       int64_t head_dim, float scale, int causal, void* out, float* lse,
                       void* stream) {
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || seq <= 0 || heads % kv_heads != 0 ||
      batch * heads > (1 << 20) || seq > (1 << 24) || !out || !lse || !(scale > 0.f)) {
    set_last_error("soup_attention_fwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (head_dim != kHeadDim) {
    set_last_error("soup_attention_fwd: head_dim must be 128");
    return SOUP_ERR_UNSUPPORTED;
  }
  if (!bhsd_ok(q, q_strides) || !bhsd_ok(k, k_strides) || !bhsd_ok(v, v_strides) ||
      !aligned16(out)) {
    set_last_error("soup_attention_fwd: q/k/v need 16-byte aligned bases and strides that are "
                   "multiples of 8 elements (last dimension contiguous)");
    return SOUP_ERR_UNSUPPORTED;
  }
  int* err = device_err_ptr();
  if (!err) {
    set_last_error("device error word unavailable");
    return SOUP_ERR_CUDA;
  }
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_bhsd_map(&mq, q, q_strides, batch, heads, seq, "q"))) return rc;
  if ((rc = make_bhsd_map(&mk, k, k_strides, batch, kv_heads, seq, "k"))) return rc;
  if ((rc = make_bhsd_map(&mv, v, v_strides, batch, kv_heads, seq, "v"))) return rc;
  static bool smem_set[64] = {false};
  if ((rc = set_smem(attn_fwd_kernel, FwdSmem::kBytes, smem_set))) return rc;
  AttnArgs a{(int)batch, (int)heads, (int)kv_heads, (int)seq, scale * 1.4426950408889634f,
             causal ? 1 : 0, static_cast<bf16*>(out), lse, 0};
  a.wait_ns = wait_limit_ns() ? wait_limit_ns() : tc::kWaitNs;
  const int nq = (int)((seq + kTile - 1) / kTile);
  return cuda_status(launch_pdl(attn_fwd_kernel, dim3((unsigned)(batch * heads * nq)),
                                dim3(kFwdThreads), FwdSmem::kBytes, as_stream(stream), mq, mk, mv,
                                a, err));
}

size_t soup_attention_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const size_t s_pad = (size_t)((seq + kTile - 1) / kTile * kTile);
  const size_t dvec = (size_t)batch * heads * s_pad * 4;
  const size_t part = (size_t)batch * heads * seq * kHeadDim * 4;
  return (dvec + 255) / 256 * 256 + 2 * ((part + 255) / 256 * 256);
}

int soup_attention_bwd(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       const void* out, const void* dout, const float* lse, int64_t batch,
                       int64_t heads, int64_t kv_heads, int64_t seq, int64_t head_dim, float scale,
                       int causal, void* dq, void* dk, void* dv, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || seq <= 0 || heads % kv_heads != 0 ||
      batch * heads > (1 << 20) || seq > (1 << 24) || !out || !dout || !lse || !dq || !dk || !dv ||
      !workspace || !(scale > 0.f)) {
    set_last_error("soup_attention_bwd: bad arguments");
    return SOUP_ERR_INVALID;
  }
  if (head_dim != kHeadDim) {
    set_last_error("soup_attention_bwd: head_dim must be 128");
    return SOUP_ERR_UNSUPPORTED;
  }
  if (!bhsd_ok(q, q_strides) || !bhsd_ok(k, k_strides) || !bhsd_ok(v, v_strides) ||
      !aligned16(out) || !aligned16(dout) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv) ||
      !aligned16(lse)) {
    set_last_error("soup_attention_bwd: operands need 16-byte aligned bases and strides that are "
                   "multiples of 8 elements");
    return SOUP_ERR_UNSUPPORTED;
  }
  const size_t need = soup_attention_bwd_workspace_bytes(batch, heads, seq);
  if (workspace_bytes < need || !aligned16(workspace)) {
    set_last_error("soup_attention_bwd: workspace too small or misaligned");
    return SOUP_ERR_WORKSPACE;
  }
  int* err = device_err_ptr();
  if (!err) {
    set_last_error("device error word unavailable");
    return SOUP_ERR_CUDA;
  }
  const int64_t s_pad = (seq + kTile - 1) / kTile * kTile;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* dvec = reinterpret_cast<float*>(ws);
  const size_t part = (size_t)batch * heads * seq * kHeadDim * 4;
  const size_t off1 = ((size_t)batch * heads * s_pad * 4 + 255) / 256 * 256;
  float* dk_part = reinterpret_cast<float*>(ws + off1);
  float* dv_part = reinterpret_cast<float*>(ws + off1 + (part + 255) / 256 * 256);
  CUtensorMap mq, mk, mv, mdo;
  int rc;
  const int64_t do_strides[3] = {seq * heads * kHeadDim, kHeadDim, heads * kHeadDim};
  if ((rc = make_bhsd_map(&mq, q, q_strides, batch, heads, seq, "q"))) return rc;
  if ((rc = make_bhsd_map(&mk, k, k_strides, batch, kv_heads, seq, "k"))) return rc;
  if ((rc = make_bhsd_map(&mv, v, v_strides, batch, kv_heads, seq, "v"))) return rc;
  if ((rc = make_bhsd_map(&mdo, dout, do_strides, batch, heads, seq, "dout"))) return rc;
  static bool dkdv_set[64] = {false}, dq_set[64] = {false};
  if ((rc = set_smem(attn_bwd_dkdv_kernel, DkvSmem::kBytes, dkdv_set))) return rc;
  if ((rc = set_smem(attn_bwd_dq_kernel, DqSmem::kBytes, dq_set))) return rc;
  cudaStream_t st = as_stream(stream);
  const int B = (int)batch, H = (int)heads, Hk = (int)kv_heads, S = (int)seq;
  const int64_t rows = (int64_t)B * S * H;
  if ((rc = cuda_status(launch_pdl(attn_bwd_dot_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256),
                                   0, st, static_cast<const bf16*>(dout),
                                   static_cast<const bf16*>(out), B, H, S, dvec))))
    return rc;
  BwdArgs a{B, H, Hk, S, scale, scale * 1.4426950408889634f, causal ? 1 : 0, lse, dvec, dk_part,
            dv_part, static_cast<bf16*>(dq), 0};
  a.wait_ns = wait_limit_ns() ? wait_limit_ns() : tc::kWaitNs;
  const int nt = (S + kTile - 1) / kTile;
  if ((rc = cuda_status(launch_pdl(attn_bwd_dkdv_kernel, dim3((unsigned)(B * H * nt)),
                                   dim3(kBwdThreads), DkvSmem::kBytes, st, mq, mk, mv, mdo, a, err))))
    return rc;
  if ((rc = cuda_status(launch_pdl(attn_bwd_dq_kernel, dim3((unsigned)(B * H * nt)),
                                   dim3(kBwdThreads), DqSmem::kBytes, st, mq, mk, mv, mdo, a, err))))
    return rc;
  const int64_t n4 = (int64_t)B * S * Hk * (kHeadDim / 4);
  int blocks = (int)((n4 + 255) / 256);
  if (blocks > 8 * num_sms()) blocks = 8 * num_sms();
  return cuda_status(launch_pdl(attn_bwd_group_sum_kernel, dim3(blocks), dim3(256), 0, st,
                                (const float*)dk_part, (const float*)dv_part, B, H, Hk, S,
                                static_cast<bf16*>(dk), static_cast<bf16*>(dv)));
}

}  // extern "C"
