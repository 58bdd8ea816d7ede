// Causal grouped-query flash attention for sm_100a on the 5th-generation tensor
// cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA), head dim 128,
// bf16 in / fp32 accumulate. Replaces the SDPA call of transformers' Qwen2
// attention (modeling_qwen2.py: Qwen2Attention.forward -> sdpa_attention_forward)
// in the QLoRA step; the reference runs it through torch SDPA.
//
// Forward (one CTA per (batch, query head, pair of 128-query tiles); heavy pairs
// first):
//   warp 0      TMA producer: both Q tiles once, then K / V tiles of 128 keys
//               into 2-stage rings (4-D tensor maps over [B, H, S, D] with any
//               b / h / s strides, so HF's transposed [B, S, H, D] views are read
//               in place)
//   warp 1      TMEM allocator + MMA issuer (lane 0): S_X = Q_X K^T per query
//               tile X, then O_X += P_X V with P_X read from TMEM, interleaved so
//               that one tile's products run during the other tile's softmax
//   warps 2..9  softmax, four warps per query tile (warps 2-5 tile A, 6-9 tile
//               B; lane quarter warp % 4): one query row per thread, its 128 key
//               columns in two passes (row maximum, then exponentials; keys
//               64-127 stay in registers, so three TMEM round trips per tile).
//               Online softmax in base 2 with a lazily updated row maximum (O and
//               the row sum are rescaled only when the maximum grows by more than
//               2^8, so most tiles skip the TMEM read-modify-write of O), P
//               written as bf16 pairs over S's last 64 columns; at the end O / l
//               in bf16 to [B, S, H, D] and the row log-sum-exp (natural units).
// Backward: dK / dV per (batch, query head, 128-key tile) over its causal
// queries in 64-query steps (S^T, dP^T double buffered in TMEM, dV += P^T dO,
// dK += dS^T Q), fp32 partials per query head summed over each KV head's group
// by a fixed-order kernel; dQ per (batch, query head, query tile) over its key
// tiles (S, dP, dQ += dS K with dS read from TMEM). Both recompute P from the
// saved log-sum-exp; no atomics, results are bitwise reproducible. Their eight
// compute warps are two per TMEM lane quarter, each owning half of a row's
// columns, and release S / dP as soon as they have read them, so the next
// tile's products run while this tile's P and dS are computed.
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
constexpr int kKStages = 2;            // forward K ring depth (a stage frees after S = Q K^T)
constexpr int kVStages = 1;            // forward V stages (one frees after both tiles' P V)

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

__device__ __forceinline__ uint32_t dynamic_smem_bytes() {
  uint32_t v;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
  return v;
}
// One bool from lane 0 to the warp.
__device__ __forceinline__ bool warp_ok(bool v) { return __shfl_sync(0xffffffffu, v ? 1 : 0, 0) != 0; }

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

// D (TMEM) [+]= A (TMEM, M rows in lanes, two bf16 of K per 32-bit column) x B (smem descriptor).
__device__ __forceinline__ void tc_mma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                                   uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers into TMEM.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// ------------------------------------------------------------- forward ----
// One CTA per (batch, query head, pair of 128-query tiles A = 2p, B = 2p + 1);
// heavy (late) pairs first. The two tiles share every K / V tile. TMEM: S_A at
// column 0, S_B at 128, O_A at 256, O_B at 384 (512 allocated); P_X (bf16, two
// keys per 32-bit column) overwrites the last 64 columns of S_X and is the A
// operand of O_X += P_X V read from TMEM. The MMA warp issues, per key tile j,
// P V of tile A, then S_A(j + 1), then P V of tile B, then S_B(j + 1): while the
// tensor core runs one tile's products the other tile's softmax runs, and each
// S_X(j + 1) follows (in issue order) the product that read P_X(j) from the same
// columns. Shared memory: Q_A, Q_B (32 KB each), K ring (2 x 32 KB), V ring
// (2 x 32 KB), barriers.
struct FwdSmem {
  static constexpr int kQ = 0;  // tile X at + X * kTileBytes
  static constexpr int kK = kQ + 2 * kTileBytes;
  static constexpr int kV = kK + kKStages * kTileBytes;
  static constexpr int kP = kV + kVStages * kTileBytes;  // tile X at + X * kTileBytes
  static constexpr int kBar = kP + 2 * kTileBytes;
  // q_full, k_full[2], k_empty[2], v_full, v_empty, s_full[2], s_free[2], p_full[2],
  // pv_done[2] (the last four per query tile), drain
  static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 2 + 2 + 2 + 2 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  static constexpr int kBytes = kUsed + 1024 <= 232448 ? kUsed + 1024 : 232448;
};
static_assert(FwdSmem::kUsed + 128 <= 232448, "attention forward shared memory exceeds 227 KB");

// Compute warps: four per query tile (warps 2-5 tile A, 6-9 tile B in the
// forward), warp w reading TMEM lane quarter w % 4. The backward kernels use the
// same eight warps as two per lane quarter, each owning half of a row's columns
// (column half (w - 2) / 4).
constexpr int kSoftmaxWarps = 8;
constexpr int kHalf = kTile / 2;
constexpr int kFwdThreads = 64 + 32 * kSoftmaxWarps;

// Q, K, V maps: 4-D {D, S, heads, B} with box {64, 128, 1, 1}; coordinates
// (d0, s0, head, b).
// 32 lanes x 16 consecutive 32-bit columns from TMEM (waits for the load).
__device__ __forceinline__ void tmem_ld16u(uint32_t taddr, uint32_t (&v)[16]) {
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers into TMEM.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}

// O row of this thread (128 fp32 TMEM columns) times alpha. A separate,
// non-inlined function: the rescale is rare, and keeping its registers out of
// the softmax loop avoids spills there. Warp-collective.
__device__ __noinline__ void rescale_o_row(uint32_t o_t, float alpha) {
  const uint64_t al2 = f2_pack(alpha, alpha);
#pragma unroll 1
  for (int c = 0; c < kHeadDim / 16; ++c) {
    uint32_t o[16];
    tmem_ld16u(o_t + c * 16, o);
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float o0, o1;
      f2_unpack(f2_mul(f2_pack(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), al2), o0, o1);
      o[i] = __float_as_uint(o0);
      o[i + 1] = __float_as_uint(o1);
    }
    tmem_st16u(o_t + c * 16, o);
    tmem_st_wait();
  }
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                    const __grid_constant__ CUtensorMap tma_v, AttnArgs a, int* err) {
  using L = FwdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if ((uint32_t)(smem - smem_raw) + L::kUsed > dynamic_smem_bytes()) {  // grid-uniform
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrAttnSmem);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBar;
  const uint32_t q_full = bar0;
  constexpr int kB = 1 + 2 * kKStages + 2 * kVStages;  // first barrier after the rings
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + kKStages + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * kKStages + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * kKStages + kVStages + s); };
  auto s_full = [&](int x) { return bar0 + 8u * (kB + x); };
  auto s_free = [&](int x) { return bar0 + 8u * (kB + 2 + x); };
  auto p_full = [&](int x) { return bar0 + 8u * (kB + 4 + x); };
  auto pv_done = [&](int x) { return bar0 + 8u * (kB + 6 + x); };
  const uint32_t drain_bar = bar0 + 8u * (kB + 8);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (a.S + kTile - 1) / kTile;
  const int npair = (nq + 1) / 2;
  const int bh = blockIdx.x % (a.B * a.H);
  const int pr = npair - 1 - blockIdx.x / (a.B * a.H);  // heavy (late) pairs first
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  // key tiles each query tile attends to (B's are a superset of A's)
  const int nkv_a = a.causal ? 2 * pr + 1 : nq;
  const int nkv_b = a.causal ? (2 * pr + 2 < nq ? 2 * pr + 2 : nq) : nq;
  const uint64_t wait_ns = a.wait_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      // the four softmax warps of a query tile arrive once each on its s_free, p_full
      const bool per_warp = bar == s_free(0) || bar == s_free(1) || bar == p_full(0) ||
                            bar == p_full(1);
      mbar_init(bar, per_warp ? 4 : 1);
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
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const uint32_t qd = sbase + L::kQ + x * kTileBytes;
        tma_load_4d(qd, &tma_q, q_full, 0, (2 * pr + x) * kTile, h, b);
        tma_load_4d(qd + kBox, &tma_q, q_full, 64, (2 * pr + x) * kTile, h, b);
      }
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < nkv_b; ++j) {
        const int sk = j % kKStages, sv = j % kVStages;
        if (!bounded_wait(k_empty(sk), ((j / kKStages) & 1) ^ 1, abort_flag, err,
                          kErrAttnProducer, wait_ns))
          break;
        const uint32_t kd = sbase + L::kK + sk * kTileBytes;
        mbar_arrive_expect_tx(k_full(sk), kTileBytes);
        tma_load_4d(kd, &tma_k, k_full(sk), 0, j * kTile, hk, b);
        tma_load_4d(kd + kBox, &tma_k, k_full(sk), 64, j * kTile, hk, b);
        ++issued_k;
        if (!bounded_wait(v_empty(sv), ((j / kVStages) & 1) ^ 1, abort_flag, err,
                          kErrAttnProducer, wait_ns))
          break;
        const uint32_t vd = sbase + L::kV + sv * kTileBytes;
        mbar_arrive_expect_tx(v_full(sv), kTileBytes);
        tma_load_4d(vd, &tma_v, v_full(sv), 0, j * kTile, hk, b);
        tma_load_4d(vd + kBox, &tma_v, v_full(sv), 64, j * kTile, hk, b);
        ++issued_v;
      }
      // let every issued copy land before the CTA may leave (bounded)
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(q_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int j = issued_k > kKStages ? issued_k - kKStages : 0; j < issued_k; ++j) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(k_full(j % kKStages), (j / kKStages) & 1) &&
               tc::globaltimer() - t0 < wait_ns) {
        }
      }
      for (int j = issued_v > kVStages ? issued_v - kVStages : 0; j < issued_v; ++j) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(v_full(j % kVStages), (j / kVStages) & 1) &&
               tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(q_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      // S_X(j) = Q_X K(j)^T; tile B is the last reader of K(j) and of V(j)
      auto issue_s = [&](int x, int j) -> bool {
        const int sk = j % kKStages;
        if (!bounded_wait(k_full(sk), (j / kKStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        // the softmax has read S_X(j - 1) for the last time
        if (j > 0 && !bounded_wait(s_free(x), (j - 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        tc_fence_after();
        const uint32_t qa = sbase + L::kQ + x * kTileBytes, kb = sbase + L::kK + sk * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)
          tc_mma_bf16(tmem + x * 128, desc_kmajor(qa, kk), desc_kmajor(kb, kk), kIdescKK,
                      kk > 0 ? 1u : 0u);
        tc_commit(s_full(x));
        if (x == 1) tc_commit(k_empty(sk));
        issued = true;
        return true;
      };
      // O_X (+)= P_X V(j), P_X from shared memory
      auto issue_pv = [&](int x, int j) -> bool {
        const int sv = j % kVStages;
        if (!bounded_wait(v_full(sv), (j / kVStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (!bounded_wait(p_full(x), j & 1, abort_flag, err, kErrAttnMma, wait_ns)) return false;
        tc_fence_after();
        const uint32_t pa = sbase + L::kP + x * kTileBytes, vb = sbase + L::kV + sv * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          tc_mma_bf16(tmem + 256 + x * 128, desc_kmajor(pa, kk), desc_mnmajor(vb, kk), kIdescKM,
                      (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pv_done(x));
        if (x == 1) tc_commit(v_empty(sv));
        return true;
      };
      // per key tile j: S_A(j + 1) as soon as the softmax of A has read S_A(j), then
      // A's P V, then the same for B; each query tile's next S overlaps its softmax
      if (ok && nkv_a > 0) ok = issue_s(0, 0);
      if (ok) ok = issue_s(1, 0);
      for (int j = 0; j < nkv_b && ok; ++j) {
        if (j < nkv_a) {
          if (j + 1 < nkv_a && !(ok = issue_s(0, j + 1))) break;
          if (!(ok = issue_pv(0, j))) break;
        }
        if (j + 1 < nkv_b && !(ok = issue_s(1, j + 1))) break;
        if (!(ok = issue_pv(1, j))) break;
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
    const int x = (warp - 2) >> 2;      // query tile A (0) or B (1)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of this thread within its tile
    const int qt = 2 * pr + x;
    const int q = qt * kTile + r;
    const int nkv = x ? nkv_b : nkv_a;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t st_t = tmem + x * 128 + lane_off;        // S_X
    const uint32_t o_t = tmem + 256 + x * 128 + lane_off;   // O_X
    uint8_t* pbox = smem + L::kP + x * kTileBytes;            // P_X: keys 0-63, then 64-127
    const uint64_t sl2 = f2_pack(a.scale_log2, a.scale_log2);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // -inf for keys beyond the sequence and (causal) keys after the query
    auto mask32 = [&](float (&v)[32], int key0) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int key = key0 + i;
        if (key >= a.S || (a.causal && key > q)) v[i] = -INFINITY;
      }
    };
    auto max32 = [&](const float (&v)[32]) -> float {
      float mx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx[u] = v[u];
#pragma unroll
      for (int i = 8; i < 32; i += 8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = fmaxf(mx[u], v[i + u]);
      }
      return fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
    };
    // exp2(v * scale_log2 - m) of 32 keys into 16 packed bf16 pairs, added to the
    // eight packed partial sums sm2 (chains fixed by key position)
    auto exp32 = [&](const float (&v)[32], uint64_t nm2, uint32_t (&w)[16], uint64_t (&sm2)[4]) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
#pragma unroll
        for (int u = 0; u < 8; u += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(v[i + u], v[i + u + 1]), sl2, nm2), x0, x1);
          x0 = fast_exp2(x0);
          x1 = fast_exp2(x1);
          sm2[u >> 1] = f2_add(sm2[u >> 1], f2_pack(x0, x1));
          w[(i + u) >> 1] = pack_bf16(x0, x1);
        }
      }
    };
    for (int j = 0; j < nkv && ok; ++j) {
      bool w = true;
      if (lane == 0) w = bounded_wait(s_full(x), j & 1, abort_flag, err, kErrAttnSoftmax, wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      const int k0 = j * kTile;
      const bool edge = (k0 + kTile > a.S) || (a.causal && j == qt);
      // pass 1: the row maximum of the raw logits (the scale is positive): keys
      // 0-63, then keys 64-127, which stay in registers
      float s[kHalf];
      tmem_ld32_async(st_t, *reinterpret_cast<float(*)[32]>(s));
      tmem_ld32_async(st_t + 32, *reinterpret_cast<float(*)[32]>(s + 32));
      tmem_ld_wait();
      if (edge) {
        mask32(*reinterpret_cast<float(*)[32]>(s), k0);
        mask32(*reinterpret_cast<float(*)[32]>(s + 32), k0 + 32);
      }
      const float m0 = fmaxf(max32(*reinterpret_cast<float(*)[32]>(s)),
                             max32(*reinterpret_cast<float(*)[32]>(s + 32)));
      tmem_ld32_async(st_t + 64, *reinterpret_cast<float(*)[32]>(s));
      tmem_ld32_async(st_t + 96, *reinterpret_cast<float(*)[32]>(s + 32));
      tmem_ld_wait();
      if (edge) {
        mask32(*reinterpret_cast<float(*)[32]>(s), k0 + 64);
        mask32(*reinterpret_cast<float(*)[32]>(s + 32), k0 + 96);
      }
      const float m1 = fmaxf(max32(*reinterpret_cast<float(*)[32]>(s)),
                             max32(*reinterpret_cast<float(*)[32]>(s + 32)));
      const float mt = fmaxf(m0, m1) * a.scale_log2;
      bool rescale = false;
      float alpha = 1.f;
      if (mt > m_used + 8.f) {  // also when m_used is still -inf
        alpha = fast_exp2(m_used - mt);
        m_used = mt;
        rescale = true;
      }
      const uint64_t nm2 = f2_pack(-m_used, -m_used);
      // the previous tile's P V product has read the P buffer, and O_X is stable
      if (j > 0) {
        if (lane == 0) w = bounded_wait(pv_done(x), (j - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
        tc_fence_after();
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
        // rescales O when any of its rows needs it (alpha = 1 for the others)
        if (__any_sync(0xffffffffu, rescale)) rescale_o_row(o_t, alpha);
      }
      // pass 2: keys 64-127 (still in registers) into P box 1, then keys 0-63, read
      // again, into box 0; S_X is free for the next tile's product after that read
      uint64_t sm2[4] = {0, 0, 0, 0};
      uint32_t pw[16];
      auto store4 = [&](uint8_t* box, int c0) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(box + swz_off(r, c0 + c)) =
              make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      };
      exp32(*reinterpret_cast<float(*)[32]>(s), nm2, pw, sm2);
      store4(pbox + kBox, 0);
      exp32(*reinterpret_cast<float(*)[32]>(s + 32), nm2, pw, sm2);
      store4(pbox + kBox, 4);
      tmem_ld32_async(st_t, *reinterpret_cast<float(*)[32]>(s));
      tmem_ld32_async(st_t + 32, *reinterpret_cast<float(*)[32]>(s + 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(x));
      if (edge) {
        mask32(*reinterpret_cast<float(*)[32]>(s), k0);
        mask32(*reinterpret_cast<float(*)[32]>(s + 32), k0 + 32);
      }
      exp32(*reinterpret_cast<float(*)[32]>(s), nm2, pw, sm2);
      store4(pbox, 0);
      exp32(*reinterpret_cast<float(*)[32]>(s + 32), nm2, pw, sm2);
      store4(pbox, 4);
      float sm[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) f2_unpack(sm2[u], sm[2 * u], sm[2 * u + 1]);
      const float sum = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      l = rescale ? l * alpha + sum : l + sum;
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(x));
    }
    if (ok && nkv > 0) {
      bool w = true;
      if (lane == 0) w = bounded_wait(pv_done(x), (nkv - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                      wait_ns);
      ok = warp_ok(w);
    }
    if (ok && nkv > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = a.out + ((int64_t)b * a.S + q) * (int64_t)(a.H * kHeadDim) + h * kHeadDim;
#pragma unroll
      for (int c = 0; c < kHeadDim / 32; ++c) {
        float o[32];
        tmem_ld32(o_t + c * 32, o);
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
// D[b, h, q] = sum_d dO[b, q, h, d] * O[b, q, h, d] (fp32) and nl2[b, h, q] =
// -lse[b, h, q] * log2(e) (the exponent offset of P in base 2); rows padded
// like lse ([B, H, S_pad]). dO and O are [B, S, H, D] contiguous. Sixteen lanes
// per row (16 bytes each), rows taken in the output's (b, h, q) order so the
// stores are contiguous, four rows per half-warp with all loads issued first.
constexpr int kDotRows = 4;
__global__ void __launch_bounds__(256) attn_bwd_dot_kernel(const bf16* __restrict__ dO,
                                                           const bf16* __restrict__ O,
                                                           const float* __restrict__ lse, int B,
                                                           int H, int S, float* __restrict__ Dv,
                                                           float* __restrict__ nl2) {
  pdl_wait();
  pdl_trigger();
  const int64_t nrows = (int64_t)B * H * S;
  const int sub = threadIdx.x & 15;
  const int64_t half = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int64_t nhalves = ((int64_t)gridDim.x * blockDim.x) >> 4;
  const int64_t s_pad = (int64_t)(S + kTile - 1) / kTile * kTile;
  for (int64_t base = half * kDotRows; base < nrows; base += nhalves * kDotRows) {
    uint4 a[kDotRows], c[kDotRows];
#pragma unroll
    for (int u = 0; u < kDotRows; ++u) {
      const int64_t i = base + u;  // (b, h, q) row-major
      if (i < nrows) {
        const int q = (int)(i % S);
        const int64_t bh = i / S;
        const int h = (int)(bh % H), b = (int)(bh / H);
        const int64_t row = ((int64_t)b * S + q) * H + h;
        a[u] = *reinterpret_cast<const uint4*>(dO + row * kHeadDim + sub * 8);
        c[u] = *reinterpret_cast<const uint4*>(O + row * kHeadDim + sub * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < kDotRows; ++u) {
      const int64_t i = base + u;
      const __nv_bfloat162* ap = reinterpret_cast<const __nv_bfloat162*>(&a[u]);
      const __nv_bfloat162* cp = reinterpret_cast<const __nv_bfloat162*>(&c[u]);
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = __bfloat1622float2(ap[e]), y = __bfloat1622float2(cp[e]);
        acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (sub == 0 && i < nrows) {
        const int q = (int)(i % S);
        const int64_t v = (i / S) * s_pad + q;
        Dv[v] = acc;
        nl2[v] = -lse[v] * kLog2e;
      }
    }
  }
}

struct BwdArgs {
  int B, H, Hk, S;
  float scale;        // softmax scale (applied to dK, dQ in fp32)
  float scale_log2;   // scale * log2(e)
  int causal;
  const float* lse;   // [B, H, S_pad] from the forward (S_pad = S rounded up to 128)
  const float* Dv;    // [B, H, S_pad] from attn_bwd_dot_kernel
  const float* nl2;   // [B, H, S_pad] -lse * log2(e), from attn_bwd_dot_kernel
  float* dk_part;     // dK/dV kernel: fp32 [B, H, S, D] per query head
  float* dv_part;
  bf16* dq;           // dQ kernel: [B, S, H, D]
  uint64_t wait_ns;
};

// dK / dV partials of one query head for one 128-key tile, stepping through its
// queries 64 at a time. TMEM: S^T and dP^T (M 128 keys x N 64 queries) double
// buffered (buffer b: S^T at column 128 b, dP^T at 128 b + 64), dV at 256, dK at
// 384. Shared memory: K, V (32 KB each, loaded once), a ring of 3 stages of
// 64-query (Q, dO) tiles (16 KB each) with their nl2 / D vectors, and separate
// P^T and dS^T buffers (16 KB each: 128 keys x 64 queries, one swizzled box), so
// this step's P / dS are computed while the tensor core runs the next step's
// S^T / dP^T and this step's dV / dK products.
constexpr int kQStep = 64;                 // queries per dK / dV step
constexpr int kDkvStages = 3;
constexpr int kStepBox = kQStep * 128;     // a [64 rows x 64 cols] bf16 box: 8 KB
constexpr int kStepTile = 2 * kStepBox;    // a 64 x 128 bf16 tile: 16 KB
constexpr int kPTBytes = kTile * 128;      // P^T / dS^T: 128 rows x 64 bf16 = 16 KB
struct DkvSmem {
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTileBytes;
  static constexpr int kQD = kV + kTileBytes;  // stage s: Q at +0, dO at +kStepTile
  static constexpr int kP = kQD + kDkvStages * 2 * kStepTile;
  static constexpr int kDS = kP + kPTBytes;
  static constexpr int kVec = kDS + kPTBytes;  // stage s: nl2, D of its 64 queries (2 x 256 B)
  static constexpr int kBar = kVec + kDkvStages * 2 * kQStep * 4;
  // kv_full, qdo_full[3], qdo_empty[3], st_full[2], st_empty[2], p_full, p_free, ds_full,
  // ds_free, acc_done, drain
  static constexpr int kNumBars = 1 + 2 * kDkvStages + 4 + 6;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kUsed = kMisc + 16;
  // alignment slack up to the 227 KB limit: the kernel checks at entry that the
  // padding to the 1024-byte boundary of its dynamic shared memory fits
  static constexpr int kBytes = kUsed + 1024 <= 232448 ? kUsed + 1024 : 232448;
};
static_assert(DkvSmem::kUsed + 128 <= 232448, "attention dK/dV shared memory exceeds 227 KB");

// Descriptors of a 64-row step tile (two 8 KB boxes of 64 columns): as a K-major
// operand with N = 64 rows (k-step kk: 16 columns), and as an MN-major operand
// whose K dimension is its 64 rows (k-step kk: rows 16 kk..16 kk + 15; LBO 8 KB).
__device__ __forceinline__ uint64_t desc_kmajor64(uint32_t base, int kk) {
  return smem_desc_sw128(base + (kk >> 2) * kStepBox + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t desc_mnmajor64(uint32_t base, int kk) {
  return smem_desc_sw128(base + kk * 2048, kStepBox, 1024);
}
// P^T / dS^T (128 rows x 64 columns, one box) as the K-major A operand.
__device__ __forceinline__ uint64_t desc_kmajor_box(uint32_t base, int kk) {
  return smem_desc_sw128(base + kk * 32, 16, 1024);
}
constexpr uint32_t kIdescKK64 = tc::idesc_bf16(64, false, false, 128);  // M 128, N 64

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

// Half a row of a packed bf16 tile (32 words = the 64 values of this thread's
// row in one column half) into that half's 64-column swizzled box.
__device__ __forceinline__ void store_half_row(uint8_t* box, int r, const uint32_t (&w)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(box + swz_off(r, c)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Rows of a packed bf16 tile (64 words = 128 values of this thread's row) into
// the K-major swizzled layout of a 128 x 128 operand tile.
__device__ __forceinline__ void store_row_tile(uint8_t* tile, int r, const uint32_t (&w)[64]) {
#pragma unroll
  for (int c = 0; c < 16; ++c)
    *reinterpret_cast<uint4*>(tile + (c >> 3) * kBox + swz_off(r, c & 7)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Maps: K / V over [B, Hk, S, D] (128-row boxes), Q over [B, H, S, D] and dO
// over [B, S, H, D] viewed as [B, H, S, D] (strides S*H*D, D, H*D), both with
// 64-row boxes.
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
  auto qdo_empty = [&](int st) { return bar0 + 8u * (1 + kDkvStages + st); };
  constexpr int kB = 1 + 2 * kDkvStages;
  auto st_full = [&](int bb) { return bar0 + 8u * (kB + bb); };
  auto st_empty = [&](int bb) { return bar0 + 8u * (kB + 2 + bb); };
  const uint32_t p_full = bar0 + 8u * (kB + 4), p_free = bar0 + 8u * (kB + 5);
  const uint32_t ds_full = bar0 + 8u * (kB + 6), ds_free = bar0 + 8u * (kB + 7);
  const uint32_t acc_done = bar0 + 8u * (kB + 8), drain_bar = bar0 + 8u * (kB + 9);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = (a.S + kTile - 1) / kTile;
  const int nq64 = (a.S + kQStep - 1) / kQStep;
  const int bh = blockIdx.x % (a.B * a.H);
  const int kt = blockIdx.x / (a.B * a.H);  // causal: early key tiles have the most queries
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  const int k0 = kt * kTile;
  const int step_first = a.causal ? kt * (kTile / kQStep) : 0;
  const int n = nq64 - step_first;
  const int64_t s_pad = (int64_t)nq * kTile;
  const uint64_t wait_ns = a.wait_ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < L::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      const bool per_warp = bar == st_empty(0) || bar == st_empty(1) || bar == p_full ||
                            bar == ds_full;
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
        const int st = i % kDkvStages;
        if (!bounded_wait(qdo_empty(st), ((i / kDkvStages) & 1) ^ 1, abort_flag, err,
                          kErrAttnProducer, wait_ns))
          break;
        const int q0 = (step_first + i) * kQStep;
        const uint32_t qd = sbase + L::kQD + st * 2 * kStepTile;
        const int64_t vrow = ((int64_t)b * a.H + h) * s_pad + q0;
        const uint32_t vd = sbase + L::kVec + st * 2 * kQStep * 4;
        mbar_arrive_expect_tx(qdo_full(st), 2 * kStepTile + 2 * kQStep * 4);
        tma_load_4d(qd, &tma_q, qdo_full(st), 0, q0, h, b);
        tma_load_4d(qd + kStepBox, &tma_q, qdo_full(st), 64, q0, h, b);
        tma_load_4d(qd + kStepTile, &tma_do, qdo_full(st), 0, q0, h, b);
        tma_load_4d(qd + kStepTile + kStepBox, &tma_do, qdo_full(st), 64, q0, h, b);
        bulk_load(vd, a.nl2 + vrow, kQStep * 4, qdo_full(st));
        bulk_load(vd + kQStep * 4, a.Dv + vrow, kQStep * 4, qdo_full(st));
        ++issued;
      }
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(kv_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int i = issued > kDkvStages ? issued - kDkvStages : 0; i < issued; ++i) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(qdo_full(i % kDkvStages), (i / kDkvStages) & 1) &&
               tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(kv_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      const uint32_t ka = sbase + L::kK, va = sbase + L::kV;
      const uint32_t pa = sbase + L::kP, dsa = sbase + L::kDS;
      auto issue_sd = [&](int i) -> bool {
        const int st = i % kDkvStages, bb = i & 1;
        if (!bounded_wait(qdo_full(st), (i / kDkvStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (i >= 2 && !bounded_wait(st_empty(bb), ((i >> 1) & 1) ^ 1, abort_flag, err, kErrAttnMma,
                                    wait_ns))
          return false;
        tc_fence_after();
        const uint32_t qd = sbase + L::kQD + st * 2 * kStepTile;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // S^T = K Q^T
          tc_mma_bf16(tmem + bb * 128, desc_kmajor(ka, kk), desc_kmajor64(qd, kk), kIdescKK64,
                      kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // dP^T = V dO^T
          tc_mma_bf16(tmem + bb * 128 + 64, desc_kmajor(va, kk), desc_kmajor64(qd + kStepTile, kk),
                      kIdescKK64, kk > 0 ? 1u : 0u);
        tc_commit(st_full(bb));
        issued = true;
        return true;
      };
      if (ok && n > 0) ok = issue_sd(0);
      if (ok && n > 1) ok = issue_sd(1);
      for (int i = 0; i < n && ok; ++i) {
        const int st = i % kDkvStages;
        const uint32_t qd = sbase + L::kQD + st * 2 * kStepTile;
        if (!(ok = bounded_wait(p_full, i & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kQStep / 16; ++kk)  // dV += P^T dO
          tc_mma_bf16(tmem + 256, desc_kmajor_box(pa, kk), desc_mnmajor64(qd + kStepTile, kk),
                      kIdescKM, (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(p_free);
        if (!(ok = bounded_wait(ds_full, i & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kQStep / 16; ++kk)  // dK += dS^T Q
          tc_mma_bf16(tmem + 384, desc_kmajor_box(dsa, kk), desc_mnmajor64(qd, kk), kIdescKM,
                      (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(ds_free);
        tc_commit(qdo_empty(st));
        if (i + 2 < n && !(ok = issue_sd(i + 2))) break;
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
    const int half = (warp - 2) >> 2;   // queries [32 half, 32 half + 32) of each 64-query step
    const int cb = half * (kQStep / 2);
    const int r = quarter * 32 + lane;  // key row of this thread
    const int key = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* pbox = smem + L::kP;
    uint8_t* dsbox = smem + L::kDS;
    const uint64_t sl2 = f2_pack(a.scale_log2, a.scale_log2);
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int st = i % kDkvStages, bb = i & 1;
      const int q0 = (step_first + i) * kQStep + cb;
      bool w = true;
      if (lane == 0) w = bounded_wait(st_full(bb), (i >> 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                      wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      float sv[32], dp[32];
      tmem_ld32_async(tmem + bb * 128 + cb + lane_off, sv);
      tmem_ld32_async(tmem + bb * 128 + 64 + cb + lane_off, dp);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(st_empty(bb));  // the step after next may overwrite them
      const float* vnl = reinterpret_cast<const float*>(smem + L::kVec + st * 2 * kQStep * 4) + cb;
      const float* vD = vnl + kQStep;
      const int qs = (step_first + i) * kQStep;
      const bool edge = (qs + kQStep > a.S) || (a.causal && qs < k0 + kTile);
      uint32_t pw[16], dw[16];
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 nl = *reinterpret_cast<const float4*>(vnl + e);
        const float4 dd = *reinterpret_cast<const float4*>(vD + e);
        float p[4], d[4];
        f2_unpack(f2_fma(f2_pack(sv[e], sv[e + 1]), sl2, f2_pack(nl.x, nl.y)), p[0], p[1]);
        f2_unpack(f2_fma(f2_pack(sv[e + 2], sv[e + 3]), sl2, f2_pack(nl.z, nl.w)), p[2], p[3]);
#pragma unroll
        for (int u = 0; u < 4; ++u) p[u] = fast_exp2(p[u]);
        const uint64_t t0 = f2_add(f2_pack(dp[e], dp[e + 1]), f2_pack(-dd.x, -dd.y));
        const uint64_t t1 = f2_add(f2_pack(dp[e + 2], dp[e + 3]), f2_pack(-dd.z, -dd.w));
        f2_unpack(f2_mul(f2_pack(p[0], p[1]), t0), d[0], d[1]);
        f2_unpack(f2_mul(f2_pack(p[2], p[3]), t1), d[2], d[3]);
        if (edge) {  // padding rows of nl2 / D may hold anything: select, do not scale
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int q = q0 + e + u;
            if (q >= a.S || (a.causal && q < key)) p[u] = d[u] = 0.f;
          }
        }
        pw[e >> 1] = pack_bf16(p[0], p[1]);
        pw[(e >> 1) + 1] = pack_bf16(p[2], p[3]);
        dw[e >> 1] = pack_bf16(d[0], d[1]);
        dw[(e >> 1) + 1] = pack_bf16(d[2], d[3]);
      }
      if (i > 0) {  // the previous step's dV product has read P^T
        if (lane == 0) w = bounded_wait(p_free, (i - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(pbox + swz_off(r, half * 4 + c)) =
            make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      tc::fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (i > 0) {  // the previous step's dK product has read dS^T
        if (lane == 0) w = bounded_wait(ds_free, (i - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(dsbox + swz_off(r, half * 4 + c)) =
            make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
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
      const int db = half * kHalf;  // this warp's 64 of the 128 head dims
      const int64_t row = (((int64_t)b * a.H + h) * a.S + key) * kHeadDim + db;
#pragma unroll
      for (int c = 0; c < kHalf / 32; ++c) {
        float v[32], g[32];
        tmem_ld32(tmem + 256 + db + c * 32 + lane_off, v);
        tmem_ld32(tmem + 384 + db + c * 32 + lane_off, g);
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

// dQ of one query tile: TMEM columns S 0, dP 128, dQ 256, dS 384 (bf16, two per
// column: the A operand of dQ += dS K read from TMEM). Shared memory: Q and dO
// (32 KB each, loaded once), a K ring (3 x 32 KB; a stage frees after its dQ
// product) and a V ring (2 x 32 KB; a stage frees after its dP product).
constexpr int kDqKStages = 3;
constexpr int kDqVStages = 2;
struct DqSmem {
  static constexpr int kQ = 0;
  static constexpr int kDO = kQ + kTileBytes;
  static constexpr int kK = kDO + kTileBytes;
  static constexpr int kV = kK + kDqKStages * kTileBytes;
  static constexpr int kBar = kV + kDqVStages * kTileBytes;
  // qdo_full, k_full[3], k_empty[3], v_full[2], v_empty[2], st_full, st_empty, ds_full,
  // buf_free, acc_done, drain
  static constexpr int kNumBars = 1 + 2 * kDqKStages + 2 * kDqVStages + 6;
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
  auto k_full = [&](int st) { return bar0 + 8u * (1 + st); };
  auto k_empty = [&](int st) { return bar0 + 8u * (1 + kDqKStages + st); };
  auto v_full = [&](int st) { return bar0 + 8u * (1 + 2 * kDqKStages + st); };
  auto v_empty = [&](int st) { return bar0 + 8u * (1 + 2 * kDqKStages + kDqVStages + st); };
  constexpr int kB = 1 + 2 * kDqKStages + 2 * kDqVStages;
  const uint32_t st_full = bar0 + 8u * kB, st_empty = bar0 + 8u * (kB + 1);
  const uint32_t ds_full = bar0 + 8u * (kB + 2), buf_free = bar0 + 8u * (kB + 3);
  const uint32_t acc_done = bar0 + 8u * (kB + 4), drain_bar = bar0 + 8u * (kB + 5);
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
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n; ++j) {
        const int sk = j % kDqKStages, sv = j % kDqVStages;
        if (!bounded_wait(k_empty(sk), ((j / kDqKStages) & 1) ^ 1, abort_flag, err,
                          kErrAttnProducer, wait_ns))
          break;
        const uint32_t kd = sbase + L::kK + sk * kTileBytes;
        mbar_arrive_expect_tx(k_full(sk), kTileBytes);
        tma_load_4d(kd, &tma_k, k_full(sk), 0, j * kTile, hk, b);
        tma_load_4d(kd + kBox, &tma_k, k_full(sk), 64, j * kTile, hk, b);
        ++issued_k;
        if (!bounded_wait(v_empty(sv), ((j / kDqVStages) & 1) ^ 1, abort_flag, err,
                          kErrAttnProducer, wait_ns))
          break;
        const uint32_t vd = sbase + L::kV + sv * kTileBytes;
        mbar_arrive_expect_tx(v_full(sv), kTileBytes);
        tma_load_4d(vd, &tma_v, v_full(sv), 0, j * kTile, hk, b);
        tma_load_4d(vd + kBox, &tma_v, v_full(sv), 64, j * kTile, hk, b);
        ++issued_v;
      }
      uint64_t t0 = tc::globaltimer();
      while (!mbar_try_wait(qdo_full, 0) && tc::globaltimer() - t0 < wait_ns) {
      }
      for (int j = issued_k > kDqKStages ? issued_k - kDqKStages : 0; j < issued_k; ++j) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(k_full(j % kDqKStages), (j / kDqKStages) & 1) &&
               tc::globaltimer() - t0 < wait_ns) {
        }
      }
      for (int j = issued_v > kDqVStages ? issued_v - kDqVStages : 0; j < issued_v; ++j) {
        t0 = tc::globaltimer();
        while (!mbar_try_wait(v_full(j % kDqVStages), (j / kDqVStages) & 1) &&
               tc::globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      bool ok = bounded_wait(qdo_full, 0, abort_flag, err, kErrAttnMma, wait_ns);
      bool issued = false;
      const uint32_t qa = sbase + L::kQ, da = sbase + L::kDO;
      auto issue_sd = [&](int j) -> bool {
        const int sk = j % kDqKStages, sv = j % kDqVStages;
        if (!bounded_wait(k_full(sk), (j / kDqKStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (!bounded_wait(v_full(sv), (j / kDqVStages) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        if (j > 0 && !bounded_wait(st_empty, (j - 1) & 1, abort_flag, err, kErrAttnMma, wait_ns))
          return false;
        tc_fence_after();
        const uint32_t kd = sbase + L::kK + sk * kTileBytes;
        const uint32_t vd = sbase + L::kV + sv * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // S = Q K^T
          tc_mma_bf16(tmem, desc_kmajor(qa, kk), desc_kmajor(kd, kk), kIdescKK, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)  // dP = dO V^T
          tc_mma_bf16(tmem + 128, desc_kmajor(da, kk), desc_kmajor(vd, kk), kIdescKK,
                      kk > 0 ? 1u : 0u);
        tc_commit(st_full);
        tc_commit(v_empty(sv));
        issued = true;
        return true;
      };
      if (ok && n > 0) ok = issue_sd(0);
      for (int j = 0; j < n && ok; ++j) {
        const int sk = j % kDqKStages;
        const uint32_t kd = sbase + L::kK + sk * kTileBytes;
        if (j + 1 < n && !(ok = issue_sd(j + 1))) break;
        if (!(ok = bounded_wait(ds_full, j & 1, abort_flag, err, kErrAttnMma, wait_ns))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dQ += dS K (dS from TMEM: 8 columns per 16 keys)
          tc_mma_bf16_tmem_a(tmem + 256, tmem + 384 + kk * 8, desc_mnmajor(kd, kk), kIdescKM,
                             (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(buf_free);
        tc_commit(k_empty(sk));
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
    const int half = (warp - 2) >> 2;   // key columns [64 half, 64 half + 64) of S / dP
    const int cb = half * kHalf;
    const int r = quarter * 32 + lane;  // query row of this thread
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int64_t vidx = ((int64_t)b * a.H + h) * ((int64_t)nq * kTile) + q;
    const float nl = q < a.S ? -a.lse[vidx] * kLog2e : 0.f;
    const float dq_d = q < a.S ? a.Dv[vidx] : 0.f;
    const uint64_t sl2 = f2_pack(a.scale_log2, a.scale_log2);
    const uint64_t nl2 = f2_pack(nl, nl), nd2 = f2_pack(-dq_d, -dq_d);
    // this half's 64 keys of dS: 32 columns of bf16 pairs from column 384 + 32 half
    const uint32_t ds_tmem = tmem + 384 + half * (kHalf / 2) + lane_off;
    bool ok = true;
    for (int j = 0; j < n && ok; ++j) {
      bool w = true;
      if (lane == 0) w = bounded_wait(st_full, j & 1, abort_flag, err, kErrAttnSoftmax, wait_ns);
      if (!(ok = warp_ok(w))) break;
      tc_fence_after();
      float sv[kHalf], dp[kHalf];
      tmem_ld32_async(tmem + cb + lane_off, *reinterpret_cast<float(*)[32]>(sv));
      tmem_ld32_async(tmem + cb + 32 + lane_off, *reinterpret_cast<float(*)[32]>(sv + 32));
      tmem_ld32_async(tmem + 128 + cb + lane_off, *reinterpret_cast<float(*)[32]>(dp));
      tmem_ld32_async(tmem + 128 + cb + 32 + lane_off, *reinterpret_cast<float(*)[32]>(dp + 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(st_empty);  // the next tile's S / dP may overwrite them
      const int k0 = j * kTile + cb;
      const bool edge = (j * kTile + kTile > a.S) || (a.causal && j == qt);
      uint32_t dw[kHalf / 2];
#pragma unroll
      for (int e = 0; e < kHalf; e += 2) {
        float p0, p1, d0, d1;
        f2_unpack(f2_fma(f2_pack(sv[e], sv[e + 1]), sl2, nl2), p0, p1);
        p0 = fast_exp2(p0);
        p1 = fast_exp2(p1);
        f2_unpack(f2_mul(f2_pack(p0, p1), f2_add(f2_pack(dp[e], dp[e + 1]), nd2)), d0, d1);
        if (edge) {
          const int key = k0 + e;
          if (key >= a.S || (a.causal && key > q)) d0 = 0.f;
          if (key + 1 >= a.S || (a.causal && key + 1 > q)) d1 = 0.f;
        }
        dw[e >> 1] = pack_bf16(d0, d1);
      }
      if (j > 0) {  // the previous tile's dQ product has read dS
        if (lane == 0) w = bounded_wait(buf_free, (j - 1) & 1, abort_flag, err, kErrAttnSoftmax,
                                        wait_ns);
        if (!(ok = warp_ok(w))) break;
        tc_fence_after();
      }
      tmem_st32u(ds_tmem, dw);
      tmem_st_wait();
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
      bf16* orow = a.dq + ((int64_t)b * a.S + q) * (int64_t)(a.H * kHeadDim) + h * kHeadDim + cb;
#pragma unroll
      for (int c = 0; c < kHalf / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + 256 + cb + c * 32 + lane_off, o);
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
#pragma unroll 6
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
                         int64_t heads, int64_t S, const char* what, int box_rows = kTile) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return SOUP_ERR_CUDA;
  }
  if (int rc = bind_context()) return rc;
  cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)S, (cuuint64_t)heads, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)strides[2] * 2, (cuuint64_t)strides[1] * 2,
                        (cuuint64_t)strides[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
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
  const int64_t npair = ((seq + kTile - 1) / kTile + 1) / 2;
  return cuda_status(launch_pdl(attn_fwd_kernel, dim3((unsigned)(batch * heads * npair)),
                                dim3(kFwdThreads), FwdSmem::kBytes, as_stream(stream), mq, mk, mv,
                                a, err));
}

size_t soup_attention_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const size_t s_pad = (size_t)((seq + kTile - 1) / kTile * kTile);
  const size_t dvec = (size_t)batch * heads * s_pad * 4;
  const size_t part = (size_t)batch * heads * seq * kHeadDim * 4;
  return 2 * ((dvec + 255) / 256 * 256) + 2 * ((part + 255) / 256 * 256);
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
  const size_t part = (size_t)batch * heads * seq * kHeadDim * 4;
  const size_t vbytes = ((size_t)batch * heads * s_pad * 4 + 255) / 256 * 256;
  float* dvec = reinterpret_cast<float*>(ws);
  float* nl2 = reinterpret_cast<float*>(ws + vbytes);
  float* dk_part = reinterpret_cast<float*>(ws + 2 * vbytes);
  float* dv_part = reinterpret_cast<float*>(ws + 2 * vbytes + (part + 255) / 256 * 256);
  CUtensorMap mq, mk, mv, mdo, mq64, mdo64;
  int rc;
  const int64_t do_strides[3] = {seq * heads * kHeadDim, kHeadDim, heads * kHeadDim};
  if ((rc = make_bhsd_map(&mq, q, q_strides, batch, heads, seq, "q"))) return rc;
  if ((rc = make_bhsd_map(&mk, k, k_strides, batch, kv_heads, seq, "k"))) return rc;
  if ((rc = make_bhsd_map(&mv, v, v_strides, batch, kv_heads, seq, "v"))) return rc;
  if ((rc = make_bhsd_map(&mdo, dout, do_strides, batch, heads, seq, "dout"))) return rc;
  if ((rc = make_bhsd_map(&mq64, q, q_strides, batch, heads, seq, "q", kQStep))) return rc;
  if ((rc = make_bhsd_map(&mdo64, dout, do_strides, batch, heads, seq, "dout", kQStep))) return rc;
  static bool dkdv_set[64] = {false}, dq_set[64] = {false};
  if ((rc = set_smem(attn_bwd_dkdv_kernel, DkvSmem::kBytes, dkdv_set))) return rc;
  if ((rc = set_smem(attn_bwd_dq_kernel, DqSmem::kBytes, dq_set))) return rc;
  cudaStream_t st = as_stream(stream);
  const int B = (int)batch, H = (int)heads, Hk = (int)kv_heads, S = (int)seq;
  const int64_t rows = (int64_t)B * S * H;
  int dot_blocks = (int)((rows + 16 * kDotRows - 1) / (16 * kDotRows));  // 16 half-warps per block
  if (dot_blocks > 16 * num_sms()) dot_blocks = 16 * num_sms();
  if ((rc = cuda_status(launch_pdl(attn_bwd_dot_kernel, dim3((unsigned)dot_blocks), dim3(256),
                                   0, st, static_cast<const bf16*>(dout),
                                   static_cast<const bf16*>(out), lse, B, H, S, dvec, nl2))))
    return rc;
  BwdArgs a{B, H, Hk, S, scale, scale * 1.4426950408889634f, causal ? 1 : 0, lse, dvec, nl2,
            dk_part, dv_part, static_cast<bf16*>(dq), 0};
  a.wait_ns = wait_limit_ns() ? wait_limit_ns() : tc::kWaitNs;
  const int nt = (S + kTile - 1) / kTile;
  if ((rc = cuda_status(launch_pdl(attn_bwd_dkdv_kernel, dim3((unsigned)(B * H * nt)),
                                   dim3(kBwdThreads), DkvSmem::kBytes, st, mq64, mk, mv, mdo64, a,
                                   err))))
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
