// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
//   C[m, n] = sum_k A(m, k) * B(n, k)  [+ sum_k2 A2(m, k2) * B2(n, k2)]
//
// The optional second K segment (Sched::kb2 > 0 blocks, read through the
// tensor maps tma_a2 / tma_b2 with the same majorness as A / B) follows the
// first in the same accumulator: a low-rank update such as a LoRA term
// x A^T B^T rides on the base GEMM as one or two extra k-blocks, its columns
// beyond the rank zero-filled by TMA (out-of-bounds box elements).
//
// A and B are each either K-major (stored [rows, K], K contiguous) or
// MN-major (stored [K, rows], rows contiguous); both are loaded by 2-D TMA
// with the 128-byte swizzle and described to the MMA with matching shared
// memory descriptors. One CTA per SM (grid <= #SMs) walks a static tile list:
//
//   warp 0      TMA producer (one elected lane)      smem ring of STAGES
//   warp 1      TMEM allocator + MMA issuer (lane 0)  2 accumulators in TMEM
//   warps 2..   epilogue (EPI_WARPS = 4 or 8): tcgen05.ld -> registers -> Epi::tile(...);
//               warp w reads TMEM lane quarter w % 4; with 8 warps the two
//               warps of a quarter take the left / right half of the columns
//
// Each tile is BM=128 rows x BN columns with BK=64 per stage; the MMA shape
// is 128 x BN x 16. The TMEM accumulators are double buffered (2 x BN fp32
// columns), so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Every mbarrier wait is bounded (kWaitNs of wall time). On expiry the
// waiting role records an error code in the device error word (`err`),
// raises a CTA-wide abort flag, the producer waits (bounded) for its copies
// still in flight, the MMA warp drains its MMAs, and the CTA frees its TMEM
// and exits. Every TMA load writes only this CTA's own shared memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <type_traits>

#include "soup_common.cuh"

namespace soup {
namespace tc {

// An epilogue whose warps read, of a tile's 32-column chunks, half their run
// in each half of the tile (not one contiguous run) declares
//   static constexpr bool kHalves = true;
template <class Epi, class = void>
struct EpiHalves {
  static constexpr bool value = false;
};
template <class Epi>
struct EpiHalves<Epi, std::void_t<decltype(Epi::kHalves)>> {
  static constexpr bool value = Epi::kHalves;
};

// An epilogue may declare `struct Carry` and
//   static void prefetch(const Params&, int row_base, int nt, int quarter, int lane,
//                        int group, int ngroups, Carry&);
// the kernel then calls prefetch for each tile before waiting for its
// accumulator (to start global loads the epilogue will need) and passes the
// Carry to tile() as its last argument.
template <class Epi, class = void>
struct EpiCarry {
  struct type {};
  static constexpr bool kHas = false;
};
template <class Epi>
struct EpiCarry<Epi, std::void_t<typename Epi::Carry>> {
  using type = typename Epi::Carry;
  static constexpr bool kHas = true;
};

constexpr int BM = 128;
constexpr int BK = 64;
// threads of a CTA with `epi_warps` epilogue warps (+ producer and MMA warps)
__host__ __device__ constexpr int gemm_threads(int epi_warps) { return 64 + 32 * epi_warps; }
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

// error codes written to the device error word
constexpr int kErrWaitProducer = 0x101;
constexpr int kErrWaitMma = 0x102;
constexpr int kErrWaitEpilogue = 0x103;
constexpr int kErrWaitPartial = 0x104;  // a stream-K partial never became ready

// ------------------------------------------------------------ PTX wrappers --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Same, acquiring at cluster scope (arrivals that come from the peer CTA).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// 2-D TMA tile load into this CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
// 2-D TMA store of a tile from this CTA's shared memory (bulk async-group of
// the issuing thread; out-of-bounds parts of the box are not written).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most one of this thread's bulk groups still reading shared memory
__device__ __forceinline__ void bulk_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the async proxy (TMA)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// MMA completion -> mbarrier arrive (tracks all prior tcgen05 ops of this thread).
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 or fp16 in, as the
// instruction descriptor says; fp32 accumulate).
__device__ __forceinline__ void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread t of the warp receives
// row (lane base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();  // .sync.aligned: the whole warp executes the load converged
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
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// The inverse of tmem_ld32: thread t writes row (lane base + t), columns
// [col, col+32); returns once the stores are complete.
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
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// gpu-scope flag accesses between CTAs of one grid
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Shared-memory matrix descriptor (sm_100 format): start address, leading
// and stride byte offsets (16-byte units), version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp32 accumulate, bf16 A and B, M=bm, N=bn (bits 7-9
// and 10-12 are the A / B formats: 1 bf16, 0 fp16; see Sched::idesc).
__host__ __device__ constexpr uint32_t idesc_bf16(int bn, bool a_mn, bool b_mn, int bm = BM) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(bn >> 3) << 17) |
         (static_cast<uint32_t>(bm >> 4) << 24);
}

// ---------------------------------------------------------- tile schedule --
// A work unit is (m tile, n tile, k split). order 0: m fastest (operand B
// streamed once while A stays hot in L2); order 1: n fastest (A streamed).
// The k split is the slowest index so concurrently running units share k.
struct Sched {
  int m_tiles, n_tiles, splits;
  int kb_total;  // number of BK blocks along K (both segments)
  int order;
  int kb2;       // trailing blocks of kb_total read from the second segment (0: none)
  // optional device flag written by an earlier kernel on the stream: when it
  // reads 0 the whole grid returns at entry (a conditional launch that needs
  // no host round trip)
  const int* gate = nullptr;
  // 1: k splits run last-first (the first wave reads the end of K, e.g. what
  // the previous GEMM over the same operand left in L2)
  int rev_split = 0;
  // limit of every mbarrier wait in ns (0: kWaitNs)
  uint64_t wait_ns = 0;
  // diagnostic only (soup_gemm_wait_expiry_check): the producer skips the copies
  // and the expected-bytes arrive of its k-block iteration `withhold` (>= 0), so
  // the MMA issuer's wait for that stage expires; -1 in every normal launch
  int withhold = -1;
  // 1: A and B are fp16 (kind::f16 with the f16 operand format) instead of bf16
  int ab_f16 = 0;
  __device__ __forceinline__ uint64_t limit() const { return wait_ns ? wait_ns : kWaitNs; }
  // the instruction descriptor with the operand format of this launch
  __device__ __forceinline__ uint32_t idesc(uint32_t bf16_desc) const {
    return ab_f16 ? (bf16_desc & ~((7u << 7) | (7u << 10))) : bf16_desc;
  }
  // maps and k offset of block kb
  __device__ __forceinline__ bool second(int kb) const { return kb >= kb_total - kb2; }
  __device__ __forceinline__ int k_elem(int kb) const {
    return (second(kb) ? kb - (kb_total - kb2) : kb) * BK;
  }
  __device__ __forceinline__ int units() const { return m_tiles * n_tiles * splits; }
  __device__ __forceinline__ void decode(int u, int& mt, int& nt, int& ks) const {
    int mn = m_tiles * n_tiles;
    ks = u / mn;
    int r = u - ks * mn;
    if (rev_split) ks = splits - 1 - ks;
    if (order == 0) {
      mt = r % m_tiles;
      nt = r / m_tiles;
    } else {
      nt = r % n_tiles;
      mt = r / n_tiles;
    }
  }
  __device__ __forceinline__ void k_range(int ks, int& kb0, int& kb1) const {
    int base = kb_total / splits, rem = kb_total % splits;
    kb0 = ks * base + min(ks, rem);
    kb1 = kb0 + base + (ks < rem ? 1 : 0);
  }

  // ---- stream-K tail (pair kernel only; splits == 1; 0 = off) ----
  // The first m_tiles * n_tiles - sk_tiles tiles of the unit order go whole
  // to the clusters, round-robin (a multiple of the cluster count). The k
  // blocks of the last sk_tiles tiles, concatenated tile after tile, are cut
  // into sk_clusters contiguous segments of equal length (+-1), one for each
  // of the first sk_clusters clusters, which do them before their whole
  // tiles. A segment covers the end of one tile and/or the start of the next.
  // The cluster holding a tile's last k block finishes it: it adds the fp32
  // partial accumulators of the tile's earlier parts, each left by the
  // cluster that computed it in that cluster's slot of sk_part, in the order
  // of k, then runs the epilogue. A cluster computes at most one such
  // earlier part, so one slot per cluster suffices. sk_flag holds one ready
  // flag per (slot, CTA of the pair, epilogue warp): set by the warp that
  // wrote that piece of the slot, cleared by the warp that consumed it, so
  // the flags are zero between launches.
  int sk_tiles = 0;
  int sk_clusters = 0;
  float* sk_part = nullptr;
  int* sk_flag = nullptr;

  __device__ __forceinline__ void tile_of(int t, int& mt, int& nt) const {
    if (order == 0) {
      mt = t % m_tiles;
      nt = t / m_tiles;
    } else {
      nt = t % n_tiles;
      mt = t / n_tiles;
    }
  }
  // concatenated stream-K k-iterations [g0, g1) of cluster c (the launcher
  // keeps sk_tiles * kb_total * sk_clusters below 2^31: 32-bit math)
  __device__ __forceinline__ void sk_segment(int c, int& g0, int& g1) const {
    g0 = g1 = 0;
    if (c >= sk_clusters) return;
    const int s = sk_tiles * kb_total;
    g0 = s * c / sk_clusters;
    g1 = s * (c + 1) / sk_clusters;
  }
  // the cluster whose segment holds concatenated k-iteration g
  __device__ __forceinline__ int sk_owner(int g) const {
    return ((g + 1) * sk_clusters - 1) / (sk_tiles * kb_total);
  }
  __device__ __forceinline__ int sk_parts(int c) const {
    int g0, g1;
    sk_segment(c, g0, g1);
    if (g1 <= g0) return 0;
    return (g0 / kb_total != (g1 - 1) / kb_total) ? 2 : 1;
  }
  // number of units in cluster c's list (of n_clusters)
  __device__ __forceinline__ int cluster_units(int c, int n_clusters) const {
    if (sk_tiles == 0) return c < units() ? (units() - c + n_clusters - 1) / n_clusters : 0;
    const int t_whole = m_tiles * n_tiles - sk_tiles;
    const int n = c < t_whole ? (t_whole - c + n_clusters - 1) / n_clusters : 0;
    return n + sk_parts(c);
  }
};

// Role of a unit in a stream-K tail.
constexpr int kRoleWhole = 0;   // the whole k range: epilogue as usual
constexpr int kRolePart = 1;    // an earlier k part: fp32 partial into this cluster's slot
constexpr int kRoleFinish = 2;  // the last k part: add the slots [fix_lo, fix_hi), then epilogue

struct Unit {
  int mt, nt, ks, kb0, kb1;
  int role, fix_lo, fix_hi;
};

// Unit i of cluster c's list: its stream-K parts first (the start of the
// later tile, then the end of the earlier one, so a cluster publishes its
// partial before it waits for others'), then its whole tiles.
__device__ __forceinline__ Unit sched_unit(const Sched& s, int c, int n_clusters, int i) {
  Unit w;
  w.role = kRoleWhole;
  w.fix_lo = w.fix_hi = 0;
  if (s.sk_tiles > 0) {
    const int n_sk = s.sk_parts(c);
    if (i < n_sk) {
      int g0, g1;
      s.sk_segment(c, g0, g1);
      const int kb = s.kb_total;
      const int t0 = g0 / kb;
      int t, lo, hi;
      if (n_sk == 2 && i == 0) {
        t = t0 + 1;
        lo = t * kb;
        hi = g1;
      } else if (n_sk == 2) {
        t = t0;
        lo = g0;
        hi = (t0 + 1) * kb;
      } else {
        t = t0;
        lo = g0;
        hi = g1;
      }
      w.ks = 0;
      w.kb0 = lo - t * kb;
      w.kb1 = hi - t * kb;
      s.tile_of(s.m_tiles * s.n_tiles - s.sk_tiles + t, w.mt, w.nt);
      if (w.kb1 < s.kb_total) {
        w.role = kRolePart;
      } else if (w.kb0 > 0) {
        w.role = kRoleFinish;
        w.fix_lo = s.sk_owner(t * kb);
        w.fix_hi = c;
      }
      return w;
    }
    i -= n_sk;
  }
  s.decode(c + i * n_clusters, w.mt, w.nt, w.ks);
  s.k_range(w.ks, w.kb0, w.kb1);
  return w;
}

// Per-epilogue-warp staging buffer: 32 rows x 32 fp32 (128 B per row); the
// 16-byte granule q of row r is stored at granule q ^ (r & 7) (bank-conflict
// free for both the row-per-thread writes and the row-segment reads).
constexpr int kStageRowBytes = 128;
constexpr int kEpiWarpBytes = 32 * kStageRowBytes;

__device__ __forceinline__ int stage_off(int row, int granule) {
  return row * kStageRowBytes + ((granule ^ (row & 7)) << 4);
}

template <int BN, int STAGES, int EPI_WARPS>
struct SmemLayout {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOff = STAGES * kStageBytes;
  static constexpr int kBarOff = kEpiOff + EPI_WARPS * kEpiWarpBytes;
  // full[S], empty[S], tfull[2], tempty[2], drain, then tmem base + abort flag
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kMiscOff + 16 + 1024;  // + alignment slack
};

// Bounded wait. Returns false when the CTA is aborting (timeout here or
// elsewhere); on a local timeout it records `code` and raises the flag.
template <bool CLUSTER = false>
__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity,
                                             volatile int* abort_flag, int* err, int code,
                                             uint64_t limit_ns) {
  auto try_wait = [&]() {
    return CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
  if (try_wait()) return true;
  uint64_t t0 = globaltimer();
  while (true) {
    if (try_wait()) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Epi must provide:
//   struct Params;
//   static __device__ void tile(const Params&, const CUtensorMap* tma_c /* the kernel's
//                               output map (valid when the launcher encoded one) */,
//                               int row_base /* first row of the CTA's
//                               128-row block */, int nt, int ks, int quarter,
//                               int lane, uint32_t tmem_acc /* lane base applied */,
//                               uint8_t* stage /* this warp's kEpiWarpBytes of smem */,
//                               int group, int ngroups /* column part of the tile */);
template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS>
__global__ void __launch_bounds__(gemm_threads(EPI_WARPS), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_a2,
                const __grid_constant__ CUtensorMap tma_b2,
                const __grid_constant__ CUtensorMap tma_c, Sched sched,
                typename Epi::Params ep, int* err) {
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "4 or 8 epilogue warps");
  using L = SmemLayout<BN, STAGES, EPI_WARPS>;
  if (sched.gate) {  // grid-uniform; the flag comes from an earlier kernel
    pdl_wait();
    if (*sched.gate == 0) return;
  }
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, multiple of 64");
  static_assert(2 * BN <= 512, "two accumulators must fit in 512 TMEM columns");
  constexpr int kTmemCols = (2 * BN <= 128) ? 128 : ((2 * BN <= 256) ? 256 : 512);
  constexpr uint32_t kIdesc = idesc_bf16(BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (sched.kb2 > 0) {
      tma_prefetch_desc(&tma_a2);
      tma_prefetch_desc(&tma_b2);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int n_units = sched.units();
  const uint64_t wait_ns = sched.limit();
  const uint32_t idesc = sched.idesc(kIdesc);
  pdl_wait();  // no thread touches global memory before this (see gemm_pair_kernel)

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        int mt, nt, ks, kb0, kb1;
        sched.decode(u, mt, nt, ks);
        sched.k_range(ks, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!bounded_wait(empty_bar(s), ph ^ 1u, abort_flag, err, kErrWaitProducer, wait_ns)) {
            ok = false;
            break;
          }
          if (static_cast<int>(it) == sched.withhold) continue;  // diagnostic launch only
          const uint32_t a_dst = sbase + s * L::kStageBytes;
          const uint32_t b_dst = a_dst + L::kABytes;
          mbar_arrive_expect_tx(full_bar(s), L::kStageBytes);
          const int k0 = sched.k_elem(kb);
          const bool seg2 = sched.second(kb);
          const CUtensorMap* ma = seg2 ? &tma_a2 : &tma_a;
          const CUtensorMap* mb = seg2 ? &tma_b2 : &tma_b;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(a_dst + j * 8192, ma, full_bar(s), mt * BM + j * 64, k0);
          } else {
            tma_load_2d(a_dst, ma, full_bar(s), k0, mt * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, mb, full_bar(s), nt * BN + j * 64, k0);
          } else {
            tma_load_2d(b_dst, mb, full_bar(s), k0, nt * BN);
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA leaves: wait for
        // the last min(it, STAGES) stages' full barriers (bounded).
        int n = it < (uint32_t)STAGES ? (int)it : STAGES;
        for (int i = 1; i <= n; ++i) {
          uint32_t j = it - i;
          uint32_t bar = full_bar(j % STAGES), ph = (j / STAGES) & 1u;
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(bar, ph) && globaltimer() - t0 < wait_ns) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++lt) {
        int mt, nt, ks, kb0, kb1;
        sched.decode(u, mt, nt, ks);
        sched.k_range(ks, kb0, kb1);
        const uint32_t acc = lt & 1u;
        const uint32_t acc_ph = (lt >> 1) & 1u;
        if (!bounded_wait(tempty_bar(acc), acc_ph ^ 1u, abort_flag, err, kErrWaitMma, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!bounded_wait(full_bar(s), ph, abort_flag, err, kErrWaitMma, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + s * L::kStageBytes;
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if (A_MN) ad = smem_desc_sw128(a_addr + k * 2048, 8192, 1024);
            else ad = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            if (B_MN) bd = smem_desc_sw128(b_addr + k * 2048, 8192, 1024);
            else bd = smem_desc_sw128(b_addr + k * 32, 16, 1024);
            tc_mma_bf16(tmem_d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(s));  // frees the stage once these MMAs finish
        }
        if (!ok) break;
        tc_commit(tfull_bar(acc));  // accumulator ready for the epilogue
      }
      if (!ok) {
        tc_commit(drain_bar);
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else {
    // ------------------------------------------------------ epilogue ----
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int e = warp - 2;
    constexpr int kGroups = EPI_WARPS / 4;
    const int group = e >> 2;
    uint8_t* stage = smem + L::kEpiOff + e * kEpiWarpBytes;
    typename EpiCarry<Epi>::type carry{};
    uint32_t lt = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++lt) {
      int mt, nt, ks;
      sched.decode(u, mt, nt, ks);
      if constexpr (EpiCarry<Epi>::kHas)
        Epi::prefetch(ep, mt * BM, nt, quarter, lane, group, kGroups, carry);
      const uint32_t acc = lt & 1u;
      const uint32_t acc_ph = (lt >> 1) & 1u;
      bool ok = true;
      if (lane == 0) ok = bounded_wait(tfull_bar(acc), acc_ph, abort_flag, err, kErrWaitEpilogue, wait_ns);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if constexpr (EpiCarry<Epi>::kHas)
        Epi::tile(ep, &tma_c, mt * BM, nt, ks, quarter, lane, taddr, stage, group, kGroups, carry);
      else
        Epi::tile(ep, &tma_c, mt * BM, nt, ks, quarter, lane, taddr, stage, group, kGroups);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores, if any, are complete
  }

  pdl_trigger();  // see gemm_pair_kernel
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}


// ============================================================ CTA pairs ====
// Same GEMM with a cluster of two CTAs on two SMs computing one 256 x BN
// tile (tcgen05 cta_group::2, MMA shape 256 x BN x 16). CTA rank r of the
// pair loads rows [r*128, r*128+128) of the A tile and columns
// [r*BN/2, (r+1)*BN/2) of the B tile into its own shared memory; the MMA,
// issued by rank 0 alone, reads both CTAs' halves and leaves rows
// [r*128, r*128+128) x BN columns of the accumulator in rank r's TMEM. Per SM
// a k-block now moves (128 + BN/2) x 64 operand elements instead of
// (128 + BN) x 64.
//
// Cross-CTA protocol (all waits bounded as in the 1-CTA kernel):
//   full[s]   rank 0's barrier only: rank 0 arms it with both CTAs' bytes;
//             both CTAs' TMA copies (cta_group::2) complete on it
//   empty[s]  one per CTA: rank 0's MMA completion arrives on both (one
//             commit with a two-CTA mask)
//   tfull[a]  one per CTA: the same, after a tile's last MMA
//   tempty[a] rank 0's only, count 2 x EPI_WARPS: every epilogue warp of both
//             CTAs arrives (rank 1 remotely) after draining its TMEM lanes
// A cluster barrier after set-up and before TMEM release keeps each CTA's
// shared memory alive while its peer may still signal it.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
// 2-D TMA tile into this CTA's shared memory, completing on an mbarrier that
// may live in the peer CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cluster_bar)
               : "memory");
}
// One commit that arrives on the barrier at offset `bar` in every CTA of
// `cta_mask` (both CTAs of the pair: 0b11). A second, separate commit per
// k-block costs about 10% of tensor throughput; this form does not.
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar), "h"((uint16_t)0x3)
               : "memory");
}
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- stream-K partial accumulators (pair kernel) ----
// A slot holds one tile's fp32 partial: per CTA of the pair and epilogue
// warp, that warp's kChunks chunks of 32 rows x 32 columns, each chunk as 8
// column groups of [32 lanes] float4 (so one store instruction of the warp
// covers 512 contiguous bytes).
template <int BN, int EPI_WARPS>
struct SkLayout {
  static constexpr int kGroups = EPI_WARPS / 4;
  static constexpr int kChunks = BN / 32 / kGroups;
  static constexpr int kWarpFloats = kChunks * 32 * 32;
  static constexpr int kSlotFloats = 2 * EPI_WARPS * kWarpFloats;
  static constexpr int kSlotFlags = 2 * EPI_WARPS;
};
// The i-th of the 32-column TMEM chunks that the epilogue warps of column
// group `group` read: a contiguous run of chunks, or (HALVES) half a run in
// each half of the tile, as EpiSwiGLU reads g and the u columns BN/2 further.
// A warp completes exactly these chunks of a stream-K tile, so its epilogue
// reads nothing another warp is still adding to.
template <int BN, int EPI_WARPS, bool HALVES>
__device__ __forceinline__ int sk_chunk(int group, int i) {
  using SL = SkLayout<BN, EPI_WARPS>;
  if constexpr (!HALVES) {
    return group * SL::kChunks + i;
  } else {
    constexpr int h = SL::kChunks / 2;
    return i < h ? group * h + i : BN / 64 + group * h + (i - h);
  }
}

// An earlier k part of a stream-K tile: this warp's columns of the
// accumulator go to the cluster's slot, then the warp's ready flag is set.
template <int BN, int EPI_WARPS, bool HALVES>
__device__ __forceinline__ void sk_put(const Sched& s, int slot, uint32_t rank, int e, int group,
                                       int lane, uint32_t taddr) {
  using SL = SkLayout<BN, EPI_WARPS>;
  const int wi = static_cast<int>(rank) * EPI_WARPS + e;
  float4* dst = reinterpret_cast<float4*>(s.sk_part + static_cast<size_t>(slot) * SL::kSlotFloats +
                                          static_cast<size_t>(wi) * SL::kWarpFloats);
#pragma unroll 1
  for (int c = 0; c < SL::kChunks; ++c) {
    float v[32];
    tmem_ld32(taddr + sk_chunk<BN, EPI_WARPS, HALVES>(group, c) * 32, v);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcg(dst + (c * 8 + j) * 32 + lane, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) st_release_gpu(s.sk_flag + slot * SL::kSlotFlags + wi, 1);
}

// The last k part of a stream-K tile: wait (bounded) for the partials of
// the tile's earlier parts, slots [w.fix_lo, w.fix_hi), add them to this
// warp's columns of the accumulator in that order (a fixed order: results
// do not vary from run to run) and clear their flags. false: the wait ran
// out or the CTA is aborting.
template <int BN, int EPI_WARPS, bool HALVES>
__device__ __forceinline__ bool sk_fix(const Sched& s, const Unit& w, uint32_t rank, int e, int group,
                                       int lane, uint32_t taddr, volatile int* abort_flag, int* err,
                                       uint64_t limit_ns) {
  using SL = SkLayout<BN, EPI_WARPS>;
  const int wi = static_cast<int>(rank) * EPI_WARPS + e;
  bool ok = true;
  if (lane == 0) {
    for (int slot = w.fix_lo; slot < w.fix_hi && ok; ++slot) {
      const int* f = s.sk_flag + slot * SL::kSlotFlags + wi;
      if (ld_acquire_gpu(f) != 0) continue;
      const uint64_t t0 = globaltimer();
      while (ld_acquire_gpu(f) == 0) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        if (globaltimer() - t0 > limit_ns) {
          *abort_flag = 1;
          atomicCAS(err, 0, kErrWaitPartial);
          ok = false;
          break;
        }
      }
    }
  }
  // lane 0 acquired every flag; the warp barrier orders the other lanes'
  // loads below after those acquires
  __syncwarp();
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (!ok) return false;
  // (chunk, slot) pairs in order; the next pair's loads are issued as soon as
  // the current one is added, so they overlap the TMEM store and load
  const int ns = w.fix_hi - w.fix_lo;
  const int npairs = SL::kChunks * ns;
  const float* part = s.sk_part + static_cast<size_t>(wi) * SL::kWarpFloats;
  auto load = [&](int p, float4 (&r)[8]) {
    const int c = p / ns;
    const float4* src = reinterpret_cast<const float4*>(
        part + static_cast<size_t>(w.fix_lo + (p - c * ns)) * SL::kSlotFloats);
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __ldcg(src + (c * 8 + j) * 32 + lane);
  };
  float4 cur[8];
  load(0, cur);
  float v[32];
#pragma unroll 1
  for (int p = 0; p < npairs; ++p) {
    const int c = p / ns, si = p - c * ns;
    const uint32_t ta = taddr + sk_chunk<BN, EPI_WARPS, HALVES>(group, c) * 32;
    if (si == 0) tmem_ld32(ta, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[4 * j] += cur[j].x;
      v[4 * j + 1] += cur[j].y;
      v[4 * j + 2] += cur[j].z;
      v[4 * j + 3] += cur[j].w;
    }
    if (p + 1 < npairs) load(p + 1, cur);  // in flight during this chunk's store and the next load
    if (si == ns - 1) tmem_st32(ta, v);
  }
  __syncwarp();
  if (lane == 0)
    for (int slot = w.fix_lo; slot < w.fix_hi; ++slot) s.sk_flag[slot * SL::kSlotFlags + wi] = 0;
  return true;
}

// Sched for this kernel counts m tiles of 2 x BM rows; the grid is
// 2 x (number of clusters) with cluster dimension (2, 1, 1). With
// sched.sk_tiles > 0 the tail tiles run as stream-K parts (see Sched).
template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS>
__global__ void __launch_bounds__(gemm_threads(EPI_WARPS), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_a2,
                     const __grid_constant__ CUtensorMap tma_b2,
                     const __grid_constant__ CUtensorMap tma_c, Sched sched,
                     typename Epi::Params ep, int* err) {
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "4 or 8 epilogue warps");
  static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
  if (sched.gate) {  // grid-uniform; the flag comes from an earlier kernel
    pdl_wait();
    if (*sched.gate == 0) return;
  }
  constexpr int BNH = BN / 2;  // B rows held by each CTA
  using L = SmemLayout<BNH, STAGES, EPI_WARPS>;
  constexpr int kTmemCols = (2 * BN <= 256) ? 256 : 512;
  constexpr uint32_t kIdesc = idesc_bf16(BN, A_MN, B_MN, 2 * BM);
  constexpr uint32_t kPairBytes = 2u * L::kStageBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBarOff;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cluster = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (sched.kb2 > 0) {
      tma_prefetch_desc(&tma_a2);
      tma_prefetch_desc(&tma_b2);
    }
  }
  if (warp == 1) {
    // both CTAs' warp 1 take part; the address lands at the same offset in each
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int n_my = sched.cluster_units(cluster, n_clusters);
  const uint64_t wait_ns = sched.limit();
  const uint32_t idesc = sched.idesc(kIdesc);
  // Launched with programmatic dependent launch: the prologue above (barriers,
  // TMEM, descriptor prefetch) may overlap the previous kernel; no thread
  // touches global memory before this wait.
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer ----
      uint32_t it = 0;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const Unit w = sched_unit(sched, cluster, n_clusters, i);
        const int a_row = w.mt * 2 * BM + static_cast<int>(rank) * BM;
        const int b_row = w.nt * BN + static_cast<int>(rank) * BNH;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!bounded_wait(empty_bar(s), ph ^ 1u, abort_flag, err, kErrWaitProducer, wait_ns)) {
            ok = false;
            break;
          }
          if (static_cast<int>(it) == sched.withhold) continue;  // diagnostic launch only
          const uint32_t a_dst = sbase + s * L::kStageBytes;
          const uint32_t b_dst = a_dst + L::kABytes;
          const uint32_t fb = cluster_addr(full_bar(s), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(s), kPairBytes);
          const int k0 = sched.k_elem(kb);
          const bool seg2 = sched.second(kb);
          const CUtensorMap* ma = seg2 ? &tma_a2 : &tma_a;
          const CUtensorMap* mb = seg2 ? &tma_b2 : &tma_b;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d_pair(a_dst + j * 8192, ma, fb, a_row + j * 64, k0);
          } else {
            tma_load_2d_pair(a_dst, ma, fb, k0, a_row);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BNH / 64; ++j)
              tma_load_2d_pair(b_dst + j * 8192, mb, fb, b_row + j * 64, k0);
          } else {
            tma_load_2d_pair(b_dst, mb, fb, k0, b_row);
          }
        }
      }
      if (!ok && rank == 0) {
        // both CTAs' copies complete on rank 0's full barriers: wait for the
        // last min(it, STAGES) stages (bounded) before leaving
        int n = it < (uint32_t)STAGES ? (int)it : STAGES;
        for (int i = 1; i <= n; ++i) {
          uint32_t j = it - i;
          uint32_t bar = full_bar(j % STAGES), ph = (j / STAGES) & 1u;
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(bar, ph) && globaltimer() - t0 < wait_ns) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ----------------------------------------- MMA issuer (rank 0) ----
      uint32_t it = 0, lt = 0;
      bool ok = true;
      bool issued = false;
      for (int i = 0; i < n_my && ok; ++i, ++lt) {
        const Unit w = sched_unit(sched, cluster, n_clusters, i);
        const int kb0 = w.kb0, kb1 = w.kb1;
        const uint32_t acc = lt & 1u;
        const uint32_t acc_ph = (lt >> 1) & 1u;
        if (!bounded_wait<true>(tempty_bar(acc), acc_ph ^ 1u, abort_flag, err, kErrWaitMma, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!bounded_wait<true>(full_bar(s), ph, abort_flag, err, kErrWaitMma, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + s * L::kStageBytes;
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if (A_MN) ad = smem_desc_sw128(a_addr + k * 2048, 8192, 1024);
            else ad = smem_desc_sw128(a_addr + k * 32, 16, 1024);
            if (B_MN) bd = smem_desc_sw128(b_addr + k * 2048, 8192, 1024);
            else bd = smem_desc_sw128(b_addr + k * 32, 16, 1024);
            tc_mma_bf16_pair(tmem_d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          // stage s of both CTAs is free once these MMAs finish
          tc_commit_pair_both(empty_bar(s));
        }
        if (!ok) break;
        tc_commit_pair_both(tfull_bar(acc));
      }
      if (!ok && issued) {
        tc_commit_pair(cluster_addr(drain_bar, 0));
        uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain_bar, 0) && globaltimer() - t0 < wait_ns) {
        }
      }
    }
  } else {
    // ------------------------------------------------------ epilogue ----
    const int quarter = warp & 3;
    const int e = warp - 2;
    constexpr int kGroups = EPI_WARPS / 4;
    const int group = e >> 2;
    uint8_t* stage = smem + L::kEpiOff + e * kEpiWarpBytes;
    typename EpiCarry<Epi>::type carry{};
    uint32_t lt = 0;
    constexpr bool kHalves = EpiHalves<Epi>::value;
    for (int i = 0; i < n_my; ++i, ++lt) {
      const Unit w = sched_unit(sched, cluster, n_clusters, i);
      const int mt = w.mt, nt = w.nt, ks = w.ks;
      const int row_base = mt * 2 * BM + static_cast<int>(rank) * BM;
      if constexpr (EpiCarry<Epi>::kHas)
        if (w.role != kRolePart) Epi::prefetch(ep, row_base, nt, quarter, lane, group, kGroups, carry);
      const uint32_t acc = lt & 1u;
      const uint32_t acc_ph = (lt >> 1) & 1u;
      bool ok = true;
      if (lane == 0) ok = bounded_wait(tfull_bar(acc), acc_ph, abort_flag, err, kErrWaitEpilogue, wait_ns);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (w.role == kRolePart) {
        // an earlier k part of a stream-K tile: the partial goes to this
        // cluster's slot; the tile's finishing cluster runs the epilogue
        sk_put<BN, EPI_WARPS, kHalves>(sched, cluster, rank, e, group, lane, taddr);
      } else {
        if (w.role == kRoleFinish &&
            !sk_fix<BN, EPI_WARPS, kHalves>(sched, w, rank, e, group, lane, taddr, abort_flag, err, wait_ns))
          break;
        // the epilogue reads only the TMEM columns this warp has just completed
        if constexpr (EpiCarry<Epi>::kHas)
          Epi::tile(ep, &tma_c, row_base, nt, ks, quarter, lane, taddr, stage, group, kGroups, carry);
        else
          Epi::tile(ep, &tma_c, row_base, nt, ks, quarter, lane, taddr, stage, group, kGroups);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(tempty_bar(acc), 0));
    }
    if (lane == 0) bulk_wait_all();  // this warp's TMA stores, if any, are complete
  }

  // the next kernel of the stream (if launched with programmatic dependent
  // launch) may start its own prologue during this teardown; it still waits
  // for this grid's completion before it reads what this grid wrote
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc
}  // namespace soup
