// Prefill path (M >= 128 tokens): fused Block-RVQ decode -> shared memory ->
// tcgen05.mma on pairs of SMs (cta_group::2, fp32 accumulators in TMEM).
//
// Two CTAs of a cluster compute a 256 (output rows) x 512, 384 or 256 (tokens) tile of y
// over all of K in stages of 64 columns.  Each CTA decodes its own 128 weight
// rows exactly (the same arithmetic as the decode GEMV: fp32 stage sum, two
// roundings in the weight type) into a 128-byte-swizzled K-major buffer and
// fetches, by TMA (no multicast), its 128-token halves of the two activation
// tiles; the leader's elected thread issues 256 x 256 x 16 pair MMAs that read
// both CTAs' buffers and accumulate each CTA's 128 rows x 512 tokens in its own
// TMEM.  Roles per CTA (576 threads): warp 0 TMA producer, warp 1 MMA issuer
// (leader) or decode forwarder (peer), warps 2-17 decoders and then the
// epilogue (TMEM -> registers -> bias -> bf16/fp16/fp32 stores of y).
//
// Why pairs: a single-CTA 128 x 128 x 16 MMA reads 8 KB of operands from
// shared memory per 64 tensor cycles, the whole port of the SM, and the
// activation fills and the decoders share that port; the single-CTA kernel
// (512 tokens x 128 rows per CTA, four accumulators, two stages) spent 1730
// cycles per 1024-cycle stage and ran the Llama-3-8B projections at 908
// TFLOP/s.  Split over a pair, each SM reads half the operand bytes and
// fetches half the activations per MMA cycle: 1470 cycles per stage, gate/up
// 917 -> 1070 TFLOP/s, the 128-GEMM 8B prefill 908 -> 987 TFLOP/s.  Measured
// before the pair kernel: a 256 x 256 single-CTA tile ran at 797 TFLOP/s and a
// persistent stream-K schedule of the 512 x 128 tile at 810-830 (its
// per-segment epilogues and refills cost more than the tail wave it removes).
// The dense weight never reaches global memory.  Every mbarrier wait is
// bounded by a %globaltimer deadline; on expiry the CTA records an error code
// (if a status word was supplied), stops issuing work, drains and frees TMEM.
// Replaces reference src/runtime.py:1501-1507 for large M (reconstruct_weight
// + F.linear, i.e. the whole weight materialised per call).
#include "../../include/wal_rvq.h"
#include "wal_rvq_decode.cuh"

#include <cuda.h>
#include <cstdint>

namespace wal {
namespace gemm {

constexpr int kBK = 64;
constexpr int kDecodeWarps = 16;
constexpr int kRowParts = kDecodeWarps * 32 / 128;  // decoder threads per weight row
constexpr int kPartBlocks = 8 / kRowParts;          // d = 8 blocks per thread per 64-column stage
constexpr int kThreads = (2 + kDecodeWarps) * 32;
constexpr int kCbCopyBytes = 256 * 16;  // one stage table, one copy
constexpr int kCbCopies = 8;            // 8-lane phases of 16-byte gathers hit 8 distinct bank quads
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s per wait, then give up

struct GemmParams {
  const uint8_t* packed;
  const uint16_t* codebooks;
  const float* stage_scales;  // fp32 [groups][R] (fast mode, or one stage) or null
  const uint16_t* row_scale;
  const uint16_t* bias;
  void* y;
  int* status;  // optional device word: nonzero after a timed-out wait
  long long ldy;
  int M, N, K;
  int chunks;   // 16-block chunks per packed tile row
  int entries;
  int y_dtype;
  int num_groups;
  int group_tile_start[65];
  int group_row_start[65];
  int tok;  // tokens per pair tile: 512, 384 or 256 (two accumulators of tok / 2)
  int vec_out;  // y and its row stride allow 16-byte stores
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed, false when the deadline passed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);           // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)((1024 >> 4) & 0x3FFF) << 32;     // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                          // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One statement for the load and its wait: the destination registers are
// outputs of the wait too, so no use of them is scheduled between the two.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// ---- pair (cta_group::2) primitives -------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// every thread of both CTAs of the pair
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// the shared::cluster address of the same shared-memory offset in CTA `rank` of the pair
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a barrier that the other CTA of the pair (or its tensor
// cores) arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}

// Activation box into this CTA's shared memory; the completed bytes count on
// the barrier at `bar_cluster` (the leader CTA's), so one barrier covers the
// boxes of both CTAs.  No multicast: each CTA fetches its own tokens.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

// Pair MMA: D[256 x N] (+)= A[256 x 16] B[N x 16]^T, A rows 0-127 and B rows
// 0..N/2-1 from the leader's shared memory, the rest from the peer's, D rows
// 0-127 in the leader's TMEM and 128-255 in the peer's (same columns).
template <bool F16>
__host__ __device__ constexpr uint32_t idesc_pair(int n) {
  return (1u << 4) | (F16 ? 0u : (1u << 7) | (1u << 10)) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

template <bool F16>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// arrive on the barrier at this offset in both CTAs once the pair MMAs issued
// so far have completed
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}

// Decode the weights of one output row for blocks u0 .. u0 + kPartBlocks - 1
// of a 64-column stage (d = 8) and store them, 16 bytes per block, into the
// swizzled B buffer.  ids[st] holds the 1-byte ids of those blocks.  Tables
// of one stage and of the fast mode already hold weight-type values.
template <int R, int NUM>
__device__ __forceinline__ void decode_stage_part(uint32_t bsm_row, int nsw, const uint32_t (&ids)[R], int u0,
                                                  uint32_t cb_lane, uint32_t rho2, int k_left) {
  using T = WT<(NUM & 4) != 0>;
  constexpr bool kTyped = R == 1 || (NUM & 3) == kFast;
#pragma unroll
  for (int j = 0; j < kPartBlocks; ++j) {
    const int u = u0 + j;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (u * 8 < k_left) {
      float s[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] = 0.f;
      uint32_t w[4];
#pragma unroll
      for (int st = 0; st < R; ++st) {
        const uint32_t id = (ids[st] >> (8 * j)) & 0xFFu;
        uint4 c;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(c.x), "=r"(c.y), "=r"(c.z), "=r"(c.w)
                     : "r"(cb_lane + (uint32_t)(st * 256 + id) * (kCbCopies * 16)));
        if (kTyped) {
          if (st == 0) {
            w[0] = c.x; w[1] = c.y; w[2] = c.z; w[3] = c.w;
          } else {
            w[0] = T::add2(w[0], c.x);
            w[1] = T::add2(w[1], c.y);
            w[2] = T::add2(w[2], c.z);
            w[3] = T::add2(w[3], c.w);
          }
        } else {
          add2_f32_f16x2(s[0], s[1], c.x);
          add2_f32_f16x2(s[2], s[3], c.y);
          add2_f32_f16x2(s[4], s[5], c.z);
          add2_f32_f16x2(s[6], s[7], c.w);
        }
      }
      if (!kTyped) {
        w[0] = T::cvt2(s[0], s[1]);
        w[1] = T::cvt2(s[2], s[3]);
        w[2] = T::cvt2(s[4], s[5]);
        w[3] = T::cvt2(s[6], s[7]);
      }
      o.x = T::mul2(w[0], rho2);
      o.y = T::mul2(w[1], rho2);
      o.z = T::mul2(w[2], rho2);
      o.w = T::mul2(w[3], rho2);
    }
    const uint32_t addr = bsm_row + ((u ^ nsw) << 4);
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(o.x), "r"(o.y), "r"(o.z), "r"(o.w)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Pair kernel (cta_group::2): two CTAs of a cluster on neighbouring SMs compute
// a 256 (output rows) x 512 (tokens) tile of y^T as 256 x 256 x 16 pair MMAs:
// each CTA decodes its own 128 weight rows (the MMA A operand, M = 256 over the
// pair) and fetches its 128-token halves of the activations (the B operand,
// N = 256 per accumulator over the pair); the leader CTA's elected thread
// issues the MMAs, which read both CTAs' shared memory and write each CTA's
// 128 rows x 512 tokens of fp32 accumulators into its own TMEM.  Per SM and
// stage the tensor cores read 64 KB of operands instead of the 128 KB of the
// single-CTA 128 x 128 MMAs, and the activation fetch halves, so the shared
// memory port (which the operand reads, the TMA fills and the decoders share)
// no longer caps the tensor pipe near half of its rate.
//   warp 0      (both CTAs) TMA producer: this CTA's 128 tokens of each
//               accumulator per 64-column stage; bytes of both CTAs count on
//               the leader's full_x[stage];
//   warp 1      (leader) MMA issuer: waits full_x + full_w, 4 x nacc pair
//               MMAs per stage, commits to empty[stage] of both CTAs;
//   warps 2-17  (both CTAs) decoders, as in the single-CTA kernel, arriving on
//               their CTA's full_w[stage] (the peer's warp 1 forwards each
//               completed stage to the leader's); then the epilogue: each thread
//               reads one output row's tokens from TMEM, the four warps of a
//               column share pass 16-token blocks through the idle stage ring
//               and store 16-byte pieces of the output rows (scalar stores
//               when y or its stride is not 16-byte aligned).
namespace pair {
constexpr int kRows = 128;                  // weight rows per CTA
constexpr int kAccN = 256;                  // TMEM columns per accumulator (MMA N at most)
constexpr int kHalf = 128;                  // tokens of one accumulator held by one CTA (at most)
constexpr int kStages = 3;
constexpr int kXBytes = 2 * kHalf * kBK * 2;  // 32 KB: this CTA's halves of both accumulators
constexpr int kWBytes = kRows * kBK * 2;      // 16 KB: decoded weights
constexpr int kPairTmemCols = 2 * kAccN;

int smem_bytes(int R) {
  return 1024 + kStages * (kXBytes + kWBytes) + R * kCbCopyBytes * kCbCopies + 8 * (3 * kStages + 1) + 16;
}
}  // namespace pair

template <int R, int NUM>
__global__ void __launch_bounds__(kThreads, 1) rvq_gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                    const __grid_constant__ GemmParams p) {
  using namespace pair;
  constexpr int S = pair::kStages;
  constexpr int NM = NUM & 3;
  constexpr bool F16 = (NUM & 4) != 0;
  using T = WT<F16>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned: [x stages][w stages][codebooks][barriers][tmem slot]
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t x_sm = base;
  const uint32_t w_sm = x_sm + S * kXBytes;
  const uint32_t cb_sm = w_sm + S * kWBytes;
  uint8_t* cb = gbase + (cb_sm - base);
  const uint32_t bar_sm = cb_sm + R * kCbCopyBytes * kCbCopies;
  const uint32_t full_w = bar_sm, full_x = bar_sm + 8 * S, empty = bar_sm + 16 * S;
  const uint32_t acc_full = bar_sm + 24 * S;
  const uint32_t tmem_slot = acc_full + 8;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));
  __shared__ volatile int abort_flag;

  const uint32_t rank = cluster_ctarank();  // 0: leader
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid x = (pair rank, token tile), y = pair of 128-row tiles: the pair runs
  // along x (a kernel with pair MMAs needs an even cluster width), and the
  // token tiles of one pair of row tiles run side by side, so the weight ids
  // stream from HBM once and the other tiles find them in L2
  const int n0 = (2 * (int)blockIdx.y + (int)rank) * kRows;  // this CTA's weight rows (maybe a padding CTA)
  const int tok = p.tok, accn = tok / 2, half = tok / 4;  // tile tokens, MMA N, tokens per CTA and accumulator
  const int m0 = (int)(blockIdx.x >> 1) * tok;
  const int nacc = p.M - m0 > accn ? 2 : 1;  // accumulators holding tokens (the same in both CTAs)
  const int kblocks = (p.K + kBK - 1) / kBK;

  int g = 0;
  while (g + 1 < p.num_groups && p.group_row_start[g + 1] <= n0) ++g;
  const int g_row0 = p.group_row_start[g], g_row1 = p.group_row_start[g + 1];
  const int g_tile0 = p.group_tile_start[g];

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      // leader: its decoder warps + the peer's forwarded arrival; peer: its decoder warps
      mbar_init(full_w + 8 * s, kDecodeWarps + (rank == 0 ? 1 : 0));
      mbar_init(full_x + 8 * s, 1);                 // the leader's expect_tx (used in the leader)
      mbar_init(empty + 8 * s, 1);                  // the pair commit (both CTAs)
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // both CTAs, same warp: one allocation for the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(kPairTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers and TMEM exist before any remote arrive or pair MMA
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  const uint32_t lead_full_w = mapa_shared(full_w, 0), lead_full_x = mapa_shared(full_x, 0);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ---------------------------
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % S;
        if (kb >= S && !mbar_wait_cluster(empty + 8 * s, ((kb / S) - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        if (abort_flag) break;
        if (rank == 0) mbar_expect_tx(full_x + 8 * s, 2 * nacc * (half * 128));
        for (int a = 0; a < nacc; ++a)
          tma_load_2d_pair(x_sm + s * kXBytes + a * (kHalf * 128), &xmap, kb * kBK, m0 + a * accn + (int)rank * half,
                           lead_full_x + 8 * s);
        ++issued;
      }
      // the leader sees both CTAs' loads land: never leave one in flight
      if (rank == 0)
        for (int kb = issued - S < 0 ? 0 : issued - S; kb < issued; ++kb)
          if (!mbar_wait(full_x + 8 * (kb % S), (kb / S) & 1)) abort_flag = 1;
    }
  } else if (warp == 1 && rank == 1) {
    // ---------------- peer: forward its decoded stages to the leader -------
    // The decoders arrive on their own CTA's barrier (a CTA-scope release);
    // this thread, with no loads of its own in flight, turns each completed
    // phase into one cluster-scope arrive on the leader's barrier.  (Decoders
    // arriving remotely themselves made every release wait for their id
    // prefetches from HBM: twice the decode time per stage.)
    if (lane == 0) {
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(full_w + 8 * s, (kb / S) & 1)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_cluster(lead_full_w + 8 * s);
      }
    }
  } else if (warp == 1) {
    // ---------------- pair MMA issuer (leader) ---------------------------
    if (lane == 0) {
      const uint32_t idesc = idesc_pair<F16>(accn);
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % S;
        const uint32_t par = (kb / S) & 1;
        if (!mbar_wait_cluster(full_x + 8 * s, par) || !mbar_wait_cluster(full_w + 8 * s, par)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t ad = smem_desc_sw128(w_sm + s * kWBytes + ks * 32);
          for (int a = 0; a < nacc; ++a) {
            const uint64_t bd = smem_desc_sw128(x_sm + s * kXBytes + a * (kHalf * 128) + ks * 32);
            umma_pair<F16>(tmem + (uint32_t)(a * kAccN), ad, bd, idesc, (kb > 0 || ks > 0) ? 1u : 0u);
          }
        }
        umma_commit_pair(empty + 8 * s);
      }
      umma_commit_pair(acc_full);  // both CTAs: every pair MMA issued above has completed
    }
  } else {
    // ---------------- decoders (both CTAs), then epilogue -----------------
    const int t = threadIdx.x - 64;
    const int row = t & (kRows - 1), part = t >> 7;
    const int n = n0 + row;
    const bool row_ok = n < g_row1;
    const uint32_t rho2 = row_ok ? T::rho2(p.row_scale[n]) : 0u;
    const int local = n - g_row0;
    const long long tile = (long long)g_tile0 + local / 16;
    const int rr = local % 16;
    const long long tile_bytes = (long long)p.chunks * R * 256;
    const uint8_t* idrow = p.packed + tile * tile_bytes + rr * 16 + part * kPartBlocks;
    const uint32_t wsm_row0 = w_sm + (row >> 3) * 1024 + (row & 7) * 128;
    const uint32_t cb_lane = cb_sm + (uint32_t)(lane & 7) * 16;
    const int nsw = row & 7;
    constexpr int kIdAhead = 4;
    auto load_ids = [&](int kb, uint32_t (&dst)[R]) {
#pragma unroll
      for (int st = 0; st < R; ++st) {
        const uint8_t* a = idrow + ((long long)(kb >> 1) * R + st) * 256 + 8 * (kb & 1);
        dst[st] = !(row_ok && kb < kblocks) ? 0u
                  : kPartBlocks == 4        ? __ldcs(reinterpret_cast<const unsigned int*>(a))
                                            : (uint32_t)__ldcs(reinterpret_cast<const unsigned short*>(a));
      }
    };
    uint32_t idq[kIdAhead + 1][R];
#pragma unroll
    for (int j = 0; j < kIdAhead; ++j) load_ids(j, idq[j]);
    // codebooks of this CTA's group, 8 copies per entry, staged by the decoder
    // warps while the first activation boxes are in flight (the producer
    // starts right after the cluster barrier); every load of a thread goes
    // out before its first store (one L2 round trip, not one per entry), and
    // lanes write the copies of one entry side by side (whole 128-byte rows,
    // no bank conflicts)
    {
      const uint16_t* books = p.codebooks + (size_t)g * R * p.entries * 8;
      const float* scales = p.stage_scales ? p.stage_scales + (size_t)g * R : nullptr;
      constexpr int kItems = R * 256 * kCbCopies / (kDecodeWarps * 32);
      const int total = R * p.entries * kCbCopies;
      uint4 v[kItems];
#pragma unroll
      for (int q = 0; q < kItems; ++q) {
        const int i = t + q * kDecodeWarps * 32;
        if (i < total) v[q] = *reinterpret_cast<const uint4*>(books + (size_t)(i / kCbCopies) * 8);
      }
#pragma unroll
      for (int q = 0; q < kItems; ++q) {
        const int i = t + q * kDecodeWarps * 32;
        if (i >= total) break;
        const int c = i % kCbCopies, se = i / kCbCopies;
        const int st = se / p.entries, e = se - st * p.entries;
        v[q].x = staged_word<R, NM, F16>(v[q].x, scales, st);
        v[q].y = staged_word<R, NM, F16>(v[q].y, scales, st);
        v[q].z = staged_word<R, NM, F16>(v[q].z, scales, st);
        v[q].w = staged_word<R, NM, F16>(v[q].w, scales, st);
        *reinterpret_cast<uint4*>(cb + ((st * 256 + e) * kCbCopies + c) * 16) = v[q];
      }
      // the decoder warps only (no bounded wait precedes it, so all arrive)
      asm volatile("bar.sync 5, %0;" ::"r"(kDecodeWarps * 32) : "memory");
    }
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % S;
      load_ids(kb + kIdAhead, idq[kIdAhead]);
      if (kb >= S && !mbar_wait_cluster(empty + 8 * s, ((kb / S) - 1) & 1)) {
        abort_flag = 1;
        break;
      }
      if (abort_flag) break;
      const int k_left = row_ok ? p.K - kb * kBK : 0;
      decode_stage_part<R, NUM>(wsm_row0 + s * kWBytes, nsw, idq[0], part * kPartBlocks, cb_lane, rho2, k_left);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(full_w + 8 * s);
#pragma unroll
      for (int j = 0; j < kIdAhead; ++j)
#pragma unroll
        for (int st = 0; st < R; ++st) idq[j][st] = idq[j + 1][st];
    }
    // epilogue: TMEM lane 32 * (warp % 4) + lane is output row n0 + that lane;
    // column a * 256 + c of accumulator a is token m0 + a * accn + c; the four
    // warps of a lane quarter split each accumulator's columns
    bool ok = !abort_flag && mbar_wait_cluster(acc_full, 0);
    ok = __all_sync(0xffffffffu, ok);  // TMEM loads are warp-wide
    if (!ok) abort_flag = 1;
    tc_fence_after();
    const int quarter = warp & 3, share = (warp - 2) >> 2;
    const int erow = quarter * 32 + lane;
    const int en = n0 + erow;
    const bool eok = en < g_row1;
    const float bias = (eok && p.bias) ? __bfloat162float(__ushort_as_bfloat16(p.bias[en])) : 0.f;
    const int cols = accn / 4;  // per warp and accumulator: 64, 48 or 32
    if (p.vec_out) {
      // The four warps of one column share (one per lane quarter, 128 rows)
      // pass each 16-token block through shared memory (the stage ring is
      // idle once the accumulators are complete) and store whole 16-byte
      // pieces of the output rows: a warp store writes two tokens' 256 or 512
      // contiguous bytes instead of 64 or 128 bytes of one token.  Two staging
      // buffers per share, so one named barrier per block orders both the
      // writes before the reads and the reads before the next reuse.
      const int esz = p.y_dtype == WAL_F32 ? 4 : 2;
      const int chunks = 8 * esz;  // 16-byte pieces per token row of 128 outputs
      uint8_t* stage = gbase + (x_sm - base) + share * 16384;
      for (int c = 0, b = 0; c < nacc * cols; c += 16, b ^= 1) {
        const int a = c / cols, c0 = share * cols + (c - a * cols);  // accumulator, its column
        uint32_t v[16];
        if (ok) tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * kAccN + c0), v);
        uint8_t* buf = stage + b * 8192;
        if (esz == 4) {
#pragma unroll
          for (int j = 0; j < 16; ++j) reinterpret_cast<float*>(buf)[j * 128 + erow] = __uint_as_float(v[j]) + bias;
        } else {
          const bool fp16 = p.y_dtype == WAL_F16;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float f = __uint_as_float(v[j]) + bias;
            reinterpret_cast<uint16_t*>(buf)[j * 128 + erow] =
                fp16 ? __half_as_ushort(__float2half_rn(f)) : __bfloat16_as_ushort(__float2bfloat16_rn(f));
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + share) : "memory");
        if (ok) {
          const int t0 = m0 + a * accn + c0;  // token of row 0 of this block
          for (int k = erow; k < 16 * chunks; k += 128) {
            const int j = k / chunks, r0 = (k - j * chunks) * (16 / esz);
            const int m = t0 + j;
            if (m >= p.M) continue;
            const uint4 w = *reinterpret_cast<const uint4*>(buf + (size_t)k * 16);
            uint8_t* dst = static_cast<uint8_t*>(p.y) + ((long long)m * p.ldy + n0 + r0) * esz;
            if (n0 + r0 + 16 / esz <= g_row1) {
              *reinterpret_cast<uint4*>(dst) = w;
            } else {  // the last rows of the layer
              const uint8_t* src = reinterpret_cast<const uint8_t*>(&w);
              for (int e = 0; e < 16 / esz && n0 + r0 + e < g_row1; ++e)
                for (int q = 0; q < esz; ++q) dst[e * esz + q] = src[e * esz + q];
            }
          }
        }
      }
    } else if (ok) {
      for (int c = 0; c < nacc * cols; c += 16) {
        const int a = c / cols, c0 = share * cols + (c - a * cols);  // accumulator, its column
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * kAccN + c0), v);
        if (!eok) continue;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + a * accn + c0 + j;
          if (m >= p.M) break;
          const float f = __uint_as_float(v[j]) + bias;
          const long long idx = (long long)m * p.ldy + en;
          if (p.y_dtype == WAL_F32) static_cast<float*>(p.y)[idx] = f;
          else if (p.y_dtype == WAL_F16) static_cast<uint16_t*>(p.y)[idx] = __half_as_ushort(__float2half_rn(f));
          else static_cast<uint16_t*>(p.y)[idx] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM or exits while the pair still works on it
  if (abort_flag && threadIdx.x == 0 && p.status) atomicExch(p.status, 1);
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPairTmemCols) : "memory");
  }
}


typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace gemm
}  // namespace wal

using namespace wal;
using namespace wal::gemm;

template <int R, int NUM>
static int launch_gemm_pair(const CUtensorMap& map, const GemmParams& p, dim3 grid, int smem, cudaStream_t s) {
  auto kern = rvq_gemm_pair_kernel<R, NUM>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;  // the CTA pair: neighbouring 128-row tiles
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, map, p) != cudaSuccess) return WAL_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

extern "C" int wal_rvq_gemm_typed(const wal_rvq_layer* layer, const void* x, int x_dtype, int64_t M, int64_t ldx,
                                  void* y, int64_t ldy, int y_dtype, int* status, void* stream) {
  if (!layer || !x || !y) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = layer->geom;
  if (M <= 0 || g.out_features <= 0 || g.in_features <= 0 || layer->num_tiles <= 0) return WAL_ERR_SHAPE;
  if (x_dtype != WAL_BF16 && x_dtype != WAL_F16) return WAL_ERR_UNSUPPORTED;  // fp32: the GEMV path
  if (layer->sum_mode != WAL_SUM_EXACT && layer->sum_mode != WAL_SUM_FAST) return WAL_ERR_INVALID_ARGUMENT;
  const bool fast = layer->sum_mode == WAL_SUM_FAST, f16 = x_dtype == WAL_F16;
  if (g.block_size != 8 || g.num_stages < 1 || g.num_stages > 2 || g.num_entries > 256) return WAL_ERR_UNSUPPORTED;
  if (g.num_groups < 1 || g.num_groups > 64) return WAL_ERR_UNSUPPORTED;
  if (!layer->packed_ids || !layer->codebooks || !layer->row_scale) return WAL_ERR_INVALID_ARGUMENT;
  // exact multi-stage sums with fp32 stage scales: the GEMV path handles them
  if (layer->stage_scales && g.num_stages > 1 && !fast) return WAL_ERR_UNSUPPORTED;
  if (ldx < g.in_features || ldy < g.out_features) return WAL_ERR_SHAPE;
  if ((ldx % 8) || ((uintptr_t)x & 15) || ((uintptr_t)layer->codebooks & 15) || ((uintptr_t)layer->packed_ids & 15))
    return WAL_ERR_ALIGNMENT;
  if (y_dtype != WAL_BF16 && y_dtype != WAL_F32 && y_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  if (M > (int64_t)1 << 30 || g.in_features > (1 << 30)) return WAL_ERR_SHAPE;
  GemmParams p{};
  p.packed = static_cast<const uint8_t*>(layer->packed_ids);
  p.codebooks = layer->codebooks;
  p.stage_scales = layer->stage_scales;
  p.row_scale = layer->row_scale;
  p.bias = layer->bias;
  p.y = y;
  p.status = status;
  p.ldy = ldy;
  p.M = (int)M;
  p.N = (int)g.out_features;
  p.K = (int)g.in_features;
  const long long blocks = (g.in_features + 7) / 8;
  p.chunks = (int)((blocks + 15) / 16);
  p.entries = g.num_entries;
  p.y_dtype = y_dtype;
  {
    const long long esz = y_dtype == WAL_F32 ? 4 : 2;
    p.vec_out = ((uintptr_t)y % 16 == 0 && (ldy * esz) % 16 == 0) ? 1 : 0;
  }
  p.num_groups = g.num_groups;
  // group boundaries; a CTA's 128 weight rows must not straddle two groups
  long long t = 0, rows = 0;
  p.group_tile_start[0] = 0;
  p.group_row_start[0] = 0;
  for (int i = 0; i < g.num_groups; ++i) {
    const long long n = g.num_groups == 1 ? g.out_features : (layer->group_rows ? layer->group_rows[i] : -1);
    if (n <= 0) return WAL_ERR_INVALID_ARGUMENT;
    if (i + 1 < g.num_groups && (rows + n) % pair::kRows != 0) return WAL_ERR_UNSUPPORTED;
    rows += n;
    t += (n + 15) / 16;
    p.group_tile_start[i + 1] = (int)t;
    p.group_row_start[i + 1] = (int)rows;
  }
  if (t != layer->num_tiles || rows != g.out_features) return WAL_ERR_SHAPE;

  EncodeTiledFn enc = encode_fn();
  if (!enc) return WAL_ERR_CUDA;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)g.in_features, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  // Token tile per pair: 512, 384 or 256 (MMA N = 256, 192 or 128).  A stage
  // takes about 1400 cycles whatever the tile (the shared-memory port: weight
  // operand reads, both SMs reading each CTA's activation half, the fills and
  // the decode), so the rule is the fewest waves of pairs on the GPU's pair
  // slots, then the smallest tile (8B q/k/v at 2048 tokens: 144 pairs of 384 in
  // two waves, 125 us, against 96 pairs of 512 in two waves, 136 us; o at 512
  // tokens: 59 us with 256 against 61 us with 512).
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long slots = sms / 2, row_pairs = ((g.out_features + pair::kRows - 1) / pair::kRows + 1) / 2;
  auto waves = [&](long long tok) { return (row_pairs * ((M + tok - 1) / tok) + slots - 1) / slots; };
  p.tok = 512;
  for (int tok : {384, 256})
    if (waves(tok) <= waves(p.tok)) p.tok = tok;
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)(p.tok / 4)};  // one box per accumulator half
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x),
          dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return WAL_ERR_CUDA;
  const int R = g.num_stages;
  const int smem = pair::smem_bytes(R);
  // CTA pairs along the weight rows: an odd tile count gets one padding CTA
  const long long row_tiles = (g.out_features + pair::kRows - 1) / pair::kRows;
  if ((row_tiles + 1) / 2 > 65535) return WAL_ERR_SHAPE;  // pairs of row tiles along grid y
  const dim3 grid((unsigned)(2 * ((M + p.tok - 1) / p.tok)), (unsigned)((row_tiles + 1) / 2));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nm = fast ? kFast : kExact;
  switch (R * 100 + nm * 10 + (f16 ? 1 : 0)) {
    case 100 + kExact * 10: return launch_gemm_pair<1, num_mode(kExact, false)>(map, p, grid, smem, s);
    case 100 + kExact * 10 + 1: return launch_gemm_pair<1, num_mode(kExact, true)>(map, p, grid, smem, s);
    case 100 + kFast * 10: return launch_gemm_pair<1, num_mode(kFast, false)>(map, p, grid, smem, s);
    case 100 + kFast * 10 + 1: return launch_gemm_pair<1, num_mode(kFast, true)>(map, p, grid, smem, s);
    case 200 + kExact * 10: return launch_gemm_pair<2, num_mode(kExact, false)>(map, p, grid, smem, s);
    case 200 + kExact * 10 + 1: return launch_gemm_pair<2, num_mode(kExact, true)>(map, p, grid, smem, s);
    case 200 + kFast * 10: return launch_gemm_pair<2, num_mode(kFast, false)>(map, p, grid, smem, s);
    case 200 + kFast * 10 + 1: return launch_gemm_pair<2, num_mode(kFast, true)>(map, p, grid, smem, s);
    default: return WAL_ERR_UNSUPPORTED;
  }
}

extern "C" int wal_rvq_gemm(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                            int64_t ldy, int y_dtype, int* status, void* stream) {
  return wal_rvq_gemm_typed(layer, x, WAL_BF16, M, ldx, y, ldy, y_dtype, status, stream);
}
