// Prefill path (M >= 256 tokens): fused Block-RVQ decode -> shared memory ->
// tcgen05.mma (5th-generation tensor cores, fp32 accumulators in TMEM).
//
// One CTA computes a 512 (tokens) x 128 (output rows) tile of y over all of K
// in stages of 64 columns (a CTA whose tokens end early loads and multiplies
// only the 128-token tiles that hold tokens), with warp specialisation:
//   warp 0      TMA producer: the activation tile [512 x 64] bf16 per stage
//               (two 256-row boxes), cp.async.bulk.tensor into a
//               128-byte-swizzled K-major buffer (no multicast), completion
//               on full_a[stage];
//   warp 1      MMA issuer (one elected lane): waits full_a + full_b, issues
//               16 x tcgen05.mma (M=128, N=128, K=16: four token tiles share
//               each decoded weight tile) into four TMEM accumulators and
//               commits to empty[stage] (the stage's buffers are free again)
//               and, after the last stage, to acc_full;
//   warps 2..17 decoders: for every stage decode the 128 x 64 weight tile
//               exactly (same arithmetic as the decode GEMV: fp32 stage sum,
//               two bf16 roundings; four threads per row, two blocks each,
//               ids loaded four stages ahead) straight into the swizzled
//               K-major B buffer,
//               fence it for the async proxy and arrive on full_b; then the
//               epilogue: TMEM -> registers (tcgen05.ld 32x32b), bias,
//               bf16/fp32 store of y.
// Sharing each decoded tile over 512 tokens keeps the exact decode (CUDA
// cores) below the tensor-core time of the same stage.  Measured on B200 with
// the Llama-3-8B projections at 2048 tokens: this tile runs at 969 TFLOP/s; a
// 256 x 256 tile (MMA N = 256, three stages: half the activation bytes from L2
// per FLOP, twice the decode per FLOP) at 797; a persistent stream-K schedule
// of the same tile (even (tile, k-block) shares per SM, split tiles summed
// through a workspace) at 810-830, its per-segment epilogues and pipeline
// refills costing more than the part-empty last wave it removes.
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

constexpr int kBM = 512;   // tokens per CTA: four 128-row MMA tiles share each decoded weight tile
constexpr int kUM = 128;   // MMA M
constexpr int kBN = 128;   // output rows per CTA (MMA N)
constexpr int kBK = 64;
constexpr int kStages = 2;
constexpr int kTmaRows = 256;  // TMA box height: two boxes per activation stage
constexpr int kDecodeWarps = 16;
constexpr int kRowParts = kDecodeWarps * 32 / 128;  // decoder threads per weight row
constexpr int kPartBlocks = 8 / kRowParts;          // d = 8 blocks per thread per 64-column stage
constexpr int kThreads = (2 + kDecodeWarps) * 32;
constexpr int kABytes = kBM * kBK * 2;  // 64 KB
constexpr int kBBytes = kBN * kBK * 2;  // 16 KB
constexpr int kCbCopyBytes = 256 * 16;  // one stage table, one copy
constexpr int kCbCopies = 8;            // 8-lane phases of 16-byte gathers hit 8 distinct bank quads
constexpr int kTmemCols = 512;          // four 128 x 128 fp32 accumulators
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

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
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

// Instruction descriptor: kind::f16, D = f32, A and B both bf16 (format 1) or
// both fp16 (format 0), both K-major, M = 128, N = kBN.
template <bool F16>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | (F16 ? 0u : (1u << 7) | (1u << 10)) | ((uint32_t)(kBN >> 3) << 17) |
         ((uint32_t)(kUM >> 4) << 24);
}

template <bool F16>
__device__ __forceinline__ void umma_16bit(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc<F16>()), "r"(accumulate), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

template <int R, int NUM>
__global__ void __launch_bounds__(kThreads, 1) rvq_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                               const __grid_constant__ GemmParams p) {
  constexpr int NM = NUM & 3;
  constexpr bool F16 = (NUM & 4) != 0;
  using T = WT<F16>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned region: [A stages][B stages][codebooks][barriers][tmem slot]
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t a_sm = base;
  const uint32_t b_sm = a_sm + kStages * kABytes;
  const uint32_t cb_sm = b_sm + kStages * kBBytes;
  uint8_t* cb = gbase + (cb_sm - base);
  const uint32_t bar_sm = cb_sm + R * kCbCopyBytes * kCbCopies;
  const uint32_t full_a = bar_sm, full_b = bar_sm + 8 * kStages, empty = bar_sm + 16 * kStages;
  const uint32_t acc_full = bar_sm + 24 * kStages;
  const uint32_t tmem_slot = acc_full + 8;
  volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * kBN;
  // 128-token MMA tiles holding real tokens (the last CTA of a small M needs
  // fewer than four) and the 256-row activation boxes they read
  const int mtiles = min(kBM / kUM, (p.M - m0 + kUM - 1) / kUM);
  const int boxes = (mtiles * kUM + kTmaRows - 1) / kTmaRows;
  const int kblocks = (p.K + kBK - 1) / kBK;

  // row group of this N tile (the host guarantees a tile never straddles groups)
  int g = 0;
  while (g + 1 < p.num_groups && p.group_row_start[g + 1] <= n0) ++g;
  const int g_row0 = p.group_row_start[g], g_row1 = p.group_row_start[g + 1];
  const int g_tile0 = p.group_tile_start[g];

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_a + 8 * s, 1);
      mbar_init(full_b + 8 * s, kDecodeWarps);
      mbar_init(empty + 8 * s, 1);
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // codebooks of this group: [R][256][8] x 8 copies (one-stage and fast-mode
  // tables converted to the weight type, exactly as the GEMV stages them)
  {
    const uint16_t* books = p.codebooks + (size_t)g * R * p.entries * 8;
    const float* scales = p.stage_scales ? p.stage_scales + (size_t)g * R : nullptr;
    for (int i = threadIdx.x; i < R * p.entries; i += kThreads) {
      const int st = i / p.entries, e = i - st * p.entries;
      uint4 v = *reinterpret_cast<const uint4*>(books + (size_t)i * 8);
      v.x = staged_word<R, NM, F16>(v.x, scales, st);
      v.y = staged_word<R, NM, F16>(v.y, scales, st);
      v.z = staged_word<R, NM, F16>(v.z, scales, st);
      v.w = staged_word<R, NM, F16>(v.w, scales, st);
#pragma unroll
      for (int c = 0; c < kCbCopies; ++c)
        *reinterpret_cast<uint4*>(cb + ((st * 256 + e) * kCbCopies + c) * 16) = v;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;

  if (warp == 0) {
    // ---------------- TMA producer -------------------------------------
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(empty + 8 * s, ((kb / kStages) - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        if (abort_flag) break;
        mbar_expect_tx(full_a + 8 * s, boxes * (kTmaRows * 128));
        for (int h = 0; h < boxes; ++h)
          tma_load_2d(a_sm + s * kABytes + h * (kTmaRows * 128), &xmap, kb * kBK, m0 + h * kTmaRows, full_a + 8 * s);
        ++issued;
      }
      // never leave a copy in flight: wait (bounded) for the last load of every stage
      for (int kb = issued - kStages < 0 ? 0 : issued - kStages; kb < issued; ++kb)
        if (!mbar_wait(full_a + 8 * (kb % kStages), (kb / kStages) & 1)) abort_flag = 1;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------------------------------
    if (lane == 0) {
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % kStages;
        const uint32_t par = (kb / kStages) & 1;
        if (!mbar_wait(full_a + 8 * s, par) || !mbar_wait(full_b + 8 * s, par)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t bd = smem_desc_sw128(b_sm + s * kBBytes + ks * 32);
#pragma unroll
          for (int mt = 0; mt < kBM / kUM; ++mt) {
            if (mt >= mtiles) break;
            const uint64_t ad = smem_desc_sw128(a_sm + s * kABytes + mt * (kUM * 128) + ks * 32);
            umma_16bit<F16>(tmem + (uint32_t)(mt * kBN), ad, bd, (kb > 0 || ks > 0) ? 1u : 0u);
          }
        }
        umma_commit(empty + 8 * s);
      }
      umma_commit(acc_full);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------- decoders, then epilogue -----------------------------
    const int t = threadIdx.x - 64;  // row t & 127 of the tile, blocks part * kPartBlocks.. of each stage
    const int row = t & (kBN - 1), part = t >> 7;
    const int n = n0 + row;
    const bool row_ok = n < g_row1;
    const uint32_t rho2 = row_ok ? T::rho2(p.row_scale[n]) : 0u;
    const int local = n - g_row0;
    const long long tile = (long long)g_tile0 + local / 16;
    const int rr = local % 16;
    const long long tile_bytes = (long long)p.chunks * R * 256;
    const uint8_t* idrow = p.packed + tile * tile_bytes + rr * 16 + part * kPartBlocks;
    const uint32_t bsm_row0 = b_sm + (row >> 3) * 1024 + (row & 7) * 128;
    const uint32_t cb_lane = cb_sm + (uint32_t)(lane & 7) * 16;
    const int nsw = row & 7;
    // stage kb covers blocks 8kb..8kb+7 = bytes 8*(kb&1) of chunk kb/2; this
    // thread's blocks are kPartBlocks bytes per part further in.  The ids
    // stream from HBM once (evict-first loads), kIdAhead stages ahead.
    static_assert(kPartBlocks == 2 || kPartBlocks == 4, "ids are loaded as 2 or 4 bytes");
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
    uint32_t idq[kIdAhead + 1][R];  // idq[0]: this stage; idq[j]: stage kb + j
#pragma unroll
    for (int j = 0; j < kIdAhead; ++j) load_ids(j, idq[j]);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % kStages;
      load_ids(kb + kIdAhead, idq[kIdAhead]);
      if (kb >= kStages && !mbar_wait(empty + 8 * s, ((kb / kStages) - 1) & 1)) {
        abort_flag = 1;
        break;
      }
      if (abort_flag) break;
      const int k_left = row_ok ? p.K - kb * kBK : 0;
      decode_stage_part<R, NUM>(bsm_row0 + s * kBBytes, nsw, idq[0], part * kPartBlocks, cb_lane, rho2, k_left);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(full_b + 8 * s);
#pragma unroll
      for (int j = 0; j < kIdAhead; ++j)
#pragma unroll
        for (int st = 0; st < R; ++st) idq[j][st] = idq[j + 1][st];
    }
    // epilogue: TMEM lanes 32*(warp%4) .. +31 are this warp's tokens
    const bool ok = !abort_flag && mbar_wait(acc_full, 0);
    if (!ok) abort_flag = 1;
    tc_fence_after();
    if (ok) {
      const int quarter = warp & 3;
      const bool vec_ok = (p.ldy % 8) == 0 && ((uintptr_t)p.y & 15) == 0;
      // kDecodeWarps / 4 warps share a lane quarter and split the four accumulators
      constexpr int kAccPerWarp = 16 / kDecodeWarps;
      for (int mi = 0; mi < kAccPerWarp; ++mi) {
      const int mt = kAccPerWarp * ((warp - 2) >> 2) + mi;
      if (mt >= mtiles) continue;  // this accumulator holds no tokens (warp-uniform)
      const int m = m0 + mt * kUM + quarter * 32 + lane;
      for (int c0 = 0; c0 < kBN; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(mt * kBN + c0), v);
        if (m >= p.M) continue;
        const int col0 = n0 + c0;
        float f[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          f[j] = __uint_as_float(v[j]);
          if (p.bias && col0 + j < g_row1) f[j] += __bfloat162float(__ushort_as_bfloat16(p.bias[col0 + j]));
        }
        const bool full = col0 + 16 <= g_row1 && vec_ok;
        if (p.y_dtype == WAL_F32) {
          float* yr = static_cast<float*>(p.y) + (long long)m * p.ldy + col0;
          if (full) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(yr + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
          } else {
            for (int j = 0; j < 16; ++j)
              if (col0 + j < g_row1) yr[j] = f[j];
          }
        } else {  // 16-bit output: bf16 or fp16, one rounding of the fp32 sum
          const bool yf16 = p.y_dtype == WAL_F16;
          uint16_t* yr = static_cast<uint16_t*>(p.y) + (long long)m * p.ldy + col0;
          if (full) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              w[j] = yf16 ? WT<true>::cvt2(f[2 * j], f[2 * j + 1]) : WT<false>::cvt2(f[2 * j], f[2 * j + 1]);
            *reinterpret_cast<uint4*>(yr) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(yr + 8) = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
            for (int j = 0; j < 16; ++j)
              if (col0 + j < g_row1)
                yr[j] = yf16 ? __half_as_ushort(__float2half_rn(f[j])) : __bfloat16_as_ushort(__float2bfloat16_rn(f[j]));
          }
        }
      }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (abort_flag && threadIdx.x == 0 && p.status) atomicExch(p.status, 1);
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

int smem_bytes(int R) {
  return 1024 + kStages * (kABytes + kBBytes) + R * kCbCopyBytes * kCbCopies + 8 * (3 * kStages + 1) + 16;
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
static int launch_gemm(const CUtensorMap& map, const GemmParams& p, dim3 grid, int smem, cudaStream_t s) {
  if (cudaFuncSetAttribute(rvq_gemm_kernel<R, NUM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return WAL_ERR_CUDA;
  rvq_gemm_kernel<R, NUM><<<grid, kThreads, smem, s>>>(map, p);
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
  p.num_groups = g.num_groups;
  // group boundaries; an N tile (kBN rows) must not straddle two groups
  long long t = 0, rows = 0;
  p.group_tile_start[0] = 0;
  p.group_row_start[0] = 0;
  for (int i = 0; i < g.num_groups; ++i) {
    const long long n = g.num_groups == 1 ? g.out_features : (layer->group_rows ? layer->group_rows[i] : -1);
    if (n <= 0) return WAL_ERR_INVALID_ARGUMENT;
    if (i + 1 < g.num_groups && (rows + n) % kBN != 0) return WAL_ERR_UNSUPPORTED;
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
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kTmaRows};  // 64 x 256: two loads per stage
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x),
          dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return WAL_ERR_CUDA;
  const int R = g.num_stages;
  const int smem = smem_bytes(R);
  const dim3 grid((unsigned)((M + kBM - 1) / kBM), (unsigned)((g.out_features + kBN - 1) / kBN));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nm = fast ? kFast : kExact;
  switch (R * 100 + nm * 10 + (f16 ? 1 : 0)) {
    case 100 + kExact * 10: return launch_gemm<1, num_mode(kExact, false)>(map, p, grid, smem, s);
    case 100 + kExact * 10 + 1: return launch_gemm<1, num_mode(kExact, true)>(map, p, grid, smem, s);
    case 100 + kFast * 10: return launch_gemm<1, num_mode(kFast, false)>(map, p, grid, smem, s);
    case 100 + kFast * 10 + 1: return launch_gemm<1, num_mode(kFast, true)>(map, p, grid, smem, s);
    case 200 + kExact * 10: return launch_gemm<2, num_mode(kExact, false)>(map, p, grid, smem, s);
    case 200 + kExact * 10 + 1: return launch_gemm<2, num_mode(kExact, true)>(map, p, grid, smem, s);
    case 200 + kFast * 10: return launch_gemm<2, num_mode(kFast, false)>(map, p, grid, smem, s);
    case 200 + kFast * 10 + 1: return launch_gemm<2, num_mode(kFast, true)>(map, p, grid, smem, s);
    default: return WAL_ERR_UNSUPPORTED;
  }
}

extern "C" int wal_rvq_gemm(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                            int64_t ldy, int y_dtype, int* status, void* stream) {
  return wal_rvq_gemm_typed(layer, x, WAL_BF16, M, ldx, y, ldy, y_dtype, status, stream);
}
