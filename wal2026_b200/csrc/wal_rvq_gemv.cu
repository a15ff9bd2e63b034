// Decode-time fused gather-GEMV (up to 32 tokens per launch), weight materialisation and
// packed-id unpacking for the Block-RVQ runtime linear.
//
// GEMV structure (one persistent wave of CTAs, 16 warps each):
//   * every CTA works inside one row group: it stages that group's codebooks
//     in shared memory once (cp.async);
//   * the CTA's tiles are processed in rounds of `slots` tiles; the 16-block
//     chunks of a tile are split over `wpt` warps (slots * wpt = 16), warp
//     `kpart` of a slot taking chunks kpart, kpart + wpt, ...;
//   * activations: staged whole in shared memory when they fit; otherwise
//     streamed through a three-deep window ring shared by the CTA: step j of a
//     round needs the same wpt chunks' columns in every slot, so four producer
//     warps (warps 16..19) copy each window once per CTA instead of once per
//     16-row tile, handing buffers to the 16 compute warps through hardware
//     named barriers (full: producer arrives, compute warps wait; empty: the
//     reverse), which lets compute warps drift up to two windows apart;
//   * each warp walks its own flat list of (tile, chunk) items with a
//     kRing-deep cp.async ring in shared memory, so id loads for later items
//     are in flight while the current one is decoded (no spin-waits: the copy
//     engine's group counters are the only synchronisation);
//   * every weight is decoded exactly in registers (wal_rvq_decode.cuh) and
//     fed to mma.sync m16n8k16 (bf16, fp32 accumulate) with the activation
//     fragment: the dense weight never exists;
//   * the wpt warps of a slot reduce their partial sums through shared memory
//     behind a named barrier of their own, in a fixed order, add the bias in
//     fp32 and write y once.
// Replaces reference src/runtime.py:1501-1507 (reconstruct + F.linear) and the
// fused Triton kernel src/triton_id_matmul.py:143-217.
#include "../../include/wal_rvq.h"
#include "wal_rvq_decode.cuh"

#include <cstdio>
#include <mutex>
#include <type_traits>
#include <vector>

namespace wal {

constexpr int kMaxGroups = 64;

struct GemvParams {
  const uint8_t* packed;
  const int4* tiles;
  const uint16_t* codebooks;
  const uint16_t* row_scale;
  const uint16_t* bias;
  const float* stage_scales;  // fp32 [groups][R] or null
  const uint16_t* x;
  void* y;
  long long ldx, ldy;
  long long num_tiles;
  int K;
  int chunks;
  int entries;
  int M;
  int y_dtype;
  int wpt;
  int num_groups;
  int pdl;                               // launched with programmatic dependent launch
  int early_release;                     // release the next kernel after the prologue (grid leaves SMs idle)
  int wpt_shift;                         // log2(wpt)
  int auto_tpc;                          // tiles per CTA when wpt was chosen automatically, else 0
  int group_tile_start[kMaxGroups + 1];  // first tile of each group, plus the total
  int group_row_start[kMaxGroups + 1];   // first output row of each group, plus N
  // CTA split (host-computed for the launch's grid): group g owns CTAs
  // [cta_start[g], cta_start[g+1]); its k-th CTA gets tiles_q[g] tiles, plus
  // one more when k < tiles_r[g]
  int cta_start[kMaxGroups + 1];
  int tiles_q[kMaxGroups];
  int tiles_r[kMaxGroups];
  // tensor-parallel push (push_ranks > 0): every fp32 output goes, as an
  // 8-byte word {value, tag}, to push_dst[p] for every rank p instead of y;
  // tag = *push_epoch + 1 (the slot's call count, read after the dependency)
  int push_ranks;
  long long push_ld;
  uint2* push_dst[WAL_MAX_RANKS];
  const unsigned* push_epoch;
};

namespace {

template <int I, int N, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    static_for<I + 1, N>(f);
  }
}

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = 4;  // chunks in flight per warp (power of two)
constexpr int kXSmemBudget = 64 * 1024;
constexpr int kMaxTokens = 32;  // tokens per GEMV launch (four n-tiles of 8); more run as slabs


__device__ __forceinline__ void store_out(void* y, long long idx, float v, int dtype) {
  if (dtype == WAL_F32) {
    static_cast<float*>(y)[idx] = v;
  } else if (dtype == WAL_BF16) {
    static_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(y)[idx] = __float2half_rn(v);
  }
}

// One output element: y (dtype) or, in push mode, a tagged 8-byte word into
// every rank's receive rows (remote ranks through NVLink peer mappings).
__device__ __forceinline__ void emit_out(const GemvParams& p, unsigned tag, int m, int row, float v) {
  if (p.push_ranks > 0) {
    const long long idx = (long long)m * p.push_ld + row;
#pragma unroll
    for (int r = 0; r < WAL_MAX_RANKS; ++r)
      if (r < p.push_ranks)
        asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};\n" ::"l"(p.push_dst[r] + idx),
                     "r"(__float_as_uint(v)), "r"(tag)
                     : "memory");
  } else {
    store_out(p.y, (long long)m * p.ldy + row, v, p.y_dtype);
  }
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_barrier_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Which group and tile range a CTA owns (division-free: the split is host-computed).
__device__ __forceinline__ void cta_range(const GemvParams& p, int cta, int* group, int* tb, int* te) {
  int g = 0;
  while (g + 1 < p.num_groups && cta >= p.cta_start[g + 1]) ++g;
  const int local = cta - p.cta_start[g];
  const int q = p.tiles_q[g], rem = p.tiles_r[g];
  *group = g;
  *tb = p.group_tile_start[g] + local * q + (local < rem ? local : rem);
  *te = *tb + q + (local < rem ? 1 : 0);
}

// Activation modes: XM = 0 read from global memory per fragment (fallback),
// 1 staged whole, 2 window ring.
constexpr int kXBufs = 3;  // window ring depth
// named barrier ids: 0 = __syncthreads, 1..8 = slot reductions (wpt >= 2),
// window ring full / empty per buffer
constexpr int kFullBar = 9;
constexpr int kEmptyBar = kFullBar + kXBufs;

template <int D, int R, int IDW, bool REPL, int MT, int XM>
struct GemvCfg {
  using L = CbLayout<D, REPL>;
  // one CTA of 16 warps per SM shares one staged codebook
  static constexpr int kW = 16;                          // compute warps
  static constexpr int kP = XM == 2 ? 4 : 0;              // window producer warps
  static constexpr int kT = (kW + kP) * 32;
  static constexpr int V = R * IDW;               // 16-byte vectors per row-chunk
  static constexpr int NW = V * 4;                // 32-bit code words per row-chunk
  static constexpr int kStageBytes = V * 256;     // one chunk of one tile (16 rows)
  static constexpr int MC = MT * 8;
  static constexpr int kAcc = MT >= 4 ? 1 : 2;  // accumulator sets (k-tile parity)
  __host__ __device__ static int cb_bytes(int entries) { return L::total_bytes(R, entries); }
  // activations: M rows plus one zero row that lanes beyond M read; the row
  // stride is padded by 32 bytes so rows read together fall in different banks
  __host__ __device__ static int x_stride(int kpad) { return kpad * 2 + 32; }
  // window ring: kXBufs buffers of MC rows x wpt chunks (rows >= M stay zero)
  __host__ __device__ static int xw_stride(int wpt) { return wpt * kChunkBlocks * D * 2 + 32; }
  __host__ __device__ static int x_bytes(int M, int kpad, int wpt) {
    if (XM == 1) return (((M + 1) * x_stride(kpad) + 127) / 128) * 128;
    if (XM == 2) return ((kXBufs * MC * xw_stride(wpt) + 127) / 128) * 128;
    return 0;
  }
  __host__ __device__ static int ring_bytes() { return kW * kRing * kStageBytes; }
  // partial sums of a slot's warps: double-buffered by round parity, except
  // with the window ring (whose smem is scarcer): one buffer and a second slot
  // barrier after the reads
  static constexpr int kRedBufs = XM == 2 ? 1 : 2;
  __host__ __device__ static int red_bytes() { return kRedBufs * kW * 16 * MC * 4; }
  __host__ __device__ static int smem(int entries, int M, int kpad, int wpt) {
    return cb_bytes(entries) + x_bytes(M, kpad, wpt) + ring_bytes() + red_bytes();
  }
};

// col_base: the lane's first global column of the chunk (unstaged activations,
// masking); xcol: the same column inside the staged buffer.
template <int D, int R, int IDW, bool REPL, int MT, int XM, bool MASK, int NUM>
__device__ __forceinline__ void gemv_chunk(float (&acc)[GemvCfg<D, R, IDW, REPL, MT, XM>::kAcc][MT][4], const uint32_t (&c0)[R * IDW * 4],
                                           const uint32_t (&c1)[R * IDW * 4], uint32_t cb, uint32_t cbl, uint32_t rho_a,
                                           uint32_t rho_b, const LaneSel& ls, const uint16_t* x, const uint32_t (&xoff)[MT],
                                           const uint32_t (&xsa)[MT], const bool (&xv)[MT], int col_base, int xcol, int K) {
  using C = GemvCfg<D, R, IDW, REPL, MT, XM>;
  using T = WT<(NUM & 4) != 0>;
  // activations of k-tile kt, then the MMAs of the decoded fragments ra (row r), rb (row r + 8)
  auto consume = [&](auto ktc, const uint32_t (&ra)[2], const uint32_t (&rb)[2]) {
    constexpr int kt = decltype(ktc)::value;
    const int col = col_base + kt * 16;  // lane's first physical column (includes 4q)
    const bool in_k = !MASK || col < K;
    uint2 xf[MT];
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if constexpr (XM != 0) {  // rows beyond M read zero rows: no predicate
        xf[i] = lds64_ordered<kt * 32>(xsa[i] + xcol * 2);
      } else {
        xf[i] = make_uint2(0u, 0u);
        if (xv[i] && in_k) xf[i] = __ldg(reinterpret_cast<const uint2*>(x + xoff[i] + col));
      }
    }
    uint32_t a[4] = {ra[0], rb[0], ra[1], rb[1]};
    if (MASK && !in_k) {
      a[0] = a[1] = a[2] = a[3] = 0u;
    }
    // with one or two n-tiles, even and odd k-tiles feed separate accumulators
    // (independent MMA chains); four n-tiles are four chains already
#pragma unroll
    for (int i = 0; i < MT; ++i) T::mma(acc[kt % C::kAcc][i], a, xf[i].x, xf[i].y);
  };
  if constexpr (R == 1) {
    // one-stage tables: one gather per row and k-tile; issue the gathers of
    // eight k-tiles before using any, so their shared-memory latency overlaps
    constexpr int kGroup = 8;
    static_for<0, D / kGroup>([&](auto gc) {
      constexpr int g0 = decltype(gc)::value * kGroup;
      uint2 pa[kGroup], pb[kGroup];
      static_for<0, kGroup>([&](auto jc) {
        constexpr int j = decltype(jc)::value, kt = g0 + j;
        constexpr int half_off = (D == 32) ? (kt & 1) * CbLayout<D, REPL>::kHalfStride : 0;
        pa[j] = lds64<half_off>(piece_addr<D, R, IDW, REPL, kt, C::NW, 0>(c0, cb, ls, cbl));
        pb[j] = lds64<half_off>(piece_addr<D, R, IDW, REPL, kt, C::NW, 0>(c1, cb, ls, cbl));
      });
      static_for<0, kGroup>([&](auto jc) {
        constexpr int j = decltype(jc)::value;
        const uint32_t ra[2] = {T::mul2(pa[j].x, rho_a), T::mul2(pa[j].y, rho_a)};
        const uint32_t rb[2] = {T::mul2(pb[j].x, rho_b), T::mul2(pb[j].y, rho_b)};
        consume(std::integral_constant<int, g0 + j>{}, ra, rb);
      });
    });
  } else {
    static_for<0, D>([&](auto ktc) {
      constexpr int kt = decltype(ktc)::value;
      uint32_t ra[2], rb[2];
      decode_row<D, R, IDW, REPL, kt, C::NW, NUM>(ra, c0, cb, cbl, rho_a, ls);
      decode_row<D, R, IDW, REPL, kt, C::NW, NUM>(rb, c1, cb, cbl, rho_b, ls);
      consume(ktc, ra, rb);
    });
  }
}

template <int D, int R, int IDW, bool REPL, int MT, int XM, int NUM>
__global__ void __launch_bounds__(GemvCfg<D, R, IDW, REPL, MT, XM>::kT)
    rvq_gemv_kernel(const __grid_constant__ GemvParams p) {
  constexpr int NM = NUM & 3;
  constexpr bool F16 = (NUM & 4) != 0;
  using T = WT<F16>;
  using C = GemvCfg<D, R, IDW, REPL, MT, XM>;
  constexpr int kWarps = C::kW;
  constexpr int kThreads = C::kT;
  using L = typename C::L;
  constexpr int V = C::V;
  constexpr int MC = C::MC;
  extern __shared__ __align__(128) uint8_t smem[];
  const int kpad = p.chunks * kChunkBlocks * D;
  uint8_t* cb = smem;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + C::cb_bytes(p.entries));
  uint8_t* ring = smem + C::cb_bytes(p.entries) + C::x_bytes(p.M, kpad, p.wpt);
  float* red = reinterpret_cast<float*>(ring + C::ring_bytes());  // [kRedBufs][kW][16][MC]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q = lane & 3;
  static_assert(kWarps == 16, "warp split assumes 16 compute warps");
  const bool producer = XM == 2 && warp >= kWarps;  // the window ring's copy warps
  const int wpt = p.wpt, wsh = p.wpt_shift;  // wpt = 1 << wsh
  const int ssh = 4 - wsh;                    // slots = 16 / wpt = 1 << ssh
  const int slots = 1 << ssh;
  const int slot = warp >> wsh, kpart = warp & (wpt - 1);
  constexpr bool kF32 = NM == kExactScaled && REPL && R > 1;  // scaled fp32 tables
  const LaneSel ls(r, q, kF32);

  int group, tb, te;
  cta_range(p, blockIdx.x, &group, &tb, &te);
  if (tb >= te) {
    if (p.pdl) grid_dependents_launch();
    return;
  }
  const int g_tile0 = p.group_tile_start[group];
  const int g_row0 = p.group_row_start[group], g_row1 = p.group_row_start[group + 1];

  // -- this warp's flat item list: rounds of `slots` tiles x its chunks -----
  const int cpw = kpart < p.chunks ? (p.chunks - kpart + wpt - 1) >> wsh : 0;  // chunks per tile
  const int ntiles = te - tb;
  const int rounds = (ntiles + slots - 1) >> ssh;
  // tiles this warp owns: tb + slot + k * slots, k < my_rounds
  const int my_rounds = !producer && slot < ntiles ? (ntiles - slot + slots - 1) >> ssh : 0;
  const int items = my_rounds * cpw;
  const long long tile_bytes = (long long)p.chunks * V * 256;
  uint8_t* wring = ring + warp * kRing * C::kStageBytes;

  // issue cursor: the next item's source (advanced incrementally), items left
  // to issue, position inside the tile's chunk list, ring slot
  constexpr int kLaneCopies = (C::kStageBytes + 511) / 512;  // 16-byte copies per lane per chunk
  // copies of this lane inside the chunk (three stages: 768 bytes, lanes 16..31 make one copy)
  const int lane_copies = (C::kStageBytes - lane * 16 + 511) / 512;
  // 64-bit base of this warp's first item plus a 32-bit running offset (the
  // host keeps a CTA's tile span below 2^31 bytes)
  const uint8_t* is_base = p.packed + (long long)(tb + slot) * tile_bytes + kpart * V * 256 + lane * 16;
  const uint32_t step_chunk = (uint32_t)(wpt * V * 256);
  const uint32_t step_tile = (uint32_t)(slots * tile_bytes) - (uint32_t)cpw * step_chunk;
  uint32_t is_off = 0;
  const uint32_t ring_lane = smem_u32(wring) + lane * 16;
  const uint32_t ring_row = smem_u32(wring) + r * 16;  // this lane's row r; row r + 8 is 128 bytes on
  const uint64_t stream_pol = l2_policy_evict_first();
  int is_left = items;
  int is_j = 0;
  uint32_t is_slot = 0;
  auto issue_ids = [&]() {
    if (is_left > 0) {
#pragma unroll
      for (int k = 0; k < kLaneCopies; ++k)
        if (k < lane_copies)
          cp_async_16_hint(ring_lane + is_slot * C::kStageBytes + k * 512, is_base + is_off + k * 512, stream_pol);
      --is_left;
      is_off += step_chunk;
      if (++is_j == cpw) {
        is_j = 0;
        is_off += step_tile;
      }
    }
    is_slot = (is_slot + 1) & (kRing - 1);
  };
  auto issue = [&]() {
    issue_ids();
    cp_async_commit();
  };

  // window ring (XM == 2): window w of a round covers chunks [w * wpt, (w + 1) * wpt);
  // step s of the CTA reads buffer s % kXBufs
  const int spr = (p.chunks + wpt - 1) >> wsh;  // steps per round, equal for every warp
  const uint32_t xw_stride = (uint32_t)C::xw_stride(wpt);
  const uint32_t xbuf_bytes = (uint32_t)MC * xw_stride;
  const uint32_t xs_s = smem_u32(xs);
  const bool x16 = (((uintptr_t)p.x & 15) == 0) && ((p.ldx & 7) == 0);
  // copies of window w into buffer b by the producer warps' threads
  auto copy_window = [&](int w, uint32_t b, uint64_t pol) {
    constexpr int kPT = C::kP * 32;
    const int col0 = w * wpt * kChunkBlocks * D;
    const uint32_t dst0 = xs_s + b * xbuf_bytes;
    constexpr int kVecShift = D == 8 ? 4 : (D == 16 ? 5 : 6);  // log2(16-byte vectors per chunk row)
    const int vsh = wsh + kVecShift;
    const int nvec = p.M << vsh;
    for (int v = (int)threadIdx.x - kWarps * 32; v < nvec; v += kPT) {
      const int m = v >> vsh, vec = v & ((1 << vsh) - 1);
      const int col = col0 + vec * 8;
      const int left = p.K - col;
      const uint32_t nb = left >= 8 ? 16u : (left > 0 ? (uint32_t)left * 2u : 0u);
      const uint16_t* src = nb ? p.x + (long long)m * p.ldx + col : p.x;
      const uint32_t dst = dst0 + (uint32_t)m * xw_stride + (uint32_t)vec * 16;
      if (x16) {
        cp_async_16_zfill(dst, src, nb, pol);
      } else {
        cp_async_8_zfill(dst, src, nb > 8 ? 8u : nb);
        cp_async_8_zfill(dst + 8, nb > 8 ? src + 4 : p.x, nb > 8 ? nb - 8 : 0u);
      }
    }
  };

  // -- prologue: weights (static) first, activations after the dependency --
  // group 0: codebooks (+ activations); groups 1..kRing-1: the first id chunks
  // Everything that depends only on the weights (codebooks, first id chunks,
  // the replicated codebook build) happens before the grid-dependency wait,
  // so with programmatic dependent launch it overlaps the previous kernel;
  // only the activations wait for it.
  // groups: 0 = codebooks, 1..kRing-1 = first id chunks, kRing = activations
  const uint16_t* gbooks = p.codebooks + (size_t)group * R * p.entries * D;
  const float* gscales = p.stage_scales ? p.stage_scales + (size_t)group * R : nullptr;
  if constexpr (!kF32) stage_codebooks_issue<D, R, REPL, NM, F16>(cb, gbooks, p.entries);
  cp_async_commit();
#pragma unroll 1
  for (int s = 0; s < kRing - 1; ++s) issue();
  if constexpr (kF32) {
    stage_codebooks_scaled<D, R>(cb, gbooks, gscales, p.entries);  // plain loads, id chunks in flight
  } else {
    cp_async_wait<kRing - 1>();  // codebooks landed
    __syncthreads();
    stage_codebooks_finish<D, R, REPL, NM, F16>(cb, gbooks, p.entries, gscales);
  }
  if (p.pdl) grid_dependency_wait();  // x (and y) belong to the previous kernel in the stream
  const uint64_t x_pol = l2_policy_evict_last();
  if constexpr (XM == 2) {
    // rows M..MC-1 of every buffer stay zero (the copies only write rows < M)
    const int zw = (int)(xw_stride / 16), per_buf = (MC - p.M) * zw;
    for (int v = threadIdx.x; v < kXBufs * per_buf; v += kThreads) {
      const int b = v / per_buf, rem = v - b * per_buf;
      const int m = p.M + rem / zw, w16 = rem - (m - p.M) * zw;
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xs) + (size_t)b * xbuf_bytes + (size_t)m * xw_stride +
                                (size_t)w16 * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if constexpr (XM == 1) {
    // rows m < M, columns [0, kpad): zero beyond K
    const int vec_per_row = kpad / 8;  // 16-byte vectors
    for (int m = 0; m <= p.M; ++m) {
      uint16_t* xdst = xs + (size_t)m * (C::x_stride(kpad) / 2);
      const uint16_t* xsrc = p.x + (long long)m * p.ldx;
      for (int v = threadIdx.x; v < vec_per_row; v += kThreads) {
        uint16_t* dst = xdst + v * 8;
        if (m == p.M) {  // the zero row
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
          continue;
        }
        const int col = v * 8;
        const uint16_t* src = xsrc + col;
        if (col + 8 <= p.K && ((uintptr_t)src & 15) == 0) {
          cp_async_16_hint((uint32_t)__cvta_generic_to_shared(dst), src, x_pol);
        } else if (col + 8 <= p.K) {
          cp_async_8((uint32_t)__cvta_generic_to_shared(dst), src);
          cp_async_8((uint32_t)__cvta_generic_to_shared(dst + 4), src + 4);
        } else {
          for (int j = 0; j < 8; ++j) dst[j] = col + j < p.K ? xsrc[col + j] : (uint16_t)0;
        }
      }
    }
  }
  cp_async_commit();
  // push tag: the slot's call count advances only in the receiving kernel,
  // which runs after this one
  const unsigned tag = p.push_ranks > 0 ? *reinterpret_cast<const volatile unsigned*>(p.push_epoch) + 1u : 0u;
  cp_async_wait<0>();
  __syncthreads();
  // A grid smaller than the GPU releases the next kernel of the stream now:
  // that kernel is scheduled once every CTA of this grid has issued this (so
  // all of them are resident) and its CTAs start their weight prologue on the
  // SMs this grid leaves idle (cfg0 2048 x 2048, 128 CTAs: 6.7 -> 5.5 us per
  // launch).  A full grid releases it after its main loop instead: released
  // early, the next kernel's CTAs sit resident beside this grid's, and a
  // decode step of the 8B stack measured 1.7% slower.
  if (p.pdl && p.early_release) grid_dependents_launch();

  // lane (r, q) feeds token 8 * i + r of n-tile i
  uint32_t xoff[MT];  // element offset of the lane's token row (unstaged activations)
  uint32_t xsa[MT];   // shared address of the lane's token row (staged activations; window: row offset)
  bool xv[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    const int m = 8 * i + r;
    xv[i] = m < p.M;
    xoff[i] = (uint32_t)((xv[i] ? m : 0) * p.ldx);
    if constexpr (XM == 2) {
      xsa[i] = (uint32_t)m * xw_stride;  // rows >= M are zero rows
    } else {
      xsa[i] = smem_u32(xs) + (uint32_t)((xv[i] ? m : p.M) * C::x_stride(kpad));
    }
  }
  // Columns K..kpad of the last chunk decode padding ids.  Staged activations
  // are zero there, so those products vanish (every decoded weight is finite
  // for finite codebooks and row scales); only unstaged activations need the
  // weight fragment masked.
  const bool need_mask = XM == 0 && kpad != p.K;
  const uint32_t cb_s = smem_u32(cb);
  const uint32_t cbl = cb_s + L::lane_offset(r, q);

  // row scales of a tile: tile t covers rows g_row0 + 16 * (t - g_tile0) ...
  auto tile_rows = [&](int t, int* row0, int* nrows) {
    *row0 = g_row0 + 16 * (t - g_tile0);
    const int left = g_row1 - *row0;
    *nrows = left < 16 ? left : 16;
  };
  uint32_t nrho_a = 0u, nrho_b = 0u;
  if (my_rounds > 0) {
    int row0, nrows;
    tile_rows(tb + slot, &row0, &nrows);
    nrho_a = r < nrows ? T::rho2(p.row_scale[row0 + r]) : 0u;
    nrho_b = r + 8 < nrows ? T::rho2(p.row_scale[row0 + r + 8]) : 0u;
  }

  if constexpr (XM == 2) {
    if (producer) {
      // window s of the CTA (window s % spr of round s / spr) goes to buffer
      // s % kXBufs once the compute warps are done with window s - kXBufs; the
      // full barrier of window s - 1 is signalled when its copies have landed
      const int T = rounds * spr;
      int w = 0;
      uint32_t b = 0;
      for (int s = 0; s < T; ++s) {
        if (s >= kXBufs) named_barrier(kEmptyBar + (int)b, kThreads);
        copy_window(w, b, x_pol);
        cp_async_commit();
        if (s >= 1) {
          cp_async_wait<1>();
          named_barrier_arrive(kFullBar + (int)(b == 0 ? kXBufs - 1 : b - 1), kThreads);
        }
        if (++w == spr) w = 0;
        if (++b == kXBufs) b = 0;
      }
      cp_async_wait<0>();
      named_barrier_arrive(kFullBar + (int)(b == 0 ? kXBufs - 1 : b - 1), kThreads);
      // complete the empty barriers of the last windows
      for (int s = T > kXBufs ? T : kXBufs; s < T + kXBufs; ++s) named_barrier(kEmptyBar + s % kXBufs, kThreads);
      return;
    }
  }

  int it = 0;
  uint32_t xs_buf = 0;  // window ring: buffer of the current step
  for (int k = 0; k < rounds; ++k) {
    const bool slot_live = k < my_rounds;  // same for all warps of a slot
    float acc[C::kAcc][MT][4];
#pragma unroll
    for (int h = 0; h < C::kAcc; ++h)
#pragma unroll
      for (int i = 0; i < MT; ++i) acc[h][i][0] = acc[h][i][1] = acc[h][i][2] = acc[h][i][3] = 0.f;
    int row0 = 0, nrows = 0;
    uint32_t rho_a = 0u, rho_b = 0u;
    if (slot_live) {
      tile_rows(tb + slot + k * slots, &row0, &nrows);
      rho_a = nrho_a;
      rho_b = nrho_b;
      if (k + 1 < my_rounds) {  // prefetch the next round's row scales
        int nr0, nn;
        tile_rows(tb + slot + (k + 1) * slots, &nr0, &nn);
        nrho_a = r < nn ? T::rho2(p.row_scale[nr0 + r]) : 0u;
        nrho_b = r + 8 < nn ? T::rho2(p.row_scale[nr0 + r + 8]) : 0u;
      }
    }
    if constexpr (XM == 2) {
      // every compute warp takes the round's spr windows, live slot or not
      for (int j = 0; j < spr; ++j) {
        const int c = kpart + j * wpt;
        named_barrier(kFullBar + (int)xs_buf, kThreads);  // this window's activations landed
        if (slot_live && c < p.chunks) {
          cp_async_wait<kRing - 2>();
          __syncwarp();
          const uint32_t st = ring_row + (uint32_t)(it & (kRing - 1)) * C::kStageBytes;
          uint32_t c0[V * 4], c1[V * 4];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(c0[4 * v]), "=r"(c0[4 * v + 1]), "=r"(c0[4 * v + 2]), "=r"(c0[4 * v + 3])
                         : "r"(st + v * 256));
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(c1[4 * v]), "=r"(c1[4 * v + 1]), "=r"(c1[4 * v + 2]), "=r"(c1[4 * v + 3])
                         : "r"(st + v * 256 + 128));
          }
          __syncwarp();
          issue();
          const uint32_t xb = xs_s + xs_buf * xbuf_bytes;
          uint32_t xsa_s[MT];
#pragma unroll
          for (int i = 0; i < MT; ++i) xsa_s[i] = xb + xsa[i];
          gemv_chunk<D, R, IDW, REPL, MT, XM, false, NUM>(acc, c0, c1, cb_s, cbl, rho_a, rho_b, ls, p.x, xoff, xsa_s,
                                                     xv, c * kChunkBlocks * D + 4 * q,
                                                     kpart * kChunkBlocks * D + 4 * q, p.K);
          ++it;
        }
        named_barrier_arrive(kEmptyBar + (int)xs_buf, kThreads);  // done with this buffer
        if (++xs_buf == kXBufs) xs_buf = 0;
      }
    } else if (slot_live) {
      for (int j = 0; j < cpw; ++j, ++it) {
        cp_async_wait<kRing - 2>();
        __syncwarp();
        // 32-bit shared addresses (the ring slot of this item, this lane's rows)
        const uint32_t st = ring_row + (uint32_t)(it & (kRing - 1)) * C::kStageBytes;
        uint32_t c0[V * 4], c1[V * 4];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(c0[4 * v]), "=r"(c0[4 * v + 1]), "=r"(c0[4 * v + 2]), "=r"(c0[4 * v + 3])
                       : "r"(st + v * 256));
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(c1[4 * v]), "=r"(c1[4 * v + 1]), "=r"(c1[4 * v + 2]), "=r"(c1[4 * v + 3])
                       : "r"(st + v * 256 + 128));
        }
        __syncwarp();
        issue();
        const int c = kpart + j * wpt;
        const int col_base = c * kChunkBlocks * D + 4 * q;
        if (need_mask && c == p.chunks - 1) {
          gemv_chunk<D, R, IDW, REPL, MT, XM, true, NUM>(acc, c0, c1, cb_s, cbl, rho_a, rho_b, ls, p.x, xoff, xsa, xv,
                                                    col_base, col_base, p.K);
        } else {
          gemv_chunk<D, R, IDW, REPL, MT, XM, false, NUM>(acc, c0, c1, cb_s, cbl, rho_a, rho_b, ls, p.x, xoff, xsa, xv,
                                                     col_base, col_base, p.K);
        }
      }
    }
    if (p.pdl && !p.early_release && k + 1 == rounds) grid_dependents_launch();
    // -- reduce the slot's wpt partial sums, add bias, write y ---------------
    if (!slot_live) continue;
    if (wpt == 1) {
#pragma unroll
      for (int i = 0; i < MT; ++i) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = r + (e >= 2 ? 8 : 0);
          const int m = i * 8 + 2 * q + (e & 1);
          if (row < nrows && m < p.M) {
            float v = C::kAcc == 2 ? acc[0][i][e] + acc[C::kAcc - 1][i][e] : acc[0][i][e];
            if (p.bias) v += __bfloat162float(__ushort_as_bfloat16(p.bias[row0 + row]));
            emit_out(p, tag, m, row0 + row, v);
          }
        }
      }
      continue;
    }
    const int rbuf = C::kRedBufs == 2 ? (k & 1) : 0;
    float* wred = red + (rbuf * kWarps + warp) * 16 * MC;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      float v4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v4[e] = C::kAcc == 2 ? acc[0][i][e] + acc[C::kAcc - 1][i][e] : acc[0][i][e];
      wred[r * MC + i * 8 + 2 * q] = v4[0];
      wred[r * MC + i * 8 + 2 * q + 1] = v4[1];
      wred[(r + 8) * MC + i * 8 + 2 * q] = v4[2];
      wred[(r + 8) * MC + i * 8 + 2 * q + 1] = v4[3];
    }
    named_barrier(1 + slot, wpt * 32);
    const float* sred = red + (rbuf * kWarps + slot * wpt) * 16 * MC;
    const int tid = kpart * 32 + lane;
    for (int e = tid; e < 16 * MC; e += wpt * 32) {
      const int row = e / MC, m = e - row * MC;
      if (row >= nrows || m >= p.M) continue;
      float v = 0.f;
      for (int w = 0; w < wpt; ++w) v += sred[(w * 16 + row) * MC + m];
      const int orow = row0 + row;
      if (p.bias) v += __bfloat162float(__ushort_as_bfloat16(p.bias[orow]));
      emit_out(p, tag, m, orow, v);
    }
    if constexpr (C::kRedBufs == 1) named_barrier(1 + slot, wpt * 32);  // reads done before the next round's writes
  }
  cp_async_wait<0>();
}

// Weight materialisation through the same decode path: fragments stored
// instead of fed to the tensor cores.  One warp per tile.
template <int D, int R, int IDW, bool REPL, int NUM>
__global__ void __launch_bounds__(kThreads) rvq_dequant_kernel(const __grid_constant__ GemvParams p, uint16_t* w,
                                                               long long ldw) {
  using C = GemvCfg<D, R, IDW, REPL, 1, 0>;
  using T = WT<(NUM & 4) != 0>;
  using L = typename C::L;
  constexpr int V = C::V;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q = lane & 3;
  const LaneSel ls(r, q, (NUM & 3) == kExactScaled && REPL && R > 1);
  int group, tb, te;
  cta_range(p, blockIdx.x, &group, &tb, &te);
  if (tb >= te) return;
  stage_codebooks<D, R, REPL, NUM>(smem, p.codebooks + (size_t)group * R * p.entries * D, p.entries,
                                  p.stage_scales ? p.stage_scales + (size_t)group * R : nullptr);
  __syncthreads();
  const uint32_t cb_s = smem_u32(smem);
  const uint32_t cbl = cb_s + L::lane_offset(r, q);
  const long long tile_bytes = (long long)p.chunks * V * 256;
  for (int t = tb + warp; t < te; t += kWarps) {
    const int4 ti = p.tiles[t];
    const uint32_t rho_a = r < ti.z ? T::rho2(p.row_scale[ti.y + r]) : 0u;
    const uint32_t rho_b = r + 8 < ti.z ? T::rho2(p.row_scale[ti.y + r + 8]) : 0u;
    const uint8_t* tbase = p.packed + (long long)t * tile_bytes;
    for (int c = 0; c < p.chunks; ++c) {
      uint32_t c0[V * 4], c1[V * 4];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const uint4 a = ldg_stream_v4(tbase + ((long long)c * V + v) * 256 + r * 16);
        const uint4 b = ldg_stream_v4(tbase + ((long long)c * V + v) * 256 + (r + 8) * 16);
        c0[4 * v] = a.x; c0[4 * v + 1] = a.y; c0[4 * v + 2] = a.z; c0[4 * v + 3] = a.w;
        c1[4 * v] = b.x; c1[4 * v + 1] = b.y; c1[4 * v + 2] = b.z; c1[4 * v + 3] = b.w;
      }
      static_for<0, D>([&](auto ktc) {
        constexpr int kt = decltype(ktc)::value;
        uint32_t ra[2], rb[2];
        decode_row<D, R, IDW, REPL, kt, C::NW, NUM>(ra, c0, cb_s, cbl, rho_a, ls);
        decode_row<D, R, IDW, REPL, kt, C::NW, NUM>(rb, c1, cb_s, cbl, rho_b, ls);
        const int col = c * kChunkBlocks * D + kt * 16 + 4 * q;
        if (col < p.K) {
          if (r < ti.z) *reinterpret_cast<uint2*>(w + (long long)(ti.y + r) * ldw + col) = make_uint2(ra[0], ra[1]);
          if (r + 8 < ti.z)
            *reinterpret_cast<uint2*>(w + (long long)(ti.y + r + 8) * ldw + col) = make_uint2(rb[0], rb[1]);
        }
      });
    }
  }
}

// Packed ids -> [R][N][blocks] (1- or 2-byte ids).  One thread per (tile row, block).
__global__ void rvq_unpack_kernel(const uint8_t* __restrict__ packed, const int4* __restrict__ tiles,
                                  long long num_tiles, int R, int idw, int blocks, int chunks, long long N,
                                  uint8_t* __restrict__ out) {
  const long long total = num_tiles * kTileRows * (long long)blocks;
  const int V = R * idw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / ((long long)kTileRows * blocks);
    const int rem = (int)(i - t * kTileRows * (long long)blocks);
    const int rr = rem / blocks, b = rem - rr * blocks;
    const int4 ti = tiles[t];
    if (rr >= ti.z) continue;
    const long long row = ti.y + rr;
    const int c = b / kChunkBlocks, j = b - c * kChunkBlocks;
    for (int s = 0; s < R; ++s) {
      const int byte_in_row = j * idw;
      const int v = s * idw + byte_in_row / 16;
      const uint8_t* src = packed + ((t * chunks + c) * V + v) * 256 + rr * 16 + byte_in_row % 16;
      uint8_t* dst = out + (((long long)s * N + row) * blocks + b) * idw;
      dst[0] = src[0];
      if (idw == 2) dst[1] = src[1];
    }
  }
}

// ---------------------------------------------------------------------------
// host-side dispatch
// ---------------------------------------------------------------------------
bool replicated(int d, int R, int entries) {
  if (entries > 256) return false;
  const int per_row = d == 32 ? 1 : 2;  // stages per 256-byte entry row
  return ((R + per_row - 1) / per_row) * 64 * 1024 <= 128 * 1024;
}

int check_layer(const wal_rvq_layer* L) {
  if (!L) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = L->geom;
  if (g.out_features <= 0 || g.in_features <= 0 || g.num_groups <= 0 || L->num_tiles <= 0) return WAL_ERR_SHAPE;
  if (g.block_size != 8 && g.block_size != 16 && g.block_size != 32) return WAL_ERR_UNSUPPORTED;
  if (g.num_stages < 1 || g.num_stages > 4) return WAL_ERR_UNSUPPORTED;
  if (g.num_entries < 1 || g.num_entries > 32767 || (g.num_stages > 1 && g.num_entries > 256))
    return WAL_ERR_UNSUPPORTED;
  if (g.in_features % 4 != 0) return WAL_ERR_UNSUPPORTED;
  if (g.num_groups > kMaxGroups) return WAL_ERR_UNSUPPORTED;
  if (L->sum_mode != WAL_SUM_EXACT && L->sum_mode != WAL_SUM_FAST) return WAL_ERR_INVALID_ARGUMENT;
  if (!L->packed_ids || !L->tile_table || !L->codebooks || !L->row_scale) return WAL_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)L->packed_ids & 15) || ((uintptr_t)L->tile_table & 15) || ((uintptr_t)L->codebooks & 15) ||
      ((uintptr_t)L->stage_scales & 3))
    return WAL_ERR_ALIGNMENT;
  return WAL_OK;
}

// Group boundaries along the tile table, from the host row counts.
int group_starts(const wal_rvq_layer* L, GemvParams* p) {
  const int G = L->geom.num_groups;
  if (G > kMaxGroups) return WAL_ERR_UNSUPPORTED;
  if (G > 1 && !L->group_rows) return WAL_ERR_INVALID_ARGUMENT;
  long long t = 0, rows = 0;
  p->group_tile_start[0] = 0;
  p->group_row_start[0] = 0;
  for (int g = 0; g < G; ++g) {
    const long long n = G == 1 ? L->geom.out_features : L->group_rows[g];
    if (n <= 0) return WAL_ERR_SHAPE;
    rows += n;
    t += (n + kTileRows - 1) / kTileRows;
    p->group_tile_start[g + 1] = (int)t;
    p->group_row_start[g + 1] = (int)rows;
  }
  if (t != L->num_tiles || rows != L->geom.out_features) return WAL_ERR_SHAPE;
  p->num_groups = G;
  return WAL_OK;
}

// Deal the grid's CTAs to groups in proportion to their tile counts (at least
// one each), and each group's tiles evenly over its CTAs.
void assign_ctas(GemvParams& p, int ctas) {
  const int G = p.num_groups;
  const long long T = p.group_tile_start[G];
  int assigned = 0;
  for (int g = 0; g < G; ++g) {
    long long cum = ((long long)ctas * p.group_tile_start[g + 1] + T / 2) / T;
    if (cum < g + 1) cum = g + 1;
    if (cum > ctas - (G - 1 - g)) cum = ctas - (G - 1 - g);
    if (g == G - 1) cum = ctas;
    const int n = (int)cum - assigned;
    const int tg = p.group_tile_start[g + 1] - p.group_tile_start[g];
    p.cta_start[g] = assigned;
    p.tiles_q[g] = tg / n;
    p.tiles_r[g] = tg % n;
    assigned = (int)cum;
  }
  p.cta_start[G] = ctas;
}

// Launch facts looked up once instead of on every call: per device its SM
// count; per (device, kernel) the shared-memory attributes, set again only
// for a larger size; per (device, kernel, threads, shared memory) the
// resident CTAs per SM.  These runtime queries took several microseconds per
// call, as long as a small layer's decode GEMV runs on the GPU.
struct KernelAttr {
  int dev;
  const void* fn;
  int smem;
};
struct KernelOcc {
  int dev;
  const void* fn;
  int threads, smem, per_sm;
};
constexpr int kMaxDevs = 64;
std::mutex g_launch_mu;
int g_sms[kMaxDevs];
std::vector<KernelAttr> g_attr;
std::vector<KernelOcc> g_occ;

int sm_count(int dev, int* sms) {
  if (dev < 0 || dev >= kMaxDevs) return WAL_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_launch_mu);
  if (g_sms[dev] == 0 && cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    g_sms[dev] = 0;
    return WAL_ERR_CUDA;
  }
  *sms = g_sms[dev];
  return WAL_OK;
}

template <typename Kern>
int launch_facts(Kern kern, int threads, int smem, int* sms, int* per_sm) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WAL_ERR_CUDA;
  int st = sm_count(dev, sms);
  if (st != WAL_OK) return st;
  const void* fn = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lk(g_launch_mu);
  KernelAttr* attr = nullptr;
  for (auto& a : g_attr)
    if (a.dev == dev && a.fn == fn) attr = &a;
  if (!attr || attr->smem < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return WAL_ERR_CUDA;
    if (attr) {
      attr->smem = smem;
    } else {
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      g_attr.push_back({dev, fn, smem});
    }
  }
  for (const auto& o : g_occ)
    if (o.dev == dev && o.fn == fn && o.threads == threads && o.smem == smem) {
      *per_sm = o.per_sm;
      return WAL_OK;
    }
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kern, threads, smem) != cudaSuccess) return WAL_ERR_CUDA;
  g_occ.push_back({dev, fn, threads, smem, *per_sm});
  return WAL_OK;
}

template <typename Kern>
int persistent_grid(Kern kern, int threads, int smem, int num_ctas, GemvParams& p, int* grid_out,
                    int* capacity_out = nullptr, bool pair_tiles = false) {
  int sms = 0, per_sm = 0;
  const int st = launch_facts(kern, threads, smem, &sms, &per_sm);
  if (st != WAL_OK) return st;
  if (per_sm < 1) return WAL_ERR_UNSUPPORTED;
  const long long capacity = (long long)sms * per_sm;
  long long grid = num_ctas > 0 ? num_ctas : capacity;
  if (grid > p.num_tiles) grid = p.num_tiles;
  // Two tiles per CTA at most: pair every CTA's tiles rather than leave some
  // CTAs one tile, so that the SMs left over are idle from the start and the
  // next kernel's prologue runs on them (8B o and down shapes, 256 tiles:
  // 128 CTAs 7.4 / 17.6 us against 148 CTAs 8.5 / 18.6 us; three or more
  // tiles per CTA measured no better packed).
  if (pair_tiles && num_ctas <= 0 && p.num_tiles > capacity && p.num_tiles <= 2 * capacity)
    grid = (p.num_tiles + 1) / 2;
  if (grid < p.num_groups) grid = p.num_groups;
  *grid_out = (int)grid;
  if (capacity_out) *capacity_out = (int)capacity;
  assign_ctas(p, (int)grid);
  return WAL_OK;
}

}  // namespace
}  // namespace wal

using namespace wal;

// Warps per tile for a CTA with tpc tiles: rounds of 16/wpt tiles, each round
// ceil(chunks/wpt) chunks, plus a small reduction cost per round growing with
// wpt.  For one n-tile of tokens, splits within 5% of the cheapest are ranked
// by the warps the first round keeps busy (8B gate/up at M = 1, 13 tiles per
// CTA: 2 warps per tile, 16 warps busy, 31.7 us against 33.2 us for one warp
// per tile, 13 warps busy; at M = 32 the same choice cost 61.3 against 54.9 us).
static int best_wpt(long long tpc, int chunks, int wmax, bool rank_busy) {
  double cost[5];
  long long busy[5];
  int n = 0;
  double best = 1e30;
  for (int w = 1; w <= wmax; w *= 2, ++n) {
    const long long slots = 16 / w;
    const long long rounds = (tpc + slots - 1) / slots;
    const long long cpw = (chunks + w - 1) / w;
    cost[n] = (double)rounds * ((double)cpw + 0.25 * (w > 1 ? 1 + w / 4.0 : 0.0));
    busy[n] = (tpc < slots ? tpc : slots) * w;
    if (cost[n] < best) best = cost[n];
  }
  int pick = -1;
  for (int i = 0; i < n; ++i)
    if (cost[i] <= (rank_busy ? best * 1.05 : best) + 1e-9 &&
        (pick < 0 || busy[i] > busy[pick] || (busy[i] == busy[pick] && cost[i] < cost[pick])))
      pick = i;
  return 1 << pick;
}

static int log2_pow2(int w) { return w == 1 ? 0 : w == 2 ? 1 : w == 4 ? 2 : w == 8 ? 3 : 4; }

template <int D, int R, int IDW, bool REPL, int MT, int XM, int NUM>
static int run_gemv(GemvParams p, int num_ctas, cudaStream_t stream) {
  using C = GemvCfg<D, R, IDW, REPL, MT, XM>;
  auto kern = rvq_gemv_kernel<D, R, IDW, REPL, MT, XM, NUM>;
  const int kpad = p.chunks * kChunkBlocks * D;
  int smem = C::smem(p.entries, p.M, kpad, p.wpt);
  if constexpr (XM == 2) {  // the window ring grows with wpt: choose among the splits that fit
    int wmax = 16;
    while (wmax > 1 && C::smem(p.entries, p.M, kpad, wmax) > 227 * 1024) wmax >>= 1;
    if (p.wpt > wmax) {
      p.wpt = p.auto_tpc > 0 ? best_wpt(p.auto_tpc, p.chunks, wmax, p.M <= 8) : wmax;
      p.wpt_shift = log2_pow2(p.wpt);
      smem = C::smem(p.entries, p.M, kpad, p.wpt);
    }
  }
  if (smem > 227 * 1024) return WAL_ERR_UNSUPPORTED;
  if (p.wpt > C::kW) return WAL_ERR_INVALID_ARGUMENT;
  int grid = 0, capacity = 0;
  const int st = persistent_grid(kern, C::kT, smem, num_ctas, p, &grid, &capacity, true);
  if (st != WAL_OK) return st;
  p.early_release = grid < capacity ? 1 : 0;
  // the in-kernel id cursor is a 32-bit offset over one CTA's tiles
  for (int g = 0; g < p.num_groups; ++g)
    if ((long long)(p.tiles_q[g] + 1) * p.chunks * C::V * 256 >= (1LL << 31)) return WAL_ERR_UNSUPPORTED;
  // programmatic dependent launch: the weight prologue (codebooks, first id
  // chunks) of this kernel overlaps the tail of the previous kernel in the
  // stream; the kernel waits on the dependency before touching x or y.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::kT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return WAL_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

template <int D, int R, int IDW, bool REPL, int NUM>
static int run_dequant(GemvParams p, uint16_t* w, long long ldw, cudaStream_t stream) {
  using C = GemvCfg<D, R, IDW, REPL, 1, 0>;
  auto kern = rvq_dequant_kernel<D, R, IDW, REPL, NUM>;
  const int smem = C::cb_bytes(p.entries);
  if (smem > 227 * 1024) return WAL_ERR_UNSUPPORTED;
  int grid = 0;
  const int st = persistent_grid(kern, kThreads, smem, 0, p, &grid);
  if (st != WAL_OK) return st;
  kern<<<grid, kThreads, smem, stream>>>(p, w, ldw);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

// mt: n-tiles of 8 tokens per launch (1, 2 or 4); xm: activation mode
// (1 staged whole, 2 window ring, 0 unstaged)
template <int D, int R, int IDW, bool REPL, int NUM>
static int run_mt(const GemvParams& p, int num_ctas, cudaStream_t stream, int mt, int xm) {
  if (mt == 1)
    return xm == 1 ? run_gemv<D, R, IDW, REPL, 1, 1, NUM>(p, num_ctas, stream)
                   : xm == 2 ? run_gemv<D, R, IDW, REPL, 1, 2, NUM>(p, num_ctas, stream)
                             : run_gemv<D, R, IDW, REPL, 1, 0, NUM>(p, num_ctas, stream);
  if (mt == 2)
    return xm == 1 ? run_gemv<D, R, IDW, REPL, 2, 1, NUM>(p, num_ctas, stream)
                   : xm == 2 ? run_gemv<D, R, IDW, REPL, 2, 2, NUM>(p, num_ctas, stream)
                             : run_gemv<D, R, IDW, REPL, 2, 0, NUM>(p, num_ctas, stream);
  // 32 rows of whole activations never fit
  return xm == 2 ? run_gemv<D, R, IDW, REPL, 4, 2, NUM>(p, num_ctas, stream)
                 : xm == 0 ? run_gemv<D, R, IDW, REPL, 4, 0, NUM>(p, num_ctas, stream) : WAL_ERR_UNSUPPORTED;
}

// Numerics mode of a launch: fast (stage tables rounded to the weight type and
// accumulated in it, stage scales folded into the staged table), exact with
// fp32 scaled multi-stage tables, or exact (one-stage tables fold their scale
// into the pre-rounding).
template <int D, int R, int IDW, bool F16>
static int dispatch_gemv(const GemvParams& p, int num_ctas, cudaStream_t stream, bool repl, int mt, int xm,
                         bool fast) {
  constexpr int kF = F16 ? 4 : 0;
  if (fast) {
    if constexpr (IDW == 1) {
      if (repl) return run_mt<D, R, IDW, true, kFast | kF>(p, num_ctas, stream, mt, xm);
    }
    return run_mt<D, R, IDW, false, kFast | kF>(p, num_ctas, stream, mt, xm);
  }
  if constexpr (IDW == 1 && R > 1) {
    if (p.stage_scales) {  // scaled multi-stage tables: fp32 replicated layout only
      if (!repl) return WAL_ERR_UNSUPPORTED;
      return run_mt<D, R, IDW, true, kExactScaled | kF>(p, num_ctas, stream, mt, xm);
    }
  }
  if constexpr (IDW == 1) {
    if (repl) return run_mt<D, R, IDW, true, kExact | kF>(p, num_ctas, stream, mt, xm);
  }
  return run_mt<D, R, IDW, false, kExact | kF>(p, num_ctas, stream, mt, xm);
}

template <int D, int R, int IDW, bool F16>
static int dispatch_dequant(const GemvParams& p, uint16_t* w, long long ldw, cudaStream_t stream, bool repl,
                            bool fast) {
  constexpr int kF = F16 ? 4 : 0;
  if (fast) {
    if constexpr (IDW == 1) {
      if (repl) return run_dequant<D, R, IDW, true, kFast | kF>(p, w, ldw, stream);
    }
    return run_dequant<D, R, IDW, false, kFast | kF>(p, w, ldw, stream);
  }
  if constexpr (IDW == 1 && R > 1) {
    if (p.stage_scales) {
      if (!repl) return WAL_ERR_UNSUPPORTED;
      return run_dequant<D, R, IDW, true, kExactScaled | kF>(p, w, ldw, stream);
    }
  }
  if constexpr (IDW == 1) {
    if (repl) return run_dequant<D, R, IDW, true, kExact | kF>(p, w, ldw, stream);
  }
  return run_dequant<D, R, IDW, false, kExact | kF>(p, w, ldw, stream);
}

// Per-(block size, weight type) dispatchers.  Each pair is compiled in its own
// translation unit (the build passes -DWAL_UNIT_D=8/16/32 and -DWAL_UNIT_T=0
// for bf16, 1 for fp16) so the kernel instantiations build in parallel; the C
// entry points are in the unit built with -DWAL_UNIT_API.
#define WAL_DECLARE_UNIT(d, t)                                                                                    \
  int wal_gemv_dispatch_d##d##_t##t(const GemvParams&, int, cudaStream_t, int, int, bool, int, int, bool);       \
  int wal_dequant_dispatch_d##d##_t##t(const GemvParams&, uint16_t*, long long, cudaStream_t, int, int, bool, bool);
// fp32 activations and weights (CUDA cores), in wal_rvq_f32.cu
int wal_rvq_gemv_f32_impl(const wal_rvq_layer* layer, const float* x, int64_t M, int64_t ldx, float* y, int64_t ldy,
                          cudaStream_t stream);
int wal_rvq_dequant_f32_impl(const wal_rvq_layer* layer, float* w, int64_t ldw, cudaStream_t stream);
WAL_DECLARE_UNIT(8, 0)
WAL_DECLARE_UNIT(16, 0)
WAL_DECLARE_UNIT(32, 0)
WAL_DECLARE_UNIT(8, 1)
WAL_DECLARE_UNIT(16, 1)
WAL_DECLARE_UNIT(32, 1)

#ifdef WAL_UNIT_D
#define WAL_CAT2(a, b, c, d) a##b##c##d
#define WAL_CAT(a, b, c, d) WAL_CAT2(a, b, c, d)
int WAL_CAT(wal_gemv_dispatch_d, WAL_UNIT_D, _t, WAL_UNIT_T)(const GemvParams& p, int num_ctas, cudaStream_t s, int R,
                                                            int idw, bool repl, int mt, int xs, bool fast) {
  constexpr int D = WAL_UNIT_D;
  constexpr bool F16 = WAL_UNIT_T != 0;
  switch (R * 10 + idw) {
    case 11: return dispatch_gemv<D, 1, 1, F16>(p, num_ctas, s, repl, mt, xs, fast);
    case 12: return dispatch_gemv<D, 1, 2, F16>(p, num_ctas, s, repl, mt, xs, fast);
    case 21: return dispatch_gemv<D, 2, 1, F16>(p, num_ctas, s, repl, mt, xs, fast);
    case 31: return dispatch_gemv<D, 3, 1, F16>(p, num_ctas, s, repl, mt, xs, fast);
    case 41: return dispatch_gemv<D, 4, 1, F16>(p, num_ctas, s, repl, mt, xs, fast);
    default: return WAL_ERR_UNSUPPORTED;
  }
}
int WAL_CAT(wal_dequant_dispatch_d, WAL_UNIT_D, _t, WAL_UNIT_T)(const GemvParams& p, uint16_t* w, long long ldw,
                                                               cudaStream_t s, int R, int idw, bool repl, bool fast) {
  constexpr int D = WAL_UNIT_D;
  constexpr bool F16 = WAL_UNIT_T != 0;
  switch (R * 10 + idw) {
    case 11: return dispatch_dequant<D, 1, 1, F16>(p, w, ldw, s, repl, fast);
    case 12: return dispatch_dequant<D, 1, 2, F16>(p, w, ldw, s, repl, fast);
    case 21: return dispatch_dequant<D, 2, 1, F16>(p, w, ldw, s, repl, fast);
    case 31: return dispatch_dequant<D, 3, 1, F16>(p, w, ldw, s, repl, fast);
    case 41: return dispatch_dequant<D, 4, 1, F16>(p, w, ldw, s, repl, fast);
    default: return WAL_ERR_UNSUPPORTED;
  }
}
#endif  // WAL_UNIT_D

#ifdef WAL_UNIT_API
static int gemv_by_d(int d, bool f16, const GemvParams& p, int num_ctas, cudaStream_t s, int R, int idw, bool repl,
                     int mt, int xs, bool fast) {
  if (d == 8) return (f16 ? wal_gemv_dispatch_d8_t1 : wal_gemv_dispatch_d8_t0)(p, num_ctas, s, R, idw, repl, mt, xs, fast);
  if (d == 16)
    return (f16 ? wal_gemv_dispatch_d16_t1 : wal_gemv_dispatch_d16_t0)(p, num_ctas, s, R, idw, repl, mt, xs, fast);
  if (d == 32)
    return (f16 ? wal_gemv_dispatch_d32_t1 : wal_gemv_dispatch_d32_t0)(p, num_ctas, s, R, idw, repl, mt, xs, fast);
  return WAL_ERR_UNSUPPORTED;
}

static int dequant_by_d(int d, bool f16, const GemvParams& p, uint16_t* w, long long ldw, cudaStream_t s, int R,
                        int idw, bool repl, bool fast) {
  if (d == 8) return (f16 ? wal_dequant_dispatch_d8_t1 : wal_dequant_dispatch_d8_t0)(p, w, ldw, s, R, idw, repl, fast);
  if (d == 16)
    return (f16 ? wal_dequant_dispatch_d16_t1 : wal_dequant_dispatch_d16_t0)(p, w, ldw, s, R, idw, repl, fast);
  if (d == 32)
    return (f16 ? wal_dequant_dispatch_d32_t1 : wal_dequant_dispatch_d32_t0)(p, w, ldw, s, R, idw, repl, fast);
  return WAL_ERR_UNSUPPORTED;
}

static int make_params(const wal_rvq_layer* L, GemvParams* p) {
  *p = GemvParams{};
  const wal_rvq_geometry& g = L->geom;
  const long long blocks = (g.in_features + g.block_size - 1) / g.block_size;
  p->packed = static_cast<const uint8_t*>(L->packed_ids);
  p->tiles = reinterpret_cast<const int4*>(L->tile_table);
  p->codebooks = L->codebooks;
  p->row_scale = L->row_scale;
  p->bias = L->bias;
  p->stage_scales = L->stage_scales;
  p->num_tiles = L->num_tiles;
  p->K = (int)g.in_features;
  p->chunks = (int)((blocks + kChunkBlocks - 1) / kChunkBlocks);
  p->entries = g.num_entries;
  return group_starts(L, p);
}

// Shared body of the GEMV entry points; push == NULL writes y, otherwise the
// fp32 rows go to every rank's receive rows (y, ldy, y_dtype unused).
static int gemv_common(const wal_rvq_layer* layer, const void* xv, int x_dtype, int64_t M, int64_t ldx, void* y,
                       int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas, const wal_tp_push* push,
                       void* stream) {
  int st = check_layer(layer);
  if (st != WAL_OK) return st;
  if (!xv || (!y && !push)) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0) return WAL_ERR_SHAPE;
  if (x_dtype == WAL_F32) {  // fp32 activations: CUDA-core kernel with fp32 weights
    if (push) return WAL_ERR_UNSUPPORTED;
    if (y_dtype != WAL_F32) return WAL_ERR_INVALID_ARGUMENT;
    return wal_rvq_gemv_f32_impl(layer, static_cast<const float*>(xv), M, ldx, static_cast<float*>(y), ldy,
                                 static_cast<cudaStream_t>(stream));
  }
  if (x_dtype != WAL_BF16 && x_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  const bool f16 = x_dtype == WAL_F16, fast = layer->sum_mode == WAL_SUM_FAST;
  const uint16_t* x = static_cast<const uint16_t*>(xv);
  const wal_rvq_geometry& g = layer->geom;
  if (push) {
    if (push->num_ranks < 1 || push->num_ranks > WAL_MAX_RANKS || push->rank < 0 || push->rank >= push->num_ranks)
      return WAL_ERR_INVALID_ARGUMENT;
    if (!push->epoch) return WAL_ERR_INVALID_ARGUMENT;
    for (int r = 0; r < push->num_ranks; ++r) {
      if (!push->dst[r]) return WAL_ERR_INVALID_ARGUMENT;
      if ((uintptr_t)push->dst[r] & 7) return WAL_ERR_ALIGNMENT;
    }
    if (push->ld_dst < g.out_features) return WAL_ERR_SHAPE;
    ldy = g.out_features;
    y_dtype = WAL_F32;
  }
  if (ldx < g.in_features || ldy < g.out_features) return WAL_ERR_SHAPE;
  if ((ldx % 4) || ((uintptr_t)x & 7)) return WAL_ERR_ALIGNMENT;
  if (ldx >= (1LL << 26)) return WAL_ERR_UNSUPPORTED;  // activation row offsets are 32-bit
  if (y_dtype != WAL_BF16 && y_dtype != WAL_F32 && y_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  if (warps_per_tile != 0 && warps_per_tile != 1 && warps_per_tile != 2 && warps_per_tile != 4 &&
      warps_per_tile != 8 && warps_per_tile != 16)
    return WAL_ERR_INVALID_ARGUMENT;
  if (num_ctas < 0) return WAL_ERR_INVALID_ARGUMENT;
  const int d = g.block_size, R = g.num_stages, idw = g.num_entries <= 256 ? 1 : 2;
  const bool repl = replicated(d, R, g.num_entries);
  GemvParams p;
  st = make_params(layer, &p);
  if (st != WAL_OK) return st;
  int wpt = warps_per_tile;
  p.auto_tpc = 0;
  if (wpt == 0) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || sm_count(dev, &sms) != WAL_OK) return WAL_ERR_CUDA;
    const long long grid = layer->num_tiles < sms ? layer->num_tiles : sms;
    const long long tpc = (layer->num_tiles + grid - 1) / grid;  // tiles per CTA (max)
    wpt = best_wpt(tpc, p.chunks, 16, M <= 8);
    p.auto_tpc = (int)tpc;
  }
  p.wpt = wpt;
  p.wpt_shift = log2_pow2(wpt);
  p.ldx = ldx;
  p.ldy = ldy;
  p.y_dtype = y_dtype;
  p.pdl = 1;
  if (push) {
    p.push_ranks = push->num_ranks;
    p.push_ld = push->ld_dst;
    p.push_epoch = push->epoch;
    p.bias = nullptr;  // partial sums of a row-parallel split carry no bias
  }
  const size_t ysz = y_dtype == WAL_F32 ? 4 : 2;
  const int kpad = p.chunks * kChunkBlocks * d;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // slabs of up to 32 tokens; a slab whose n-tiles do not fit in shared memory
  // (large multi-stage codebooks) runs as two slabs of half the tokens
  int cap = kMaxTokens;
  for (int64_t m0 = 0; m0 < M;) {
    const int mm = (int)((M - m0) < cap ? (M - m0) : cap);
    p.x = x + m0 * ldx;
    if (push) {
      for (int r = 0; r < push->num_ranks; ++r) p.push_dst[r] = static_cast<uint2*>(push->dst[r]) + m0 * push->ld_dst;
    } else {
      p.y = static_cast<uint8_t*>(y) + (size_t)(m0 * ldy) * ysz;
    }
    p.M = mm;
    const int mt = mm <= 8 ? 1 : (mm <= 16 ? 2 : 4);
    // whole activations when small, else the window ring, else (shared memory
    // taken by a large codebook) unstaged reads
    int xm = mt < 4 && (long long)mm * kpad * 2 <= kXSmemBudget ? 1 : 2;
    int rs = gemv_by_d(d, f16, p, num_ctas, s, R, idw, repl, mt, xm, fast);
    if (rs == WAL_ERR_UNSUPPORTED && xm == 1) rs = gemv_by_d(d, f16, p, num_ctas, s, R, idw, repl, mt, xm = 2, fast);
    if (rs == WAL_ERR_UNSUPPORTED && xm == 2) rs = gemv_by_d(d, f16, p, num_ctas, s, R, idw, repl, mt, 0, fast);
    if (rs == WAL_ERR_UNSUPPORTED && mt > 1) {
      cap = mt == 4 ? 16 : 8;
      continue;
    }
    if (rs != WAL_OK) return rs;
    m0 += mm;
  }
  return WAL_OK;
}

extern "C" int wal_rvq_gemv_typed(const wal_rvq_layer* layer, const void* x, int x_dtype, int64_t M, int64_t ldx,
                                  void* y, int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas, void* stream) {
  return gemv_common(layer, x, x_dtype, M, ldx, y, ldy, y_dtype, warps_per_tile, num_ctas, nullptr, stream);
}

extern "C" int wal_rvq_gemv_ex(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                               int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas, void* stream) {
  return gemv_common(layer, x, WAL_BF16, M, ldx, y, ldy, y_dtype, warps_per_tile, num_ctas, nullptr, stream);
}

extern "C" int wal_rvq_gemv(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                            int64_t ldy, int y_dtype, void* stream) {
  return gemv_common(layer, x, WAL_BF16, M, ldx, y, ldy, y_dtype, 0, 0, nullptr, stream);
}

extern "C" int wal_rvq_gemv_push(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                                 const wal_tp_push* push, void* stream) {
  if (!push) return WAL_ERR_INVALID_ARGUMENT;
  return gemv_common(layer, x, WAL_BF16, M, ldx, nullptr, 0, WAL_F32, 0, 0, push, stream);
}

extern "C" int wal_rvq_dequant_typed(const wal_rvq_layer* layer, void* w, int64_t ldw, int w_dtype, void* stream) {
  int st = check_layer(layer);
  if (st != WAL_OK) return st;
  if (!w) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = layer->geom;
  if (ldw < g.in_features) return WAL_ERR_SHAPE;
  if (w_dtype == WAL_F32) {
    if ((uintptr_t)w & 3) return WAL_ERR_ALIGNMENT;
    return wal_rvq_dequant_f32_impl(layer, static_cast<float*>(w), ldw, static_cast<cudaStream_t>(stream));
  }
  if (w_dtype != WAL_BF16 && w_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  if ((ldw % 4) || ((uintptr_t)w & 7)) return WAL_ERR_ALIGNMENT;
  const int d = g.block_size, R = g.num_stages, idw = g.num_entries <= 256 ? 1 : 2;
  const bool repl = replicated(d, R, g.num_entries);
  GemvParams p;
  st = make_params(layer, &p);
  if (st != WAL_OK) return st;
  p.wpt = 1;
  p.wpt_shift = 0;
  return dequant_by_d(d, w_dtype == WAL_F16, p, static_cast<uint16_t*>(w), ldw, static_cast<cudaStream_t>(stream), R,
                      idw, repl, layer->sum_mode == WAL_SUM_FAST);
}

extern "C" int wal_rvq_dequant(const wal_rvq_layer* layer, uint16_t* w, int64_t ldw, void* stream) {
  return wal_rvq_dequant_typed(layer, w, ldw, WAL_BF16, stream);
}

extern "C" int wal_rvq_unpack_ids(const wal_rvq_layer* layer, void* ids, void* stream) {
  int st = check_layer(layer);
  if (st != WAL_OK) return st;
  if (!ids) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = layer->geom;
  const int idw = g.num_entries <= 256 ? 1 : 2;
  const int blocks = (int)((g.in_features + g.block_size - 1) / g.block_size);
  const int chunks = (blocks + kChunkBlocks - 1) / kChunkBlocks;
  const long long total = layer->num_tiles * kTileRows * (long long)blocks;
  long long grid = (total + 255) / 256;
  if (grid > 65535) grid = 65535;
  rvq_unpack_kernel<<<(int)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(layer->packed_ids), reinterpret_cast<const int4*>(layer->tile_table),
      layer->num_tiles, g.num_stages, idw, blocks, chunks, g.out_features, static_cast<uint8_t*>(ids));
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}
#endif  // WAL_UNIT_API
