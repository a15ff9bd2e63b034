// Decode-time fused gather-GEMV (M <= 16 tokens), weight materialisation and
// packed-id unpacking for the Block-RVQ runtime linear.
//
// GEMV structure (one persistent wave of CTAs, 8 warps each):
//   * a CTA owns a contiguous range of 16-row tiles and stages the codebooks
//     of the tile's row group in shared memory (restaged only when the group
//     changes);
//   * each tile's 16-block chunks are split over `wpt` warps (K split); a warp
//     streams its chunks' ids from HBM with 16-byte no-allocate loads
//     (prefetching the next chunk), decodes every weight exactly in registers
//     and feeds mma.sync m16n8k16 (bf16, fp32 accumulate) with the activation
//     fragment, so the dense weight never exists;
//   * the partial sums of the wpt warps are reduced in shared memory in a
//     fixed order, the bias is added in fp32 and y is written once.
// Replaces reference src/runtime.py:1501-1507 (reconstruct + F.linear) and the
// fused Triton kernel src/triton_id_matmul.py:143-217.
#include "../../include/wal_rvq.h"
#include "wal_rvq_decode.cuh"

#include <cstdio>
#include <type_traits>

namespace wal {
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

struct GemvParams {
  const uint8_t* packed;
  const int4* tiles;
  const uint16_t* codebooks;
  const uint16_t* row_scale;
  const uint16_t* bias;
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
};

__device__ __forceinline__ void store_out(void* y, long long idx, float v, int dtype) {
  if (dtype == WAL_F32) {
    static_cast<float*>(y)[idx] = v;
  } else if (dtype == WAL_BF16) {
    static_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(y)[idx] = __float2half_rn(v);
  }
}

// Process one chunk of one tile for one warp: D k-tiles of 16 columns.
template <int D, int R, int IDW, bool REPL, int MT, bool MASK>
__device__ __forceinline__ void gemv_chunk(float (&acc)[2][MT][4], const uint32_t (&c0)[R * IDW * 4],
                                           const uint32_t (&c1)[R * IDW * 4], uint32_t cb_base, int stage_bytes,
                                           uint32_t rho_a, uint32_t rho_b, int qh_shift, const uint16_t* xrow0,
                                           const uint16_t* xrow1, bool xv0, bool xv1, int col_base, int K) {
  constexpr int V = R * IDW;
  static_for<0, D>([&](auto ktc) {
    constexpr int kt = decltype(ktc)::value;
    uint32_t ra[2], rb[2];
    decode_row<D, R, IDW, REPL, kt, V>(ra, c0, cb_base, stage_bytes, rho_a, qh_shift);
    decode_row<D, R, IDW, REPL, kt, V>(rb, c1, cb_base, stage_bytes, rho_b, qh_shift);
    const int col = col_base + kt * 16;  // lane's first physical column (includes 4q)
    uint2 xa = make_uint2(0u, 0u), xb = make_uint2(0u, 0u);
    const bool in_k = !MASK || col < K;
    if (xv0 && in_k) xa = __ldg(reinterpret_cast<const uint2*>(xrow0 + col));
    if (MT == 2 && xv1 && in_k) xb = __ldg(reinterpret_cast<const uint2*>(xrow1 + col));
    uint32_t a[4] = {ra[0], rb[0], ra[1], rb[1]};
    if (MASK && !in_k) {
      a[0] = a[1] = a[2] = a[3] = 0u;
    }
    // even and odd k-tiles feed separate accumulators: two independent MMA chains
    mma_bf16_16816(acc[kt & 1][0], a, xa.x, xa.y);
    if (MT == 2) mma_bf16_16816(acc[kt & 1][MT - 1], a, xb.x, xb.y);
  });
}

template <int D, int R, int IDW, bool REPL, int MT>
__global__ void __launch_bounds__(kThreads) rvq_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  using L = CbLayout<D, REPL>;
  constexpr int V = R * IDW;
  const int sb = L::stage_bytes(p.entries);
  uint8_t* cb = smem;
  float* red = reinterpret_cast<float*>(smem + R * sb);  // [kWarps][16][MT*8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q = lane & 3;
  const int wpt = p.wpt;
  const int slots = kWarps / wpt;
  const int slot = warp / wpt, kpart = warp - slot * wpt;
  const int qh_shift = 8 * (q >> 1);
  const uint32_t cb_base = smem_u32(cb) + L::lane_offset(r, q);
  // first physical column of this lane inside a chunk's first k-tile (for d = 8
  // this is block q>>1, piece q&1: 8*(q>>1) + 4*(q&1) = 4q)
  const int lane_col = 4 * q;
  const long long tile_bytes = (long long)p.chunks * V * 256;
  const long long G = gridDim.x;
  const long long t_begin = (p.num_tiles * blockIdx.x) / G;
  const long long t_end = (p.num_tiles * (blockIdx.x + 1)) / G;
  const int m0 = r, m1 = 8 + r;
  const bool xv0 = m0 < p.M, xv1 = (MT == 2) && (m1 < p.M);
  const uint16_t* xrow0 = p.x + (long long)(xv0 ? m0 : 0) * p.ldx;
  const uint16_t* xrow1 = p.x + (long long)(xv1 ? m1 : 0) * p.ldx;
  const int kpad = p.chunks * kChunkBlocks * D;
  const bool need_mask = kpad != p.K;

  int cur_group = -1;
  long long t = t_begin;
  while (t < t_end) {
    const int g = p.tiles[t].x;
    if (g != cur_group) {
      __syncthreads();
      stage_codebooks<D, R, REPL>(cb, p.codebooks + (size_t)g * R * p.entries * D, p.entries);
      __syncthreads();
      cur_group = g;
    }
    int n_here = 1;
    while (n_here < slots && t + n_here < t_end && p.tiles[t + n_here].x == g) ++n_here;
    const long long my_t = t + slot;
    const bool active = slot < n_here;
    float acc[2][MT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < MT; ++i) acc[h][i][0] = acc[h][i][1] = acc[h][i][2] = acc[h][i][3] = 0.f;
    int4 ti = make_int4(0, 0, 0, 0);
    if (active) {
      ti = p.tiles[my_t];
      const int row0 = ti.y, nrows = ti.z;
      const uint32_t rho_a = r < nrows ? rho_pair(p.row_scale[row0 + r]) : 0u;
      const uint32_t rho_b = r + 8 < nrows ? rho_pair(p.row_scale[row0 + r + 8]) : 0u;
      const uint8_t* tbase = p.packed + my_t * tile_bytes;
      uint32_t cur0[V * 4], cur1[V * 4], nxt0[V * 4], nxt1[V * 4];
      int c = kpart;
      if (c < p.chunks) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const uint4 a = ldg_stream_v4(tbase + ((long long)c * V + v) * 256 + r * 16);
          const uint4 b = ldg_stream_v4(tbase + ((long long)c * V + v) * 256 + (r + 8) * 16);
          cur0[4 * v] = a.x; cur0[4 * v + 1] = a.y; cur0[4 * v + 2] = a.z; cur0[4 * v + 3] = a.w;
          cur1[4 * v] = b.x; cur1[4 * v + 1] = b.y; cur1[4 * v + 2] = b.z; cur1[4 * v + 3] = b.w;
        }
      }
      for (; c < p.chunks; c += wpt) {
        const int cn = c + wpt;
        if (cn < p.chunks) {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const uint4 a = ldg_stream_v4(tbase + ((long long)cn * V + v) * 256 + r * 16);
            const uint4 b = ldg_stream_v4(tbase + ((long long)cn * V + v) * 256 + (r + 8) * 16);
            nxt0[4 * v] = a.x; nxt0[4 * v + 1] = a.y; nxt0[4 * v + 2] = a.z; nxt0[4 * v + 3] = a.w;
            nxt1[4 * v] = b.x; nxt1[4 * v + 1] = b.y; nxt1[4 * v + 2] = b.z; nxt1[4 * v + 3] = b.w;
          }
        }
        const int col_base = c * kChunkBlocks * D + lane_col;
        if (need_mask && c == p.chunks - 1) {
          gemv_chunk<D, R, IDW, REPL, MT, true>(acc, cur0, cur1, cb_base, sb, rho_a, rho_b, qh_shift, xrow0, xrow1,
                                                xv0, xv1, col_base, p.K);
        } else {
          gemv_chunk<D, R, IDW, REPL, MT, false>(acc, cur0, cur1, cb_base, sb, rho_a, rho_b, qh_shift, xrow0,
                                                 xrow1, xv0, xv1, col_base, p.K);
        }
        if (cn < p.chunks) {
#pragma unroll
          for (int i = 0; i < V * 4; ++i) {
            cur0[i] = nxt0[i];
            cur1[i] = nxt1[i];
          }
        }
      }
    }
    // partial sums -> shared memory: red[warp][row][m]
    constexpr int MC = MT * 8;
    float* wred = red + warp * 16 * MC;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      wred[r * MC + i * 8 + 2 * q] = acc[0][i][0] + acc[1][i][0];
      wred[r * MC + i * 8 + 2 * q + 1] = acc[0][i][1] + acc[1][i][1];
      wred[(r + 8) * MC + i * 8 + 2 * q] = acc[0][i][2] + acc[1][i][2];
      wred[(r + 8) * MC + i * 8 + 2 * q + 1] = acc[0][i][3] + acc[1][i][3];
    }
    __syncthreads();
    const int per_slot = 16 * MC;
    for (int e = threadIdx.x; e < n_here * per_slot; e += kThreads) {
      const int s = e / per_slot;
      const int rem = e - s * per_slot;
      const int row = rem / MC, m = rem - row * MC;
      const int4 tt = p.tiles[t + s];
      if (row >= tt.z || m >= p.M) continue;
      float v = 0.f;
      for (int w = 0; w < wpt; ++w) v += red[((s * wpt + w) * 16 + row) * MC + m];
      const int orow = tt.y + row;
      if (p.bias) v += __bfloat162float(__ushort_as_bfloat16(p.bias[orow]));
      store_out(p.y, (long long)m * p.ldy + orow, v, p.y_dtype);
    }
    __syncthreads();
    t += n_here;
  }
}

// Weight materialisation: same decode path, fragments stored instead of fed
// to the tensor cores.  One warp per tile, all chunks.
template <int D, int R, int IDW, bool REPL>
__global__ void __launch_bounds__(kThreads) rvq_dequant_kernel(GemvParams p, uint16_t* w, long long ldw) {
  extern __shared__ __align__(128) uint8_t smem[];
  using L = CbLayout<D, REPL>;
  constexpr int V = R * IDW;
  const int sb = L::stage_bytes(p.entries);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q = lane & 3;
  const int qh_shift = 8 * (q >> 1);
  const uint32_t cb_base = smem_u32(smem) + L::lane_offset(r, q);
  const long long tile_bytes = (long long)p.chunks * V * 256;
  const long long G = gridDim.x;
  const long long t_begin = (p.num_tiles * blockIdx.x) / G;
  const long long t_end = (p.num_tiles * (blockIdx.x + 1)) / G;
  int cur_group = -1;
  long long t = t_begin;
  while (t < t_end) {
    const int g = p.tiles[t].x;
    if (g != cur_group) {
      __syncthreads();
      stage_codebooks<D, R, REPL>(smem, p.codebooks + (size_t)g * R * p.entries * D, p.entries);
      __syncthreads();
      cur_group = g;
    }
    int n_here = 1;
    while (n_here < kWarps && t + n_here < t_end && p.tiles[t + n_here].x == g) ++n_here;
    if (warp < n_here) {
      const long long my_t = t + warp;
      const int4 ti = p.tiles[my_t];
      const uint32_t rho_a = r < ti.z ? rho_pair(p.row_scale[ti.y + r]) : 0u;
      const uint32_t rho_b = r + 8 < ti.z ? rho_pair(p.row_scale[ti.y + r + 8]) : 0u;
      const uint8_t* tbase = p.packed + my_t * tile_bytes;
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
          decode_row<D, R, IDW, REPL, kt, V>(ra, c0, cb_base, sb, rho_a, qh_shift);
          decode_row<D, R, IDW, REPL, kt, V>(rb, c1, cb_base, sb, rho_b, qh_shift);
          const int col = c * kChunkBlocks * D + kt * 16 + 4 * q;
          if (col < p.K) {
            if (r < ti.z) *reinterpret_cast<uint2*>(w + (long long)(ti.y + r) * ldw + col) = make_uint2(ra[0], ra[1]);
            if (r + 8 < ti.z)
              *reinterpret_cast<uint2*>(w + (long long)(ti.y + r + 8) * ldw + col) = make_uint2(rb[0], rb[1]);
          }
        });
      }
    }
    t += n_here;
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
  const int copies = d == 8 ? 8 : 4;
  return (long long)R * entries * d * 2 * copies <= 160 * 1024;
}

int smem_bytes(int d, int R, int entries, bool repl, int mt) {
  const int copies = repl ? (d == 8 ? 8 : 4) : 1;
  return R * entries * d * 2 * copies + kWarps * 16 * mt * 8 * 4;
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
  if (!L->packed_ids || !L->tile_table || !L->codebooks || !L->row_scale) return WAL_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)L->packed_ids & 15) || ((uintptr_t)L->tile_table & 15) || ((uintptr_t)L->codebooks & 15))
    return WAL_ERR_ALIGNMENT;
  const bool repl = replicated(g.block_size, g.num_stages, g.num_entries);
  if (smem_bytes(g.block_size, g.num_stages, g.num_entries, repl, 2) > 227 * 1024) return WAL_ERR_UNSUPPORTED;
  return WAL_OK;
}

// Grid of one persistent wave: SMs x resident CTAs per SM, capped by the tile count.
template <typename Kern>
int persistent_grid(Kern kern, int smem, int num_ctas, long long num_tiles, int* grid_out) {
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WAL_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return WAL_ERR_CUDA;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  if (per_sm < 1) return WAL_ERR_UNSUPPORTED;
  long long grid = num_ctas > 0 ? num_ctas : (long long)sms * per_sm;
  if (grid > num_tiles) grid = num_tiles;
  if (grid < 1) grid = 1;
  *grid_out = (int)grid;
  return WAL_OK;
}

}  // namespace
}  // namespace wal

using namespace wal;

template <int D, int R, int IDW, bool REPL, int MT>
static int run_gemv(const GemvParams& p, int num_ctas, cudaStream_t stream, int entries) {
  auto kern = rvq_gemv_kernel<D, R, IDW, REPL, MT>;
  const int smem = smem_bytes(D, R, entries, REPL, MT);
  int grid = 0;
  const int st = persistent_grid(kern, smem, num_ctas, p.num_tiles, &grid);
  if (st != WAL_OK) return st;
  kern<<<grid, kThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

template <int D, int R, int IDW, bool REPL>
static int run_dequant(const GemvParams& p, uint16_t* w, long long ldw, cudaStream_t stream, int entries) {
  auto kern = rvq_dequant_kernel<D, R, IDW, REPL>;
  const int smem = smem_bytes(D, R, entries, REPL, 1);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WAL_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return WAL_ERR_CUDA;
  long long grid = (p.num_tiles + kWarps - 1) / kWarps;
  if (grid > 4LL * sms) grid = 4LL * sms;
  kern<<<(int)grid, kThreads, smem, stream>>>(p, w, ldw);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

template <int D, int R, int IDW>
static int dispatch_gemv(const GemvParams& p, int num_ctas, cudaStream_t stream, int entries, bool repl, int mt) {
  if (repl) {
    if constexpr (IDW == 1) {
      return mt == 1 ? run_gemv<D, R, IDW, true, 1>(p, num_ctas, stream, entries)
                     : run_gemv<D, R, IDW, true, 2>(p, num_ctas, stream, entries);
    }
  }
  return mt == 1 ? run_gemv<D, R, IDW, false, 1>(p, num_ctas, stream, entries)
                 : run_gemv<D, R, IDW, false, 2>(p, num_ctas, stream, entries);
}

template <int D, int R, int IDW>
static int dispatch_dequant(const GemvParams& p, uint16_t* w, long long ldw, cudaStream_t stream, int entries,
                            bool repl) {
  if (repl) {
    if constexpr (IDW == 1) return run_dequant<D, R, IDW, true>(p, w, ldw, stream, entries);
  }
  return run_dequant<D, R, IDW, false>(p, w, ldw, stream, entries);
}

#define WAL_FOR_ALL_CONFIGS(FN, ...)                                                    \
  switch (d * 100 + R * 10 + idw) {                                                    \
    case 811: return FN<8, 1, 1>(__VA_ARGS__);                                          \
    case 812: return FN<8, 1, 2>(__VA_ARGS__);                                          \
    case 821: return FN<8, 2, 1>(__VA_ARGS__);                                          \
    case 831: return FN<8, 3, 1>(__VA_ARGS__);                                          \
    case 841: return FN<8, 4, 1>(__VA_ARGS__);                                          \
    case 1611: return FN<16, 1, 1>(__VA_ARGS__);                                        \
    case 1612: return FN<16, 1, 2>(__VA_ARGS__);                                        \
    case 1621: return FN<16, 2, 1>(__VA_ARGS__);                                        \
    case 1631: return FN<16, 3, 1>(__VA_ARGS__);                                        \
    case 1641: return FN<16, 4, 1>(__VA_ARGS__);                                        \
    case 3211: return FN<32, 1, 1>(__VA_ARGS__);                                        \
    case 3212: return FN<32, 1, 2>(__VA_ARGS__);                                        \
    case 3221: return FN<32, 2, 1>(__VA_ARGS__);                                        \
    case 3231: return FN<32, 3, 1>(__VA_ARGS__);                                        \
    case 3241: return FN<32, 4, 1>(__VA_ARGS__);                                        \
    default: return WAL_ERR_UNSUPPORTED;                                                \
  }

static GemvParams make_params(const wal_rvq_layer* L) {
  GemvParams p{};
  const wal_rvq_geometry& g = L->geom;
  const long long blocks = (g.in_features + g.block_size - 1) / g.block_size;
  p.packed = static_cast<const uint8_t*>(L->packed_ids);
  p.tiles = reinterpret_cast<const int4*>(L->tile_table);
  p.codebooks = L->codebooks;
  p.row_scale = L->row_scale;
  p.bias = L->bias;
  p.num_tiles = L->num_tiles;
  p.K = (int)g.in_features;
  p.chunks = (int)((blocks + kChunkBlocks - 1) / kChunkBlocks);
  p.entries = g.num_entries;
  return p;
}

extern "C" int wal_rvq_gemv_ex(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                               int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas, void* stream) {
  int st = check_layer(layer);
  if (st != WAL_OK) return st;
  if (!x || !y) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0) return WAL_ERR_SHAPE;
  const wal_rvq_geometry& g = layer->geom;
  if (ldx < g.in_features || ldy < g.out_features) return WAL_ERR_SHAPE;
  if ((ldx % 4) || ((uintptr_t)x & 7)) return WAL_ERR_ALIGNMENT;
  if (y_dtype != WAL_BF16 && y_dtype != WAL_F32 && y_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  if (warps_per_tile != 0 && warps_per_tile != 1 && warps_per_tile != 2 && warps_per_tile != 4 &&
      warps_per_tile != 8)
    return WAL_ERR_INVALID_ARGUMENT;
  if (num_ctas < 0) return WAL_ERR_INVALID_ARGUMENT;
  const int d = g.block_size, R = g.num_stages, idw = g.num_entries <= 256 ? 1 : 2;
  const bool repl = replicated(d, R, g.num_entries);
  GemvParams p = make_params(layer);
  int wpt = warps_per_tile;
  if (wpt == 0) {
    // enough (tile, warp) work units to fill every SM with several warps
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    wpt = 1;
    while (wpt < kWarps && layer->num_tiles * wpt < (long long)sms * 16 && wpt * 2 <= p.chunks) wpt *= 2;
  }
  p.wpt = wpt;
  p.ldx = ldx;
  p.ldy = ldy;
  p.y_dtype = y_dtype;
  const size_t ysz = y_dtype == WAL_F32 ? 4 : 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int64_t m0 = 0; m0 < M; m0 += 16) {
    const int mm = (int)((M - m0) < 16 ? (M - m0) : 16);
    p.x = x + m0 * ldx;
    p.y = static_cast<uint8_t*>(y) + (size_t)(m0 * ldy) * ysz;
    p.M = mm;
    const int mt = mm <= 8 ? 1 : 2;
    auto run = [&]() -> int { WAL_FOR_ALL_CONFIGS(dispatch_gemv, p, num_ctas, s, g.num_entries, repl, mt) };
    const int rs = run();
    if (rs != WAL_OK) return rs;
  }
  return WAL_OK;
}

extern "C" int wal_rvq_gemv(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                            int64_t ldy, int y_dtype, void* stream) {
  return wal_rvq_gemv_ex(layer, x, M, ldx, y, ldy, y_dtype, 0, 0, stream);
}

extern "C" int wal_rvq_dequant(const wal_rvq_layer* layer, uint16_t* w, int64_t ldw, void* stream) {
  int st = check_layer(layer);
  if (st != WAL_OK) return st;
  if (!w) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = layer->geom;
  if (ldw < g.in_features) return WAL_ERR_SHAPE;
  if ((ldw % 4) || ((uintptr_t)w & 7)) return WAL_ERR_ALIGNMENT;
  const int d = g.block_size, R = g.num_stages, idw = g.num_entries <= 256 ? 1 : 2;
  const bool repl = replicated(d, R, g.num_entries);
  GemvParams p = make_params(layer);
  p.wpt = 1;
  WAL_FOR_ALL_CONFIGS(dispatch_dequant, p, w, ldw, static_cast<cudaStream_t>(stream), g.num_entries, repl)
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
