// fp32 activations: the reference's forward in torch.float32 builds an fp32
// weight, w = (sum_s fp32(C_s[id]) [* fp32 stage scale]) * fp32(rho) with one
// fp32 rounding per operation (src/runtime.py:379-414 with out_dtype float32),
// and multiplies in fp32 (src/runtime.py:1501-1507).  Tensor cores have no
// fp32 x fp32 product of that precision, so this path decodes each weight
// exactly in fp32 and accumulates with fp32 fused multiply-adds on the CUDA
// cores; it serves the rare fp32 caller correctly rather than fast.
//
// One warp per 16-row tile: lane (row = lane & 15, half = lane >> 4) decodes
// blocks 8 * half .. 8 * half + 7 of every 16-block chunk of its row (one
// 8-byte id load per stage, or one 16-byte load of 2-byte ids) and keeps one
// fp32 accumulator per token; the two halves are added with one shuffle.
// Codebooks are read through the read-only data cache (small per layer).
#include "../../include/wal_rvq.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kWarps = 8;
constexpr int kTokens = 8;  // tokens per launch (more run as slabs)

struct F32Params {
  const uint8_t* packed;
  const int4* tiles;  // group, first row, rows, 0
  const uint16_t* codebooks;
  const uint16_t* row_scale;
  const uint16_t* bias;
  const float* stage_scales;
  long long num_tiles;
  int K, d, R, idw, chunks, entries, fast;
  // GEMV
  const float* x;
  long long ldx;
  float* y;
  long long ldy;
  int M;
  // dequant
  float* w;
  long long ldw;
};

__device__ __forceinline__ float f16(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Ids of this lane's 8 blocks of stage s in chunk c (1- or 2-byte ids).
__device__ __forceinline__ void load_ids(const F32Params& p, long long t, int c, int s, int rr, int half,
                                         uint32_t (&ids)[8]) {
  const int V = p.R * p.idw;
  const uint8_t* base = p.packed + ((t * p.chunks + c) * V) * 256 + rr * 16;
  if (p.idw == 1) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(base + s * 256 + half * 8));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ids[j] = (v.x >> (8 * j)) & 0xFFu;
      ids[4 + j] = (v.y >> (8 * j)) & 0xFFu;
    }
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (s * 2 + half) * 256));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ids[2 * j] = w[j] & 0xFFFFu;
      ids[2 * j + 1] = w[j] >> 16;
    }
  }
}

// Exact fp32 weight of column j of the block whose stage ids are ids_s (row scale rho).
__device__ __forceinline__ float weight_f32(const F32Params& p, const uint16_t* books, const float* scales,
                                            const uint32_t* ids, int j, float rho) {
  float acc = 0.0f;
  for (int s = 0; s < p.R; ++s) {
    float v = f16(__ldg(books + ((size_t)s * p.entries + ids[s]) * p.d + j));
    if (scales) v = __fmul_rn(v, scales[s]);
    acc = (s == 0 && p.fast) ? v : __fadd_rn(acc, v);
  }
  return __fmul_rn(acc, rho);
}

template <bool GEMV>
__global__ void __launch_bounds__(kWarps * 32) rvq_f32_kernel(const __grid_constant__ F32Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = lane & 15, half = lane >> 4;
  const long long t = (long long)blockIdx.x * kWarps + warp;
  if (t >= p.num_tiles) return;
  const int4 ti = p.tiles[t];
  const bool live = rr < ti.z;
  const int row = ti.y + rr;
  const uint16_t* books = p.codebooks + (size_t)ti.x * p.R * p.entries * p.d;
  const float* scales = p.stage_scales ? p.stage_scales + (size_t)ti.x * p.R : nullptr;
  const float rho = live ? f16(p.row_scale[row]) : 0.0f;
  float acc[kTokens];
#pragma unroll
  for (int m = 0; m < kTokens; ++m) acc[m] = 0.0f;
  const int bpc = 16;  // blocks per chunk
  for (int c = 0; c < p.chunks; ++c) {
    uint32_t ids[4][8];
    for (int s = 0; s < p.R; ++s) load_ids(p, t, c, s, rr, half, ids[s]);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int k0 = (c * bpc + half * 8 + b) * p.d;
      uint32_t bid[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) bid[s] = ids[s][b];
      for (int j = 0; j < p.d; ++j) {
        const int k = k0 + j;
        if (k >= p.K) break;
        const float wv = weight_f32(p, books, scales, bid, j, rho);
        if constexpr (GEMV) {
#pragma unroll
          for (int m = 0; m < kTokens; ++m)
            if (m < p.M) acc[m] = fmaf(wv, __ldg(p.x + m * p.ldx + k), acc[m]);
        } else {
          if (live) p.w[(long long)row * p.ldw + k] = wv;
        }
      }
    }
  }
  if constexpr (GEMV) {
#pragma unroll
    for (int m = 0; m < kTokens; ++m) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 16);
    if (half == 0 && live) {
      const float b = p.bias ? __uint_as_float((uint32_t)p.bias[row] << 16) : 0.0f;
      for (int m = 0; m < p.M; ++m) p.y[m * p.ldy + row] = acc[m] + b;
    }
  }
}

int fill_params(const wal_rvq_layer* L, F32Params* p) {
  const wal_rvq_geometry& g = L->geom;
  if (g.num_stages > 4) return WAL_ERR_UNSUPPORTED;
  *p = F32Params{};
  p->packed = static_cast<const uint8_t*>(L->packed_ids);
  p->tiles = reinterpret_cast<const int4*>(L->tile_table);
  p->codebooks = L->codebooks;
  p->row_scale = L->row_scale;
  p->bias = L->bias;
  p->stage_scales = L->stage_scales;
  p->num_tiles = L->num_tiles;
  p->K = (int)g.in_features;
  p->d = g.block_size;
  p->R = g.num_stages;
  p->idw = g.num_entries <= 256 ? 1 : 2;
  p->chunks = (int)(((g.in_features + g.block_size - 1) / g.block_size + 15) / 16);
  p->entries = g.num_entries;
  p->fast = L->sum_mode == WAL_SUM_FAST;
  return WAL_OK;
}

}  // namespace

// Entry points called from the C ABI unit (arguments already validated there
// except the fp32-specific ones).
int wal_rvq_gemv_f32_impl(const wal_rvq_layer* layer, const float* x, int64_t M, int64_t ldx, float* y, int64_t ldy,
                          cudaStream_t stream) {
  const wal_rvq_geometry& g = layer->geom;
  if (ldx < g.in_features || ldy < g.out_features) return WAL_ERR_SHAPE;
  if (((uintptr_t)x & 3) || ((uintptr_t)y & 3)) return WAL_ERR_ALIGNMENT;
  F32Params p;
  int st = fill_params(layer, &p);
  if (st != WAL_OK) return st;
  p.ldx = ldx;
  p.ldy = ldy;
  const unsigned grid = (unsigned)((layer->num_tiles + kWarps - 1) / kWarps);
  for (int64_t m0 = 0; m0 < M; m0 += kTokens) {
    p.x = x + m0 * ldx;
    p.y = y + m0 * ldy;
    p.M = (int)(M - m0 < kTokens ? M - m0 : kTokens);
    rvq_f32_kernel<true><<<grid, kWarps * 32, 0, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return WAL_ERR_CUDA;
  }
  return WAL_OK;
}

int wal_rvq_dequant_f32_impl(const wal_rvq_layer* layer, float* w, int64_t ldw, cudaStream_t stream) {
  F32Params p;
  int st = fill_params(layer, &p);
  if (st != WAL_OK) return st;
  p.w = w;
  p.ldw = ldw;
  const unsigned grid = (unsigned)((layer->num_tiles + kWarps - 1) / kWarps);
  rvq_f32_kernel<false><<<grid, kWarps * 32, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}
