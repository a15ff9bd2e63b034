// Block-RVQ encodings with per-block corrections (reference
// src/runtime.py:389-412, PackedBlockRVQGroup.reconstruct_weight): after the
// fp32 stage sum S of a block (d columns),
//   sign residual    S += (sigma * residual_scale) @ H    sigma_i = +-1 from a packed sign bit,
//                                                       H the fixed d x d sign-correction matrix
//   block scale      S *= block_scale
//   transform        S = inverse_polar(S)  or  S = S @ M  (DCT, Hadamard, PCA ... matrix)
//   transform bias   S += bias
// and then the usual w = T(T(S) * T(rho)) in the weight type T (fp32: S * rho).
// These steps mix the d columns of a block, so every weight of a block needs
// the whole block: one lane owns whole blocks of one row (8 blocks of a
// 16-block chunk per lane, two lanes per row, one warp per 16-row tile),
// evaluates the pipeline in fp32 registers and, for the GEMV, multiplies each
// weight with up to 8 tokens on the CUDA cores (fp32 fused multiply-add);
// the materialising kernel stores the weights instead.  The matrix products
// run in ascending index order with fused multiply-adds, so a weight can
// differ from the reference's (whose CPU matrix product sums in its own
// order) in the last fp32 bit before rounding: after the rounding to the
// weight type such a difference surfaces in about one weight in 10^4.
#include "../../include/wal_rvq.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kWarps = 8;
constexpr int kTokens = 8;
constexpr float kPi = 3.14159265358979323846f;

struct CorrParams {
  const uint8_t* packed;
  const int4* tiles;
  const uint16_t* codebooks;
  const uint16_t* row_scale;
  const uint16_t* bias;
  const float* stage_scales;
  wal_rvq_corrections corr;
  long long num_tiles;
  int K, d, R, idw, chunks, entries, blocks;
  int wtype;  // WAL_BF16, WAL_F16 or WAL_F32
  // GEMV
  const void* x;
  long long ldx;
  void* y;
  long long ldy;
  int y_dtype;
  int M;
  // materialise
  void* w;
  long long ldw;
};

__device__ __forceinline__ float f16v(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ float bf16v(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ float round_to(float v, int wtype) {
  if (wtype == WAL_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (wtype == WAL_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float load_x(const CorrParams& p, int m, int k) {
  if (p.wtype == WAL_F32) return __ldg(static_cast<const float*>(p.x) + m * p.ldx + k);
  const uint16_t b = __ldg(static_cast<const uint16_t*>(p.x) + m * p.ldx + k);
  return p.wtype == WAL_F16 ? f16v(b) : bf16v(b);
}

// Ids of this lane's 8 blocks of stage s in chunk c.
__device__ __forceinline__ void load_ids(const CorrParams& p, long long t, int c, int s, int rr, int half,
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

// The pre-rounding block vector of unit u (row-major unit index) of group g.
template <int D>
__device__ __forceinline__ void block_vector(const CorrParams& p, int g, long long u, const uint32_t* ids,
                                             float (&v)[D]) {
  const uint16_t* books = p.codebooks + (size_t)g * p.R * p.entries * D;
  const float* scales = p.stage_scales ? p.stage_scales + (size_t)g * p.R : nullptr;
#pragma unroll
  for (int j = 0; j < D; ++j) v[j] = 0.0f;
  for (int s = 0; s < p.R; ++s) {
    const uint16_t* e = books + ((size_t)s * p.entries + ids[s]) * D;
#pragma unroll
    for (int j = 0; j < D; ++j) {
      float c = f16v(__ldg(e + j));
      if (scales) c = __fmul_rn(c, scales[s]);
      v[j] = __fadd_rn(v[j], c);
    }
  }
  const int flags = p.corr.group_flags ? __ldg(p.corr.group_flags + g) : 0;
  if (flags & WAL_CORR_SIGN) {
    const uint32_t bits = (uint32_t)__ldg(p.corr.residual_signs + u);
    const float rs = f16v(__ldg(p.corr.residual_scale + u));
    float c[D];
#pragma unroll
    for (int j = 0; j < D; ++j) c[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      const float a = ((bits >> i) & 1u) ? rs : -rs;
#pragma unroll
      for (int j = 0; j < D; ++j) c[j] = fmaf(a, __ldg(p.corr.sign_matrix + i * D + j), c[j]);
    }
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = __fadd_rn(v[j], c[j]);
  }
  if (flags & WAL_CORR_BLOCK_SCALE) {
    const float bs = f16v(__ldg(p.corr.block_scale + u));
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = __fmul_rn(v[j], bs);
  }
  if (flags & WAL_CORR_POLAR) {
    // radii first, then angle groups of widths 1, 2, 4, ... (each angle in units of pi)
    float cur[D];
    cur[0] = v[0];
    int offset = 1;
#pragma unroll
    for (int width = 1; width < D; width *= 2) {
      float nxt[D];
#pragma unroll
      for (int k = 0; k < D; ++k) {
        if (k < width) {
          const float ang = __fmul_rn(kPi, v[offset + k]);
          nxt[2 * k] = __fmul_rn(cur[k], cosf(ang));
          nxt[2 * k + 1] = __fmul_rn(cur[k], sinf(ang));
        }
      }
#pragma unroll
      for (int k = 0; k < D; ++k)
        if (k < 2 * width) cur[k] = nxt[k];
      offset += width;
    }
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = cur[j];
  } else if (flags & WAL_CORR_MATRIX) {
    const float* m = p.corr.transform + (size_t)g * D * D;
    float o[D];
#pragma unroll
    for (int j = 0; j < D; ++j) o[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < D; ++i) {
#pragma unroll
      for (int j = 0; j < D; ++j) o[j] = fmaf(v[i], __ldg(m + i * D + j), o[j]);
    }
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = o[j];
  }
  if (flags & WAL_CORR_BIAS) {
    const float* b = p.corr.transform_bias + (size_t)g * D;
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = __fadd_rn(v[j], __ldg(b + j));
  }
}

template <int D, bool GEMV>
__global__ void __launch_bounds__(kWarps * 32) rvq_corrected_kernel(const __grid_constant__ CorrParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = lane & 15, half = lane >> 4;
  const long long t = (long long)blockIdx.x * kWarps + warp;
  if (t >= p.num_tiles) return;
  const int4 ti = p.tiles[t];
  const bool live = rr < ti.z;
  const int row = ti.y + rr;
  const float rho_w = live ? round_to(f16v(p.row_scale[row]), p.wtype) : 0.0f;
  float acc[kTokens];
#pragma unroll
  for (int m = 0; m < kTokens; ++m) acc[m] = 0.0f;
  for (int c = 0; c < p.chunks; ++c) {
    uint32_t ids[4][8];
    for (int s = 0; s < p.R; ++s) load_ids(p, t, c, s, rr, half, ids[s]);
    for (int b8 = 0; b8 < 8; ++b8) {
      const int b = c * 16 + half * 8 + b8;
      if (b >= p.blocks || !live) continue;
      uint32_t bid[4] = {ids[0][b8], ids[1][b8], ids[2][b8], ids[3][b8]};
      float v[D];
      block_vector<D>(p, ti.x, (long long)row * p.blocks + b, bid, v);
#pragma unroll
      for (int j = 0; j < D; ++j) {
        const int k = b * D + j;
        if (k >= p.K) break;
        const float wv = p.wtype == WAL_F32 ? __fmul_rn(v[j], rho_w)
                                            : round_to(__fmul_rn(round_to(v[j], p.wtype), rho_w), p.wtype);
        if constexpr (GEMV) {
#pragma unroll
          for (int m = 0; m < kTokens; ++m)
            if (m < p.M) acc[m] = fmaf(wv, load_x(p, m, k), acc[m]);
        } else {
          const long long o = (long long)row * p.ldw + k;
          if (p.wtype == WAL_F32) {
            static_cast<float*>(p.w)[o] = wv;
          } else if (p.wtype == WAL_F16) {
            static_cast<__half*>(p.w)[o] = __float2half_rn(wv);
          } else {
            static_cast<__nv_bfloat16*>(p.w)[o] = __float2bfloat16_rn(wv);
          }
        }
      }
    }
  }
  if constexpr (GEMV) {
#pragma unroll
    for (int m = 0; m < kTokens; ++m) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], 16);
    if (half == 0 && live) {
      const float bias = p.bias ? bf16v(p.bias[row]) : 0.0f;
      for (int m = 0; m < p.M; ++m) {
        const float o = acc[m] + bias;
        const long long idx = m * p.ldy + row;
        if (p.y_dtype == WAL_F32) {
          static_cast<float*>(p.y)[idx] = o;
        } else if (p.y_dtype == WAL_F16) {
          static_cast<__half*>(p.y)[idx] = __float2half_rn(o);
        } else {
          static_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(o);
        }
      }
    }
  }
}

int fill(const wal_rvq_layer* L, const wal_rvq_corrections* corr, int wtype, CorrParams* p) {
  if (!L || !corr) return WAL_ERR_INVALID_ARGUMENT;
  const wal_rvq_geometry& g = L->geom;
  if (g.out_features <= 0 || g.in_features <= 0 || L->num_tiles <= 0) return WAL_ERR_SHAPE;
  if (g.block_size != 8 && g.block_size != 16 && g.block_size != 32) return WAL_ERR_UNSUPPORTED;
  if (g.num_stages < 1 || g.num_stages > 4) return WAL_ERR_UNSUPPORTED;
  if (L->sum_mode != WAL_SUM_EXACT) return WAL_ERR_UNSUPPORTED;  // the reference's fast path has no corrections
  if (!L->packed_ids || !L->tile_table || !L->codebooks || !L->row_scale || !corr->group_flags)
    return WAL_ERR_INVALID_ARGUMENT;
  if (wtype != WAL_BF16 && wtype != WAL_F16 && wtype != WAL_F32) return WAL_ERR_INVALID_ARGUMENT;
  *p = CorrParams{};
  p->packed = static_cast<const uint8_t*>(L->packed_ids);
  p->tiles = reinterpret_cast<const int4*>(L->tile_table);
  p->codebooks = L->codebooks;
  p->row_scale = L->row_scale;
  p->bias = L->bias;
  p->stage_scales = L->stage_scales;
  p->corr = *corr;
  p->num_tiles = L->num_tiles;
  p->K = (int)g.in_features;
  p->d = g.block_size;
  p->R = g.num_stages;
  p->idw = g.num_entries <= 256 ? 1 : 2;
  p->blocks = (int)((g.in_features + g.block_size - 1) / g.block_size);
  p->chunks = (p->blocks + 15) / 16;
  p->entries = g.num_entries;
  p->wtype = wtype;
  return WAL_OK;
}

template <bool GEMV>
int launch(const CorrParams& p, cudaStream_t s) {
  const unsigned grid = (unsigned)((p.num_tiles + kWarps - 1) / kWarps);
  if (p.d == 8) rvq_corrected_kernel<8, GEMV><<<grid, kWarps * 32, 0, s>>>(p);
  else if (p.d == 16) rvq_corrected_kernel<16, GEMV><<<grid, kWarps * 32, 0, s>>>(p);
  else rvq_corrected_kernel<32, GEMV><<<grid, kWarps * 32, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

}  // namespace

extern "C" {

int wal_rvq_gemv_corrected(const wal_rvq_layer* layer, const wal_rvq_corrections* corr, const void* x, int x_dtype,
                           int64_t M, int64_t ldx, void* y, int64_t ldy, int y_dtype, void* stream) {
  CorrParams p;
  int st = fill(layer, corr, x_dtype, &p);
  if (st != WAL_OK) return st;
  if (!x || !y) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0 || ldx < layer->geom.in_features || ldy < layer->geom.out_features) return WAL_ERR_SHAPE;
  if (y_dtype != WAL_BF16 && y_dtype != WAL_F16 && y_dtype != WAL_F32) return WAL_ERR_INVALID_ARGUMENT;
  p.ldx = ldx;
  p.ldy = ldy;
  p.y_dtype = y_dtype;
  const size_t xs = x_dtype == WAL_F32 ? 4 : 2, ys = y_dtype == WAL_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += kTokens) {
    p.x = static_cast<const uint8_t*>(x) + (size_t)(m0 * ldx) * xs;
    p.y = static_cast<uint8_t*>(y) + (size_t)(m0 * ldy) * ys;
    p.M = (int)(M - m0 < kTokens ? M - m0 : kTokens);
    st = launch<true>(p, static_cast<cudaStream_t>(stream));
    if (st != WAL_OK) return st;
  }
  return WAL_OK;
}

int wal_rvq_dequant_corrected(const wal_rvq_layer* layer, const wal_rvq_corrections* corr, void* w, int64_t ldw,
                              int w_dtype, void* stream) {
  CorrParams p;
  int st = fill(layer, corr, w_dtype, &p);
  if (st != WAL_OK) return st;
  if (!w) return WAL_ERR_INVALID_ARGUMENT;
  if (ldw < layer->geom.in_features) return WAL_ERR_SHAPE;
  p.w = w;
  p.ldw = ldw;
  return launch<false>(p, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
