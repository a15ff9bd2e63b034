// ID-route linear: one int16 id per weight into a scalar fp16 route table
// (reference src/runtime.py:52-97, PackedIDRouteLinear, and its fused Triton
// kernel src/triton_id_matmul.py:19-67).  The weight is, bit for bit, the
// reference's dequantised bf16 weight:
//
//   w[n, k] = bf16_rn( fp16_rn( codebook_sum[ids[n, k]] * row_scale[n] ) )
//
// (fp16 gather times fp16 row scale rounded to fp16, `reconstruct_weight`
// src/runtime.py:89-93, then `.to(x.dtype)` in `forward` :95-97).
//
// At 2 bytes of ids per weight this format can be HBM-bound, so the GEMV is
// built around the id stream: tiles of 16 rows, chunks of 128 columns stored
// as 8 x 512-byte warp-wide vectors (4 KB), read with cp.async into a per-warp
// ring (two chunks in flight per warp); the route table sits in shared memory
// replicated in 8 bank-spread copies so the 32 random 2-byte gathers of a warp
// fall on at most a few bank conflicts; every weight is formed with one packed
// fp16 multiply (exact product, one fp16 rounding) and one bf16 conversion,
// and fed to mma.sync m16n8k16 (bf16 in, fp32 accumulate) with the activation
// fragment (same k-permutation as the Block-RVQ GEMV).
#include "../../include/wal_rvq.h"
#include "wal_rvq_decode.cuh"

#include <cstring>
#include <vector>

namespace wal {
namespace idroute {

constexpr int kW = 16;               // warps per CTA
constexpr int kT = kW * 32;
constexpr int kRing = 2;             // chunks in flight per warp
constexpr int kChunkBytes = 4096;    // 16 rows x 128 columns x 2 bytes
constexpr int kChunkCols = 128;
constexpr int kMaxTable = 64 * 1024; // bytes of shared memory for the replicated table
constexpr int kXBudget = 40 * 1024;

struct Params {
  const uint8_t* packed;
  const uint16_t* table;  // fp16 [routes]
  const uint16_t* row_scale;
  const uint16_t* bias;
  const uint16_t* x;
  void* y;
  long long ldx, ldy;
  int N, K, M, routes, chunks, tiles, y_dtype, copies_log2;
};

template <int I, int N, typename F>
__device__ __forceinline__ void sfor(F&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    sfor<I + 1, N>(f);
  }
}

// Table gather (the table is written once before a barrier; the address
// depends on ids read after it, so the load needs no ordering of its own).
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// fp16x2 (gathered pair) * fp16x2 (row scale) rounded to fp16, then each half
// converted to bf16 (round to nearest): the reference's two roundings.
__device__ __forceinline__ uint32_t weight_pair(uint32_t h2, uint32_t rho2) {
  uint32_t p;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(p) : "r"(h2), "r"(rho2));
  float lo, hi;
  asm("{\n .reg .f16 a, b;\n mov.b32 {a, b}, %2;\n cvt.f32.f16 %0, a;\n cvt.f32.f16 %1, b;\n}" : "=f"(lo), "=f"(hi) : "r"(p));
  return pack_bf16x2_rn(lo, hi);
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Byte address of id's copy for this lane.  Replicated table (COMPACT false):
// entry e of copy c is the 32-bit word e * copies + c (value in the low half);
// compact table (large route tables): one fp16 per entry.
template <int CL2>
__device__ __forceinline__ uint32_t gather_addr(uint32_t id, uint32_t tbl_lane) {
  return CL2 < 0 ? tbl_lane + (id << 1) : tbl_lane + (id << (CL2 + 2));
}

// CL2: log2 of the table copies (word per entry), or -1 for the compact table.
template <int MT, bool XS, int CL2>
__global__ void __launch_bounds__(kT, 1) idroute_gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr bool COMPACT = CL2 < 0;
  constexpr int copies = COMPACT ? 1 : 1 << (CL2 < 0 ? 0 : CL2);
  const int table_bytes = COMPACT ? p.routes * 2 : p.routes * copies * 4;
  const int kpad = p.chunks * kChunkCols;
  const int xstride = kpad * 2 + 32;  // bytes per staged activation row
  uint8_t* tbl = smem;
  uint8_t* xs = smem + ((table_bytes + 127) & ~127);
  const int xbytes = XS ? (((p.M + 1) * xstride + 127) & ~127) : 0;
  uint8_t* ring = xs + xbytes;
  float* red = reinterpret_cast<float*>(ring + kW * kRing * kChunkBytes);  // [kW][16][MT*8]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, q = lane & 3;
  // whole tiles per CTA, chunks of a tile split over the 16 warps
  const int tq = p.tiles / gridDim.x, tr = p.tiles % gridDim.x;
  const int tb = blockIdx.x * tq + (blockIdx.x < tr ? blockIdx.x : tr);
  const int te = tb + tq + (blockIdx.x < tr ? 1 : 0);

  // table: fp16 entries, one per 32-bit word, `copies` copies interleaved
  // (compact: plain fp16 array)
  for (int e = threadIdx.x; e < p.routes; e += kT) {
    const uint32_t v = p.table[e];
    if (COMPACT) {
      reinterpret_cast<uint16_t*>(tbl)[e] = (uint16_t)v;
    } else {
      uint32_t* w = reinterpret_cast<uint32_t*>(tbl) + (size_t)e * copies;
      for (int c = 0; c < copies; ++c) w[c] = v;
    }
  }
  // this warp's items: for each tile, chunks warp, warp + 16, ...
  const int cpw = warp < p.chunks ? (p.chunks - warp + kW - 1) / kW : 0;
  const int items = (te - tb) * cpw;
  const uint32_t ring_w = smem_u32(ring) + warp * kRing * kChunkBytes;
  const uint64_t pol = l2_policy_evict_first();
  // issue cursor: next item's tile and chunk, advanced without division
  int is_left = items, is_t = tb, is_c = warp;
  auto issue = [&](int slot) {
    if (is_left > 0) {
      const uint8_t* src = p.packed + ((long long)is_t * p.chunks + is_c) * kChunkBytes + lane * 16;
#pragma unroll
      for (int v = 0; v < 8; ++v) cp_async_16_hint(ring_w + slot * kChunkBytes + v * 512 + lane * 16, src + v * 512, pol);
      --is_left;
      is_c += kW;
      if (is_c >= p.chunks) {
        is_c = warp;
        ++is_t;
      }
    }
    cp_commit();
  };
  issue(0);
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  if (XS) {
    for (int m = 0; m <= p.M; ++m) {
      uint16_t* dst = reinterpret_cast<uint16_t*>(xs + m * xstride);
      for (int col = threadIdx.x * 8; col < kpad; col += kT * 8) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (m < p.M) {
          const uint16_t* src = p.x + (long long)m * p.ldx + col;
          if (col + 8 <= p.K && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
            v = *reinterpret_cast<const uint4*>(src);
          } else {
            uint16_t t8[8];
            for (int j = 0; j < 8; ++j) t8[j] = col + j < p.K ? src[j] : (uint16_t)0;
            memcpy(&v, t8, 16);
          }
        }
        *reinterpret_cast<uint4*>(dst + col) = v;
      }
    }
  }
  __syncthreads();
  // the next kernel of the stream may launch now: its CTAs take each SM as this
  // grid's CTA there exits, overlapping their prologue with this grid's tail
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

  const uint32_t tbl_lane = smem_u32(tbl) + (COMPACT ? 0u : (uint32_t)((lane & (copies - 1)) * 4));
  uint32_t xsa[MT];
  uint32_t xoff[MT];
  bool xv[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    const int m = 8 * i + r;
    xv[i] = m < p.M;
    xsa[i] = smem_u32(xs) + (uint32_t)((xv[i] ? m : p.M) * xstride);
    xoff[i] = (uint32_t)((xv[i] ? m : 0) * p.ldx);
  }

  int it = 0;
  for (int t = tb; t < te; ++t) {
    float acc[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    const int row_a = 16 * t + r, row_b = row_a + 8;
    const uint32_t rho_a = row_a < p.N ? (uint32_t)p.row_scale[row_a] * 0x10001u : 0u;
    const uint32_t rho_b = row_b < p.N ? (uint32_t)p.row_scale[row_b] * 0x10001u : 0u;
    for (int j = 0; j < cpw; ++j, ++it) {
      issue((it + 1) & 1);
      cp_wait<1>();
      __syncwarp();
      const uint32_t slot = ring_w + (it & 1) * kChunkBytes + lane * 16;
      const int c = warp + j * kW;
      uint4 ida[4], idb[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(ida[g].x), "=r"(ida[g].y), "=r"(ida[g].z), "=r"(ida[g].w)
                     : "r"(slot + g * 512));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(idb[g].x), "=r"(idb[g].y), "=r"(idb[g].z), "=r"(idb[g].w)
                     : "r"(slot + (4 + g) * 512));
      }
      __syncwarp();
      const int col_base = c * kChunkCols + 4 * q;
      sfor<0, 8>([&](auto ktc) {
        constexpr int kt = decltype(ktc)::value;
        // ids of row r / r+8 for this k-tile: words (kt&1)*2, +1 of vector kt/2
        const uint32_t wa0 = (kt & 1) ? ida[kt >> 1].z : ida[kt >> 1].x;
        const uint32_t wa1 = (kt & 1) ? ida[kt >> 1].w : ida[kt >> 1].y;
        const uint32_t wb0 = (kt & 1) ? idb[kt >> 1].z : idb[kt >> 1].x;
        const uint32_t wb1 = (kt & 1) ? idb[kt >> 1].w : idb[kt >> 1].y;
        auto pair = [&](uint32_t w2) {
          const uint32_t lo = lds_u16(gather_addr<CL2>(w2 & 0xFFFFu, tbl_lane));
          const uint32_t hi = lds_u16(gather_addr<CL2>(w2 >> 16, tbl_lane));
          return lo | (hi << 16);
        };
        uint32_t a[4];
        a[0] = weight_pair(pair(wa0), rho_a);
        a[1] = weight_pair(pair(wb0), rho_b);
        a[2] = weight_pair(pair(wa1), rho_a);
        a[3] = weight_pair(pair(wb1), rho_b);
        const int col = col_base + kt * 16;
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          uint2 xf = make_uint2(0u, 0u);
          if (XS) {
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(xf.x), "=r"(xf.y) : "r"(xsa[i] + col * 2));
          } else if (xv[i] && col < p.K) {
            xf = __ldg(reinterpret_cast<const uint2*>(p.x + xoff[i] + col));
          }
          if (!XS && col >= p.K) a[0] = a[1] = a[2] = a[3] = 0u;
          mma_bf16_16816(acc[i], a, xf.x, xf.y);
        }
      });
    }
    // fixed-order reduction of the 16 warps' partial sums for this tile
    constexpr int MC = MT * 8;
    float* wred = red + warp * 16 * MC;
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      wred[r * MC + i * 8 + 2 * q] = acc[i][0];
      wred[r * MC + i * 8 + 2 * q + 1] = acc[i][1];
      wred[(r + 8) * MC + i * 8 + 2 * q] = acc[i][2];
      wred[(r + 8) * MC + i * 8 + 2 * q + 1] = acc[i][3];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 16 * MC; e += kT) {
      const int row = e / MC, m = e - row * MC;
      const int n = 16 * t + row;
      if (n >= p.N || m >= p.M) continue;
      float v = 0.f;
      for (int w = 0; w < kW; ++w) v += red[(w * 16 + row) * MC + m];
      if (p.bias) v += __bfloat162float(__ushort_as_bfloat16(p.bias[n]));
      const long long idx = (long long)m * p.ldy + n;
      if (p.y_dtype == WAL_F32) static_cast<float*>(p.y)[idx] = v;
      else static_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(v);
    }
    __syncthreads();
  }
  cp_wait<0>();
}

// The weight [N, K] through the same arithmetic (one thread per weight pair):
// bf16 (the forward's weight) or the fp16 product (the reference's
// reconstruct_weight before the dtype cast).
__global__ void idroute_dequant_kernel(const __grid_constant__ Params p, uint16_t* w, long long ldw, int f16) {
  const long long pairs = (long long)p.N * (p.K / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < pairs; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (p.K / 2));
    const int k = (int)(i - (long long)n * (p.K / 2)) * 2;
    const int t = n >> 4, rr = n & 15, c = k / kChunkCols, cc = k % kChunkCols;
    // inverse of the packing: (row half, k-pair group, lane, 8-byte half)
    const int h = rr >> 3, rlow = rr & 7, g = cc >> 5, in32 = cc & 31;
    const int khalf = in32 >> 4, qq = (in32 & 15) >> 2, j = in32 & 3;
    const uint8_t* v = p.packed + ((long long)t * p.chunks + c) * kChunkBytes + (h * 4 + g) * 512 +
                       (rlow * 4 + qq) * 16 + khalf * 8 + j * 2;
    const uint32_t id0 = *reinterpret_cast<const uint16_t*>(v), id1 = *reinterpret_cast<const uint16_t*>(v + 2);
    const uint32_t h2 = (uint32_t)p.table[id0] | ((uint32_t)p.table[id1] << 16);
    const uint32_t rho2 = (uint32_t)p.row_scale[n] * 0x10001u;
    uint32_t out;
    if (f16) {
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(out) : "r"(h2), "r"(rho2));
    } else {
      out = weight_pair(h2, rho2);
    }
    *reinterpret_cast<uint32_t*>(w + (long long)n * ldw + k) = out;
  }
}

}  // namespace idroute
}  // namespace wal

using namespace wal::idroute;

namespace {

int check(const wal_idroute_layer* L) {
  if (!L) return WAL_ERR_INVALID_ARGUMENT;
  if (L->out_features <= 0 || L->in_features <= 0 || L->num_routes <= 0) return WAL_ERR_SHAPE;
  if (L->num_routes > 32767) return WAL_ERR_UNSUPPORTED;
  if (L->in_features % 8) return WAL_ERR_UNSUPPORTED;
  if (L->out_features > (1 << 30) || L->in_features > (1 << 28)) return WAL_ERR_SHAPE;
  if (!L->packed_ids || !L->codebook_sum || !L->row_scale) return WAL_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)L->packed_ids & 15) return WAL_ERR_ALIGNMENT;
  return WAL_OK;
}

Params make_params(const wal_idroute_layer* L) {
  Params p{};
  p.packed = static_cast<const uint8_t*>(L->packed_ids);
  p.table = L->codebook_sum;
  p.row_scale = L->row_scale;
  p.bias = L->bias;
  p.N = (int)L->out_features;
  p.K = (int)L->in_features;
  p.routes = L->num_routes;
  p.chunks = (int)((L->in_features + kChunkCols - 1) / kChunkCols);
  p.tiles = (int)((L->out_features + 15) / 16);
  int cl2 = 3;  // 8 copies when they fit; -1: compact fp16 table
  while (cl2 >= 0 && (long long)p.routes * (4 << cl2) > kMaxTable) --cl2;
  p.copies_log2 = cl2;
  return p;
}

template <int MT, bool XS, int CL2>
int launch(Params p, cudaStream_t s) {
  auto kern = idroute_gemv_kernel<MT, XS, CL2>;
  const int table = ((CL2 < 0 ? p.routes * 2 : p.routes * (4 << (CL2 < 0 ? 0 : CL2))) + 127) & ~127;
  const int kpad = p.chunks * kChunkCols;
  const int xbytes = XS ? (((p.M + 1) * (kpad * 2 + 32) + 127) & ~127) : 0;
  const int smem = table + xbytes + kW * kRing * kChunkBytes + kW * 16 * MT * 8 * 4;
  if (smem > 227 * 1024) return WAL_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return WAL_ERR_CUDA;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = p.tiles < sms ? p.tiles : sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return WAL_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

}  // namespace

extern "C" {

int wal_idroute_packed_size(int64_t out_features, int64_t in_features, size_t* packed_bytes) {
  if (!packed_bytes) return WAL_ERR_INVALID_ARGUMENT;
  if (out_features <= 0 || in_features <= 0) return WAL_ERR_SHAPE;
  const long long tiles = (out_features + 15) / 16, chunks = (in_features + kChunkCols - 1) / kChunkCols;
  *packed_bytes = (size_t)(tiles * chunks * kChunkBytes);
  return WAL_OK;
}

int wal_idroute_pack(int64_t out_features, int64_t in_features, int32_t num_routes, const int16_t* ids, void* packed,
                     size_t packed_bytes) {
  if (!ids || !packed) return WAL_ERR_INVALID_ARGUMENT;
  if (num_routes <= 0 || num_routes > 32767) return WAL_ERR_UNSUPPORTED;
  size_t need = 0;
  int st = wal_idroute_packed_size(out_features, in_features, &need);
  if (st != WAL_OK) return st;
  if (packed_bytes < need) return WAL_ERR_BUFFER_TOO_SMALL;
  std::memset(packed, 0, need);
  const long long chunks = (in_features + kChunkCols - 1) / kChunkCols;
  uint8_t* out = static_cast<uint8_t*>(packed);
  for (long long n = 0; n < out_features; ++n) {
    const long long t = n >> 4;
    const int rr = (int)(n & 15), h = rr >> 3, rlow = rr & 7;
    for (long long k = 0; k < in_features; ++k) {
      const int16_t id = ids[n * in_features + k];
      if (id < 0 || id >= num_routes) return WAL_ERR_ID_RANGE;
      const long long c = k / kChunkCols;
      const int cc = (int)(k % kChunkCols), g = cc >> 5, in32 = cc & 31;
      const int khalf = in32 >> 4, qq = (in32 & 15) >> 2, j = in32 & 3;
      uint8_t* dst = out + (t * chunks + c) * kChunkBytes + (h * 4 + g) * 512 + (rlow * 4 + qq) * 16 + khalf * 8 + j * 2;
      std::memcpy(dst, &id, 2);
    }
  }
  return WAL_OK;
}

int wal_idroute_gemv(const wal_idroute_layer* layer, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                     int64_t ldy, int y_dtype, void* stream) {
  int st = check(layer);
  if (st != WAL_OK) return st;
  if (!x || !y) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0) return WAL_ERR_SHAPE;
  if (ldx < layer->in_features || ldy < layer->out_features || ldx >= (1LL << 26)) return WAL_ERR_SHAPE;
  if ((ldx % 4) || ((uintptr_t)x & 7)) return WAL_ERR_ALIGNMENT;
  if (y_dtype != WAL_BF16 && y_dtype != WAL_F32) return WAL_ERR_INVALID_ARGUMENT;
  Params p = make_params(layer);
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
    const bool xs = (long long)(mm + 1) * (p.chunks * kChunkCols * 2 + 32) <= kXBudget;
    // 8 copies of the table (the common small tables) or the compact table;
    // intermediate copy counts round down to the next form that fits
    auto go = [&](bool stage_x) {
      if (p.copies_log2 >= 3) {
        p.copies_log2 = 3;
        if (mm <= 8) return stage_x ? launch<1, true, 3>(p, s) : launch<1, false, 3>(p, s);
        return stage_x ? launch<2, true, 3>(p, s) : launch<2, false, 3>(p, s);
      }
      if (p.copies_log2 >= 0) {
        p.copies_log2 = 0;
        if (mm <= 8) return stage_x ? launch<1, true, 0>(p, s) : launch<1, false, 0>(p, s);
        return stage_x ? launch<2, true, 0>(p, s) : launch<2, false, 0>(p, s);
      }
      if (mm <= 8) return stage_x ? launch<1, true, -1>(p, s) : launch<1, false, -1>(p, s);
      return stage_x ? launch<2, true, -1>(p, s) : launch<2, false, -1>(p, s);
    };
    int rs = go(xs);
    if (rs == WAL_ERR_UNSUPPORTED && xs) rs = go(false);  // activations do not fit beside the table
    if (rs != WAL_OK) return rs;
  }
  return WAL_OK;
}

int wal_idroute_dequant(const wal_idroute_layer* layer, uint16_t* w, int64_t ldw, int w_dtype, void* stream) {
  int st = check(layer);
  if (st != WAL_OK) return st;
  if (!w) return WAL_ERR_INVALID_ARGUMENT;
  if (w_dtype != WAL_BF16 && w_dtype != WAL_F16) return WAL_ERR_INVALID_ARGUMENT;
  if (ldw < layer->in_features || (ldw % 2) || ((uintptr_t)w & 3)) return WAL_ERR_ALIGNMENT;
  Params p = make_params(layer);
  const long long pairs = (long long)p.N * (p.K / 2);
  long long grid = (pairs + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  idroute_dequant_kernel<<<(int)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p, w, ldw, w_dtype == WAL_F16);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

}  // extern "C"
