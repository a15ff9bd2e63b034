// Device-side building blocks shared by the Block-RVQ kernels: shared-memory
// codebook layouts, staging, the exact per-weight decode and the tensor-core
// fragment conventions.
//
// Exact decode (reference src/runtime.py:379-414, restated per weight):
//   S  = ((+0.0f + fp32(c_0)) + fp32(c_1)) + ...      fp32, round-to-nearest
//   wb = bf16_rn(S)                                   first rounding
//   w  = bf16_rn(wb * bf16_rn(fp32(rho)))             second rounding
// For one stage the first rounding depends only on the codebook entry, so it
// is done once when the codebook is staged (the staged table then holds bf16
// values); for two or more stages the table holds the raw fp16 values and the
// sum is formed with the mixed-precision add (fp16 operand converted exactly).
//
// Fragment convention (mma.sync m16n8k16, bf16 in, fp32 accumulate): lane
// (r = lane/4, q = lane%4) owns, for rows r and r+8 of a 16-row tile, the four
// consecutive physical columns 16*kt + 4q .. 4q+3 of k-tile kt.  Physical
// columns 4q, 4q+1 sit in logical k slots 2q, 2q+1 and 4q+2, 4q+3 in slots
// 2q+8, 2q+9; the activation fragment uses the same map, so the product is a
// plain dot product over a permutation of k.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wal {

constexpr int kTileRows = 16;
constexpr int kChunkBlocks = 16;

// ---------------------------------------------------------------------------
// scalar helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float add_f32_f16(uint16_t h, float acc) {
  float d;
  asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(acc));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ uint32_t mul_bf16x2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// fp16 bits -> bf16 bits of bf16_rn(+0.0f + fp32(h)) (first rounding, one stage)
__device__ __forceinline__ uint32_t preround_pair(uint32_t h2) {
  const float lo = add_f32_f16((uint16_t)(h2 & 0xFFFFu), 0.0f);
  const float hi = add_f32_f16((uint16_t)(h2 >> 16), 0.0f);
  return pack_bf16x2_rn(lo, hi);
}

// fp16 row scale -> bf16x2 with both halves bf16_rn(fp32(rho))
__device__ __forceinline__ uint32_t rho_pair(uint16_t rho_bits) {
  const float f = __half2float(__ushort_as_half(rho_bits));
  const uint32_t b = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
  return b | (b << 16);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 lds_v2(uint32_t saddr) {
  uint2 v;
  asm("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(saddr) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------------------
// Shared-memory codebook layout.
//
// An entry of d values is split into d/4 pieces of 8 bytes.  A lane always
// reads one piece per (row, stage, k-tile).  In the replicated layout every
// piece is stored once per lane class so that the 16 lanes of a half-warp
// phase always hit 16 distinct bank pairs whatever ids they hold:
//   d = 8 : 8 copies, entry stride 128 B, lane offset (r&3)*32 + q*8
//   d = 16: 4 copies, entry stride 128 B, lane offset (r&3)*32 + q*8
//   d = 32: 4 copies, entry stride 256 B (+128 B for the second 16 columns)
// The plain layout stores each entry once (entry stride 2*d bytes) and is used
// when replication does not fit (large routed codebooks).
// ---------------------------------------------------------------------------
template <int D, bool REPL>
struct CbLayout {
  static constexpr int kPieces = D / 4;
  static constexpr int kCopies = REPL ? (D == 8 ? 8 : 4) : 1;
  static constexpr int kEntryStride = REPL ? (D == 32 ? 256 : 128) : 2 * D;
  static constexpr int kHalfStride = REPL ? 128 : 32;  // only D == 32 uses it
  __host__ __device__ static constexpr int stage_bytes(int entries) { return entries * D * 2 * kCopies; }
  __device__ static int piece_offset(int e, int j, int c) {
    if (!REPL) return (e * kPieces + j) * 8;
    if (D == 8) return ((e * 8 + c) * 2 + j) * 8;
    if (D == 16) return ((e * 4 + c) * 4 + j) * 8;
    return (((e * 2 + (j >> 2)) * 4 + c) * 4 + (j & 3)) * 8;
  }
  __device__ static int lane_offset(int r, int q) {
    if (REPL) return (r & 3) * 32 + q * 8;
    return D == 8 ? (q & 1) * 8 : q * 8;
  }
};

__device__ __forceinline__ void cp_async_16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gptr));
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }

// Stage R codebooks of one group (fp16 [R][entries][D] in global memory) into
// shared memory.  Every 16-byte run of an entry is fetched with cp.async into
// its copy-0 position (all fetches in flight at once), then copy 0 is expanded
// into the other copies; one-stage tables are pre-rounded to bf16 in place
// (first rounding).  Caller brackets the call with __syncthreads().
template <int D, int R, bool REPL>
__device__ void stage_codebooks(uint8_t* cb, const uint16_t* __restrict__ books, int entries) {
  using L = CbLayout<D, REPL>;
  const int sb = L::stage_bytes(entries);
  constexpr int kRuns = D / 8;  // 16-byte runs per entry (two pieces each)
  const int total_runs = R * entries * kRuns;
  const uint32_t base = smem_u32(cb);
  for (int i = threadIdx.x; i < total_runs; i += blockDim.x) {
    const int s = i / (entries * kRuns);
    const int rem = i - s * entries * kRuns;
    const int e = rem / kRuns;
    const int run = rem - e * kRuns;
    const uint16_t* src = books + ((size_t)s * entries + e) * D + 8 * run;
    cp_async_16(base + s * sb + L::piece_offset(e, 2 * run, 0), src);
  }
  cp_async_wait_all();
  if (R > 1 && !REPL) return;  // raw fp16 table, single copy: done
  __syncthreads();
  const int total_pieces = R * entries * L::kPieces;
  for (int i = threadIdx.x; i < total_pieces; i += blockDim.x) {
    const int s = i / (entries * L::kPieces);
    const int rem = i - s * entries * L::kPieces;
    const int e = rem / L::kPieces;
    const int j = rem - e * L::kPieces;
    uint8_t* sbase = cb + s * sb;
    uint2 v = *reinterpret_cast<const uint2*>(sbase + L::piece_offset(e, j, 0));
    if (R == 1) {
      v.x = preround_pair(v.x);
      v.y = preround_pair(v.y);
      *reinterpret_cast<uint2*>(sbase + L::piece_offset(e, j, 0)) = v;
    }
#pragma unroll
    for (int c = 1; c < L::kCopies; ++c) *reinterpret_cast<uint2*>(sbase + L::piece_offset(e, j, c)) = v;
  }
}

// ---------------------------------------------------------------------------
// Id extraction from one row's chunk registers.
// codes[v*4 + w] holds 32-bit word w of 16-byte vector v of this row's chunk.
// Block-in-chunk for k-tile KT of a lane with q:
//   D = 8 : 2*KT + (q >> 1)      D = 16: KT      D = 32: KT >> 1
// ---------------------------------------------------------------------------
template <int D, int IDW, int KT, int S, int V>
__device__ __forceinline__ uint32_t extract_id(const uint32_t (&codes)[V * 4], int qh_shift) {
  if (IDW == 1) {
    if (D == 8) {
      constexpr int b0 = 2 * KT;  // even; lane adds q>>1
      constexpr int word = S * 4 + (b0 >> 2);
      constexpr int sh = 8 * (b0 & 3);
      return (codes[word] >> (sh + qh_shift)) & 0xFFu;  // qh_shift = 8*(q>>1)
    } else {
      constexpr int b = (D == 16) ? KT : (KT >> 1);
      constexpr int word = S * 4 + (b >> 2);
      constexpr int sh = 8 * (b & 3);
      return (codes[word] >> sh) & 0xFFu;
    }
  } else {
    if (D == 8) {
      constexpr int b0 = 2 * KT;
      constexpr int v = S * 2 + (b0 >> 3);
      constexpr int word = v * 4 + ((b0 & 7) >> 1);
      return (codes[word] >> (qh_shift << 1)) & 0xFFFFu;  // 16*(q>>1)
    } else {
      constexpr int b = (D == 16) ? KT : (KT >> 1);
      constexpr int v = S * 2 + (b >> 3);
      constexpr int word = v * 4 + ((b & 7) >> 1);
      constexpr int sh = 16 * (b & 1);
      return (codes[word] >> sh) & 0xFFFFu;
    }
  }
}

// Decode the lane's two bf16x2 words of one row for k-tile KT:
// out[0] = columns 4q, 4q+1; out[1] = columns 4q+2, 4q+3.
template <int D, int R, int IDW, bool REPL, int KT, int V>
__device__ __forceinline__ void decode_row(uint32_t (&out)[2], const uint32_t (&codes)[V * 4], uint32_t cb_base,
                                           int stage_bytes, uint32_t rho2, int qh_shift) {
  using L = CbLayout<D, REPL>;
  constexpr int half_off = (D == 32) ? (KT & 1) * L::kHalfStride : 0;
  if (R == 1) {
    const uint32_t id = extract_id<D, IDW, KT, 0, V>(codes, qh_shift);
    const uint2 p = lds_v2(cb_base + id * L::kEntryStride + half_off);
    out[0] = mul_bf16x2_rn(p.x, rho2);
    out[1] = mul_bf16x2_rn(p.y, rho2);
  } else {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int s = 0; s < R; ++s) {
      uint32_t id;
      if (s == 0) id = extract_id<D, IDW, KT, 0, V>(codes, qh_shift);
      if (s == 1) id = extract_id<D, IDW, KT, 1, V>(codes, qh_shift);
      if (s == 2) id = extract_id<D, IDW, KT, 2, V>(codes, qh_shift);
      if (s == 3) id = extract_id<D, IDW, KT, 3, V>(codes, qh_shift);
      const uint2 p = lds_v2(cb_base + s * stage_bytes + id * L::kEntryStride + half_off);
      s0 = add_f32_f16((uint16_t)(p.x & 0xFFFFu), s0);
      s1 = add_f32_f16((uint16_t)(p.x >> 16), s1);
      s2 = add_f32_f16((uint16_t)(p.y & 0xFFFFu), s2);
      s3 = add_f32_f16((uint16_t)(p.y >> 16), s3);
    }
    out[0] = mul_bf16x2_rn(pack_bf16x2_rn(s0, s1), rho2);
    out[1] = mul_bf16x2_rn(pack_bf16x2_rn(s2, s3), rho2);
  }
}

}  // namespace wal
