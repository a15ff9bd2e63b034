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
// Numerics modes (template parameter NUM = NM | (F16 ? 4 : 0)):
//   NM = kExact        the sum above (reference per_group reconstruct_weight);
//   NM = kExactScaled  the same with per-stage fp32 scales, multi-stage tables
//                      staged as fp32 products RN(fp32(c) * scale);
//   NM = kFast         reference reconstruct_weight_fast (src/runtime.py:568-598):
//                      every stage table rounded to the weight type once
//                      (times the weight-type stage scale, rounded), the
//                      stages added in the weight type in order, then one
//                      multiply by the row scale: w = T(T(T(c_0) + T(c_1)) * T(rho)).
//   F16                weights, activations and MMA operands in fp16 instead of
//                      bf16 (the reference's forward in x.dtype: .to(float16)
//                      replaces .to(bfloat16) in every rounding above).
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

// (a0, a1) += fp32 of the two fp16 halves of h2 (lo half -> a0), round-to-nearest.
// The halves are split inside the asm so no 16-bit extraction is materialised.
__device__ __forceinline__ void add2_f32_f16x2(float& a0, float& a1, uint32_t h2) {
  asm("{\n .reg .f16 lo, hi;\n mov.b32 {lo, hi}, %2;\n add.rn.f32.f16 %0, lo, %0;\n add.rn.f32.f16 %1, hi, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(h2));
}

// fp16 bits -> bf16 bits of bf16_rn(+0.0f + fp32(h)) (first rounding, one stage)
__device__ __forceinline__ uint32_t preround_pair(uint32_t h2) {
  float lo = 0.0f, hi = 0.0f;
  add2_f32_f16x2(lo, hi, h2);
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

// (a0, a1) += (b0, b1), two fp32 round-to-nearest adds in one packed instruction
__device__ __forceinline__ void add_f32x2(float& a0, float& a1, float b0, float b1) {
  unsigned long long a, b;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

constexpr int kExact = 0, kExactScaled = 1, kFast = 2;
__host__ __device__ constexpr int num_mode(int nm, bool f16) { return nm | (f16 ? 4 : 0); }

// Packed pair arithmetic in the weight type (bf16 or fp16), round-to-nearest.
template <bool F16>
struct WT {
  static __device__ __forceinline__ uint32_t cvt2(float lo, float hi) {
    uint32_t d;
    if constexpr (F16) {
      asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    } else {
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    }
    return d;
  }
  static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (F16) {
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    } else {
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    }
    return d;
  }
  static __device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (F16) {
      asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    } else {
      asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    }
    return d;
  }
  // fp16 row scale -> both halves T(fp32(rho)) (for fp16 the value itself)
  static __device__ __forceinline__ uint32_t rho2(uint16_t rho_bits) {
    if constexpr (F16) {
      return (uint32_t)rho_bits | ((uint32_t)rho_bits << 16);
    } else {
      return rho_pair(rho_bits);
    }
  }
  // fp16 pair -> T pair of the plain conversion (sign of zero kept): the
  // reference's codebook.to(dtype)
  static __device__ __forceinline__ uint32_t from_f16x2(uint32_t h2) {
    if constexpr (F16) {
      return h2;
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&h2);
      return cvt2(__half2float(__low2half(h)), __half2float(__high2half(h)));
    }
  }
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (F16) {
      asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
          "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
          : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
          : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
      mma_bf16_16816(d, a, b0, b1);
    }
  }
};

// fp16 stage-scale bits of the fast mode: T(scale) as a pair.  The packed
// scales are fp32 values converted exactly from the reference's fp16 buffer.
template <bool F16>
__device__ __forceinline__ uint32_t scale2(float sc) {
  return WT<F16>::cvt2(sc, sc);
}

// ---------------------------------------------------------------------------
// Shared-memory codebook layout.
//
// An entry of d values is split into d/4 pieces of 8 bytes.  A lane always
// reads one piece per (row, stage, k-tile).  In the replicated layout every
// piece is stored once per lane class so that the 16 lanes of a half-warp
// phase always hit 16 distinct bank pairs whatever ids they hold:
//   d = 8 : 8 copies x 16 B per stage entry, lane offset (r&3)*32 + q*8
//   d = 16: 4 copies x 32 B per stage entry, lane offset (r&3)*32 + q*8
//   d = 32: 4 copies x 64 B per stage entry (second 16 columns at +128 B)
// Replicated entry rows are 256 bytes (two stages side by side for d = 8/16,
// one stage for d = 32), so the byte address of a lane's piece is
//   id * 256 + lane_offset + constant
// and one byte permute builds id * 256 + lane_offset from the packed id word
// (id byte -> byte 1, lane offset -> byte 0): no multiply, no add per gather.
// The plain layout stores each entry once (entry stride 2*d bytes) and is used
// when replication does not fit (large routed codebooks).
// ---------------------------------------------------------------------------
// Scaled multi-stage tables (per-stage fp32 scales) use an fp32 replicated
// layout: a lane's four columns are 16 bytes of fp32; the 8 lanes of a
// quarter-warp phase of a 128-bit load are 8 lane classes (r & 1) * 4 + q, each
// with its own 16-byte copy of the columns it reads (d = 8: half q & 1 of the
// entry; d = 16: quarter q; d = 32: quarter q of 16-column half kt & 1, halves
// 128 bytes apart).  Entry rows keep 128 bytes per stage (per half for
// d = 32) and the same id * 256 addressing, lane offset ((r & 1) * 4 + q) * 16.
template <int D, bool REPL, bool F32 = false>
struct CbLayout {
  static constexpr int kPieces = D / 4;
  static constexpr int kCopies = REPL ? (D == 8 ? 8 : 4) : 1;
  static constexpr int kStagesPerRow = REPL ? (D == 32 ? 1 : 2) : 1;
  static constexpr int kEntryStride = REPL ? 256 : 2 * D;
  static constexpr int kHalfStride = REPL ? 128 : 32;  // only D == 32 uses it
  static constexpr int kTableBytesRepl = 256 * 256;
  __host__ __device__ static constexpr int tables(int R) { return (R + kStagesPerRow - 1) / kStagesPerRow; }
  // multi-stage codebooks have at most 256 entries, so plain stages sit 256 entries apart
  __host__ __device__ static constexpr int total_bytes(int R, int entries) {
    return REPL ? tables(R) * kTableBytesRepl : (R == 1 ? entries * D * 2 : R * 256 * D * 2);
  }
  // constant byte offset of stage s inside the staged codebooks
  __host__ __device__ static constexpr int stage_offset(int s) {
    return REPL ? (s / kStagesPerRow) * kTableBytesRepl + (s % kStagesPerRow) * 128 : s * 256 * D * 2;
  }
  __device__ static int piece_offset(int s, int e, int j, int c, int entries) {
    (void)entries;
    if (!REPL) return stage_offset(s) + (e * kPieces + j) * 8;
    int inner;
    if (D == 8) {
      inner = c * 16 + j * 8;
    } else if (D == 16) {
      inner = c * 32 + j * 8;
    } else {
      inner = (j >> 2) * 128 + c * 32 + (j & 3) * 8;
    }
    return stage_offset(s) + e * 256 + inner;
  }
  __device__ static int lane_offset(int r, int q) {
    if (F32) return ((r & 1) * 4 + q) * 16;
    if (REPL) return (r & 3) * 32 + q * 8;
    return D == 8 ? (q & 1) * 8 : q * 8;
  }
};

__device__ __forceinline__ void cp_async_16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gptr));
}

// L2 cache policies: codebooks and activations are re-read by every CTA (and
// by the next launch), the id stream is read once.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cp_async_16_hint(uint32_t saddr, const void* gptr, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(gptr), "l"(pol));
}

__device__ __forceinline__ void cp_async_8(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(saddr), "l"(gptr));
}

// Zero-filling copies: only the first src_bytes are read, the rest of the
// destination is written as zeros (src_bytes = 0 reads nothing).
__device__ __forceinline__ void cp_async_16_zfill(uint32_t saddr, const void* gptr, uint32_t src_bytes, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(saddr), "l"(gptr),
               "r"(src_bytes), "l"(pol));
}
__device__ __forceinline__ void cp_async_8_zfill(uint32_t saddr, const void* gptr, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(saddr), "l"(gptr), "r"(src_bytes));
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }

// One-stage tables with a stage scale: the staged value is
// T(+0.0f + RN(fp32(c) * scale)).  Applied in place after the plain
// staging copied the raw fp16 entries (called instead of the unscaled
// pre-rounding).
template <bool F16 = false>
__device__ __forceinline__ uint32_t preround_pair_scaled(uint32_t h2, float sc) {
  const __half2 h = *reinterpret_cast<const __half2*>(&h2);
  const float lo = __fadd_rn(0.0f, __fmul_rn(__half2float(__low2half(h)), sc));
  const float hi = __fadd_rn(0.0f, __fmul_rn(__half2float(__high2half(h)), sc));
  return WT<F16>::cvt2(lo, hi);
}

// First rounding of a one-stage table in the weight type: T(+0.0f + fp32(c)).
template <bool F16>
__device__ __forceinline__ uint32_t preround_pair_t(uint32_t h2) {
  float lo = 0.0f, hi = 0.0f;
  add2_f32_f16x2(lo, hi, h2);
  return WT<F16>::cvt2(lo, hi);
}

// In-place transform of one staged 32-bit word (two fp16 entries) of stage s.
//   exact, one stage:          first rounding (optionally after the fp32 stage scale)
//   fast, any stage count:     T(c), times T(scale_s) rounded when scales exist
//   exact, several stages:     raw fp16 (summed in fp32 by the decode)
template <int R, int NM, bool F16>
__device__ __forceinline__ uint32_t staged_word(uint32_t h2, const float* scales, int s) {
  if constexpr (NM == kFast) {
    uint32_t v = WT<F16>::from_f16x2(h2);
    if (scales) v = WT<F16>::mul2(v, scale2<F16>(scales[s]));
    return v;
  } else if constexpr (R == 1) {
    return scales ? preround_pair_scaled<F16>(h2, scales[0]) : preround_pair_t<F16>(h2);
  } else {
    return h2;
  }
}

// 16-byte unit i of one stage's replicated table: entry e, run (16-byte
// piece of the entry) and byte offset inside the entry's 256-byte row.  The
// units of an entry are numbered so that consecutive lanes write consecutive
// 16-byte slots of a 128-byte row (copies of a run side by side), so a warp's
// stores into the table never conflict.
template <int D>
struct ReplUnit {
  static constexpr int kRuns = D / 8;
  static constexpr int kCopies = D == 8 ? 8 : 4;
  static constexpr int kUnits = kRuns * kCopies;  // per entry: 8 (D = 8, 16) or 16 (D = 32)
  static constexpr int kCopyStride = D == 8 ? 16 : 32;
  // copy c of the run sits at off; copy 0 of the same run at off - c * kCopyStride
  __device__ __forceinline__ static void decode(int i, int& e, int& c, int& off) {
    e = i / kUnits;
    const int u = i - e * kUnits;
    if constexpr (D == 32) {  // half h, copy c, run-in-half b: h * 128 + c * 32 + b * 16
      c = (u >> 1) & 3;
      off = (u >> 3) * 128 + c * 32 + (u & 1) * 16;
    } else if constexpr (D == 16) {  // copy c, run: c * 32 + run * 16
      c = u >> 1;
      off = u * 16;
    } else {  // copy c: c * 16
      c = u;
      off = u * 16;
    }
  }
};

__device__ __forceinline__ uint4 ldg16_hint(const void* p, uint64_t pol) {
  uint4 v;
  asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;\n"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

template <int R, int NM, bool F16>
__device__ __forceinline__ void staged_vec(uint4& v, const float* scales, int s) {
  v.x = staged_word<R, NM, F16>(v.x, scales, s);
  v.y = staged_word<R, NM, F16>(v.y, scales, s);
  v.z = staged_word<R, NM, F16>(v.z, scales, s);
  v.w = staged_word<R, NM, F16>(v.w, scales, s);
}

// Stage R codebooks of one group (fp16 [R][entries][D] in global memory) into
// shared memory, in two steps so the copies overlap other prologue work:
//   stage_codebooks_issue  - every 16-byte run of an entry is fetched with
//                            cp.async into its copy-0 position (not committed;
//                            plain layouts that need converting are skipped);
//   stage_codebooks_finish - after the caller's cp.async wait + __syncthreads:
//                            replicated layouts: copy 0 is expanded into the
//                            other copies, converted on the way when the
//                            numerics need it (staged_word: pre-rounding of
//                            one-stage tables, fast-mode tables), with lanes
//                            mapped so that each warp store fills whole
//                            128-byte rows (copy 0 itself is converted last,
//                            from copy 1); plain layouts that need converting
//                            are read here with 16-byte loads, 8 per thread in
//                            flight, converted in registers and stored once.
//                            Follow it with __syncthreads().
// (Expanding entry by entry made the 32 lanes of a warp store into the same
// four banks: 2.2 us per launch for a d = 8 table; fetching every copy from
// global memory instead made all CTAs re-read the same few L2 lines eight
// times over and tripled the launch; landing a 128 KB routed table first and
// converting it in place cost 1.3 us.)
template <int D, int R, bool REPL, int NM = kExact, bool F16 = false>
__device__ void stage_codebooks_issue(uint8_t* cb, const uint16_t* __restrict__ books, int entries) {
  using L = CbLayout<D, REPL>;
  constexpr bool kConvert = NM == kFast || R == 1;
  if constexpr (REPL || !kConvert) {
    constexpr int kRuns = D / 8;
    const uint32_t base = smem_u32(cb);
    const uint64_t keep = l2_policy_evict_last();
#pragma unroll
    for (int s = 0; s < R; ++s) {
      const uint16_t* sbooks = books + (size_t)s * entries * D;
      for (int e = threadIdx.x; e < entries; e += blockDim.x) {
#pragma unroll
        for (int run = 0; run < kRuns; ++run)
          cp_async_16_hint(base + L::piece_offset(s, e, 2 * run, 0, entries), sbooks + (size_t)e * D + 8 * run, keep);
      }
    }
  }
}

template <int D, int R, bool REPL, int NM = kExact, bool F16 = false>
__device__ void stage_codebooks_finish(uint8_t* cb, const uint16_t* __restrict__ books, int entries,
                                       const float* scales = nullptr) {
  using L = CbLayout<D, REPL>;
  constexpr bool kConvert = NM == kFast || R == 1;
  if constexpr (REPL) {
    using U = ReplUnit<D>;
    auto expand = [&](const float* sc) {
#pragma unroll
      for (int s = 0; s < R; ++s) {
        uint8_t* sbase = cb + L::stage_offset(s);
        for (int i = threadIdx.x; i < entries * U::kUnits; i += blockDim.x) {
          int e, c, off;
          U::decode(i, e, c, off);
          if (c == 0) continue;  // the source
          uint8_t* row = sbase + e * 256;
          uint4 v = *reinterpret_cast<const uint4*>(row + off - c * U::kCopyStride);
          if constexpr (kConvert) staged_vec<R, NM, F16>(v, sc, s);
          *reinterpret_cast<uint4*>(row + off) = v;
        }
      }
    };
    if (scales) expand(scales);
    else expand(nullptr);
    if constexpr (kConvert) {
      __syncthreads();  // every copy-0 read above is done; copy 1 holds the converted runs
      constexpr int kRuns = D / 8;
#pragma unroll
      for (int s = 0; s < R; ++s) {
        uint8_t* sbase = cb + L::stage_offset(s);
        for (int i = threadIdx.x; i < entries * kRuns; i += blockDim.x) {
          const int e = i / kRuns, run = i - e * kRuns;
          const int off0 = D == 32 ? (run >> 1) * 128 + (run & 1) * 16 : run * 16;
          uint8_t* row = sbase + e * 256;
          *reinterpret_cast<uint4*>(row + off0) = *reinterpret_cast<const uint4*>(row + off0 + U::kCopyStride);
        }
      }
    }
  } else if constexpr (kConvert) {
    // plain layout: entry e of stage s is D contiguous values, so a stage is
    // one contiguous run of 16-byte vectors
    constexpr int kBatch = 8;
    const uint64_t keep = l2_policy_evict_last();
    auto load_convert = [&](const float* sc) {
#pragma unroll
      for (int s = 0; s < R; ++s) {
        const uint4* src = reinterpret_cast<const uint4*>(books + (size_t)s * entries * D);
        uint4* dst = reinterpret_cast<uint4*>(cb + L::stage_offset(s));
        const int n16 = entries * D / 8;
        for (int i0 = threadIdx.x; i0 < n16; i0 += kBatch * blockDim.x) {
          uint4 v[kBatch];
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            const int i = i0 + k * blockDim.x;
            if (i < n16) v[k] = ldg16_hint(src + i, keep);
          }
#pragma unroll
          for (int k = 0; k < kBatch; ++k) {
            const int i = i0 + k * blockDim.x;
            if (i < n16) {
              staged_vec<R, NM, F16>(v[k], sc, s);
              dst[i] = v[k];
            }
          }
        }
      }
    };
    if (scales) load_convert(scales);
    else load_convert(nullptr);
  }
}

// fp32 replicated tables for scaled multi-stage codebooks: every thread
// converts whole entries, value RN(fp32(c) * scale[s]) (stage 0 also + 0.0f,
// as the reference's sum starts from +0.0), and writes the 8 lane-class
// copies.  Follow with __syncthreads().
template <int D, int R>
__device__ void stage_codebooks_scaled(uint8_t* cb, const uint16_t* __restrict__ books, const float* scales,
                                       int entries) {
  using L = CbLayout<D, true, true>;
  for (int s = 0; s < R; ++s) {
    const float sc = scales[s];
    for (int e = threadIdx.x; e < entries; e += blockDim.x) {
      const uint16_t* src = books + ((size_t)s * entries + e) * D;
      float v[D];
#pragma unroll
      for (int j = 0; j < D; j += 8) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + j));
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[t]);
          v[j + 2 * t] = __fmul_rn(__half2float(__low2half(h)), sc);
          v[j + 2 * t + 1] = __fmul_rn(__half2float(__high2half(h)), sc);
        }
      }
      if (s == 0) {
#pragma unroll
        for (int j = 0; j < D; ++j) v[j] = __fadd_rn(0.0f, v[j]);
      }
      uint8_t* row = cb + L::stage_offset(s) + e * 256;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (D == 8) {
          const int h = (c & 1) * 4;
          *reinterpret_cast<float4*>(row + c * 16) = make_float4(v[h], v[h + 1], v[h + 2], v[h + 3]);
        } else if (D == 16) {
          const int q4 = (c & 3) * 4;
          *reinterpret_cast<float4*>(row + c * 16) = make_float4(v[q4], v[q4 + 1], v[q4 + 2], v[q4 + 3]);
        } else {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int b = hf * 16 + (c & 3) * 4;
            *reinterpret_cast<float4*>(row + hf * 128 + c * 16) = make_float4(v[b], v[b + 1], v[b + 2], v[b + 3]);
          }
        }
      }
    }
  }
}

// One-call staging for kernels without other prologue work.
template <int D, int R, bool REPL, int NUM = 0>
__device__ void stage_codebooks(uint8_t* cb, const uint16_t* __restrict__ books, int entries,
                                const float* scales = nullptr) {
  constexpr int NM = NUM & 3;
  constexpr bool F16 = (NUM & 4) != 0;
  if constexpr (NM == kExactScaled && REPL && R > 1) {
    stage_codebooks_scaled<D, R>(cb, books, scales, entries);
    return;
  }
  stage_codebooks_issue<D, R, REPL, NM, F16>(cb, books, entries);
  cp_async_wait_all();
  __syncthreads();
  stage_codebooks_finish<D, R, REPL, NM, F16>(cb, books, entries, scales);
}

// ---------------------------------------------------------------------------
// Id extraction from one row's chunk registers.
// codes[v*4 + w] holds 32-bit word w of 16-byte vector v of this row's chunk
// (vector v = stage * idw + half).  Block-in-chunk for k-tile KT of lane q:
//   D = 8 : 2*KT + (q >> 1)      D = 16: KT      D = 32: KT >> 1
// Lane-dependent byte selection (D = 8) goes through a precomputed
// __byte_perm selector: sel8[KT & 1] = 0x4440 + (2*(KT&1) + (q>>1)) for 1-byte
// ids, sel16 = (q>>1) ? 0x4432 : 0x4410 for 2-byte ids.
// ---------------------------------------------------------------------------
struct LaneSel {
  uint32_t sel8[2];   // id byte -> byte 0
  uint32_t self8[2];  // id byte -> byte 1, lane offset (second operand, byte 0) -> byte 0
  uint32_t sel16;
  uint32_t lane_off;  // replicated-layout lane offset (< 256)
  __device__ LaneSel(int r, int q, bool f32 = false) {
    const uint32_t qh = (uint32_t)(q >> 1);
    sel8[0] = 0x4440u + qh;
    sel8[1] = 0x4442u + qh;
    self8[0] = 0x5504u | (qh << 4);
    self8[1] = 0x5504u | ((2u + qh) << 4);
    sel16 = qh ? 0x4432u : 0x4410u;
    lane_off = f32 ? (uint32_t)(((r & 1) * 4 + q) * 16) : (uint32_t)((r & 3) * 32 + q * 8);
  }
};

// Replicated layouts: byte address id * 256 + lane offset from one permute.
template <int D, int KT, int S, int NW>
__device__ __forceinline__ uint32_t id_addr256(const uint32_t (&codes)[NW], const LaneSel& ls) {
  if (D == 8) {
    return __byte_perm(codes[S * 4 + (KT >> 1)], ls.lane_off, ls.self8[KT & 1]);
  } else {
    constexpr int b = (D == 16) ? KT : (KT >> 1);
    return __byte_perm(codes[S * 4 + (b >> 2)], ls.lane_off, 0x5504u | ((uint32_t)(b & 3) << 4));
  }
}

template <int D, int IDW, int KT, int S, int NW>
__device__ __forceinline__ uint32_t extract_id(const uint32_t (&codes)[NW], const LaneSel& ls) {
  if (IDW == 1) {
    if (D == 8) {
      return __byte_perm(codes[S * 4 + (KT >> 1)], 0u, ls.sel8[KT & 1]);
    } else {
      constexpr int b = (D == 16) ? KT : (KT >> 1);
      return __byte_perm(codes[S * 4 + (b >> 2)], 0u, 0x4440u + (b & 3));
    }
  } else {
    if (D == 8) {
      constexpr int b0 = 2 * KT;
      return __byte_perm(codes[(S * 2 + (b0 >> 3)) * 4 + ((b0 & 7) >> 1)], 0u, ls.sel16);
    } else {
      constexpr int b = (D == 16) ? KT : (KT >> 1);
      return __byte_perm(codes[(S * 2 + (b >> 3)) * 4 + ((b & 7) >> 1)], 0u, (b & 1) ? 0x4432u : 0x4410u);
    }
  }
}

// Decode the lane's two bf16x2 words of one row for k-tile KT:
// out[0] = columns 4q, 4q+1; out[1] = columns 4q+2, 4q+3 (both already
// multiplied by the row scale with the second rounding).
// cbl = shared codebook base + this lane's offset; SB = bytes per stage.
template <int OFF>
__device__ __forceinline__ uint2 lds64(uint32_t saddr) {
  uint2 v;
  asm("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(saddr), "n"(OFF));
  return v;
}

template <int OFF>
__device__ __forceinline__ float4 lds128(uint32_t saddr) {
  float4 v;
  asm("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4+%5];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(saddr), "n"(OFF));
  return v;
}

// Ordered variant for buffers written earlier in the kernel (activations).
template <int OFF>
__device__ __forceinline__ uint2 lds64_ordered(uint32_t saddr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(saddr), "n"(OFF));
  return v;
}

template <int D, int R, int IDW, bool REPL, int KT, int NW, int E>
__device__ __forceinline__ uint32_t piece_addr(const uint32_t (&codes)[NW], uint32_t cb, const LaneSel& ls,
                                               uint32_t cbl) {
  using L = CbLayout<D, REPL>;
  if constexpr (REPL && IDW == 1) {
    return cb + id_addr256<D, KT, E, NW>(codes, ls);
  } else {
    return cbl + extract_id<D, IDW, KT, E, NW>(codes, ls) * L::kEntryStride;
  }
}

// Decode the lane's two weight-type words of one row for k-tile KT:
// out[0] = columns 4q, 4q+1; out[1] = columns 4q+2, 4q+3 (both already
// multiplied by the row scale with the final rounding).
// cb = shared codebook base, cbl = cb + this lane's offset (plain layouts).
template <int D, int R, int IDW, bool REPL, int KT, int NW, int NUM = 0>
__device__ __forceinline__ void decode_row(uint32_t (&out)[2], const uint32_t (&codes)[NW], uint32_t cb, uint32_t cbl,
                                           uint32_t rho2, const LaneSel& ls) {
  using L = CbLayout<D, REPL>;
  constexpr int NM = NUM & 3;
  constexpr bool F16 = (NUM & 4) != 0;
  using T = WT<F16>;
  constexpr int half_off = (D == 32) ? (KT & 1) * L::kHalfStride : 0;
  if constexpr (NM == kExactScaled && REPL && R > 1) {  // scaled fp32 tables (LaneSel built with f32 = true)
    float4 t = lds128<L::stage_offset(0) + half_off>(cb + id_addr256<D, KT, 0, NW>(codes, ls));
#pragma unroll
    for (int s = 1; s < R; ++s) {
      float4 u;
      if (s == 1) u = lds128<L::stage_offset(1) + half_off>(cb + id_addr256<D, KT, 1, NW>(codes, ls));
      if (s == 2) u = lds128<L::stage_offset(2) + half_off>(cb + id_addr256<D, KT, 2, NW>(codes, ls));
      if (s == 3) u = lds128<L::stage_offset(3) + half_off>(cb + id_addr256<D, KT, 3, NW>(codes, ls));
      add_f32x2(t.x, t.y, u.x, u.y);
      add_f32x2(t.z, t.w, u.z, u.w);
    }
    out[0] = T::mul2(T::cvt2(t.x, t.y), rho2);
    out[1] = T::mul2(T::cvt2(t.z, t.w), rho2);
  } else if constexpr (R == 1 || NM == kFast) {
    // tables already in the weight type: one stage is the (pre-rounded) value,
    // the fast mode adds the stages in the weight type, in order
    uint2 acc = lds64<L::stage_offset(0) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 0>(codes, cb, ls, cbl));
#pragma unroll
    for (int s = 1; s < R; ++s) {
      uint2 p;
      if (s == 1) p = lds64<L::stage_offset(1) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 1>(codes, cb, ls, cbl));
      if (s == 2) p = lds64<L::stage_offset(2) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 2>(codes, cb, ls, cbl));
      if (s == 3) p = lds64<L::stage_offset(3) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 3>(codes, cb, ls, cbl));
      acc.x = T::add2(acc.x, p.x);
      acc.y = T::add2(acc.y, p.y);
    }
    out[0] = T::mul2(acc.x, rho2);
    out[1] = T::mul2(acc.y, rho2);
  } else {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int s = 0; s < R; ++s) {
      uint2 p;
      if (s == 0) p = lds64<L::stage_offset(0) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 0>(codes, cb, ls, cbl));
      if (s == 1) p = lds64<L::stage_offset(1) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 1>(codes, cb, ls, cbl));
      if (s == 2) p = lds64<L::stage_offset(2) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 2>(codes, cb, ls, cbl));
      if (s == 3) p = lds64<L::stage_offset(3) + half_off>(piece_addr<D, R, IDW, REPL, KT, NW, 3>(codes, cb, ls, cbl));
      add2_f32_f16x2(s0, s1, p.x);
      add2_f32_f16x2(s2, s3, p.y);
    }
    out[0] = T::mul2(T::cvt2(s0, s1), rho2);
    out[1] = T::mul2(T::cvt2(s2, s3), rho2);
  }
}

}  // namespace wal
