// Decode attention for the Llama-shaped stacks: one new query token per
// sequence, grouped-query heads, softmax(q k^T * scale) v over cache positions
// [0, n).  Replaces the PyTorch scaled_dot_product_attention call (and the copy
// of its output) in the decode step; no reference counterpart (the reference
// runs Hugging Face attention).
//
// Split-K over positions: CTA (b, kv head, split) handles up to 128 positions
// for all G = hq / hkv query heads that share the kv head.  The split's K and
// V rows are copied to shared memory (cp.async, zero-filled past the end);
// scores and the weighted values run on the tensor cores (mma.sync m16n8k16,
// bf16 in, fp32 accumulate) with the G heads as the rows of the A tiles, each
// warp owning 32 positions; the exp2 weights P are re-packed from the score
// fragments into bf16 A fragments of the P.V product without leaving
// registers.  Each CTA keeps (max, sum, un-normalised output) per head in
// fp32 and writes them to a workspace slot.  The last CTA of each (b, kv head)
// to finish (a counter in the workspace, returned to zero) merges the splits in
// split order - deterministic - and writes the bf16 output row in the layout
// the o-projection reads.  Softmax uses base-2 exponentials of scores
// multiplied by scale * log2(e).
#include "../../include/wal_rvq.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace {

constexpr int kThreads = 128;     // 4 warps
constexpr int kMaxChunk = kThreads;  // positions per split: 32 per warp

struct AttnParams {
  const uint16_t* q;
  long long ld_q;
  const uint16_t* k;
  const uint16_t* v;
  long long cache_len;
  int n, hq, hkv, hd, nsplit, chunk;
  float qscale;  // scale * log2(e)
  uint16_t* out;
  long long ld_out;
  float* part;        // [B * hkv][nsplit][G][hd] un-normalised outputs
  float2* stats;      // [B * hkv][nsplit][G] (max, sum of exp2)
  unsigned* counter;  // [B * hkv]
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t v;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(v) : "f"(hi), "f"(lo));
  return v;
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // A rows 8..15 are zero (at most 8 query heads share a kv head)
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&m)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(m[0]), "=r"(m[1]), "=r"(m[2]), "=r"(m[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&m)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(m[0]), "=r"(m[1]), "=r"(m[2]), "=r"(m[3])
               : "r"(addr));
}

// Merge of a (sequence, kv head)'s splits by its last CTA: split weights
// exp2(m_s - M), the normalising sum, then the weighted sum of the split
// outputs in split order (deterministic), written as the bf16 output row.
// scratch: shared memory for 2 * nsplit * G floats.
template <int HD, int G>
__device__ __forceinline__ void merge_splits(const AttnParams& p, int bh, int b, int kvh, float* scratch) {
  constexpr int NW = kThreads / 32;
  __shared__ float inv_l[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = p.nsplit;
  float* wgt = scratch;           // [nsplit][G] exp2(m_s - M)
  float* lsm = wgt + ns * G;      // [nsplit][G] split sums
  const float2* st = p.stats + (long long)bh * ns * G;
  for (int i = tid; i < ns * G; i += kThreads) {
    const float2 v = __ldcg(st + i);
    wgt[i] = v.x;
    lsm[i] = v.y;
  }
  __syncthreads();
  for (int g = warp; g < G; g += NW) {
    float m = -INFINITY;
    for (int s2 = lane; s2 < ns; s2 += 32) m = fmaxf(m, wgt[s2 * G + g]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int s2 = lane; s2 < ns; s2 += 32) {
      const float w = exp2f(wgt[s2 * G + g] - m);
      wgt[s2 * G + g] = w;
      l = fmaf(w, lsm[s2 * G + g], l);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) inv_l[g] = 1.f / l;
  }
  __syncthreads();
  const float4* src = reinterpret_cast<const float4*>(p.part + (long long)bh * ns * G * HD);
  uint16_t* orow = p.out + (long long)b * p.ld_out + (long long)kvh * G * HD;
  for (int i = tid; i < G * HD / 4; i += kThreads) {
    const int g = i / (HD / 4);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int s2 = 0; s2 < ns; ++s2) {
      const float w = wgt[s2 * G + g];
      const float4 c = __ldcg(src + (long long)s2 * (G * HD / 4) + i);
      a.x = fmaf(w, c.x, a.x); a.y = fmaf(w, c.y, a.y); a.z = fmaf(w, c.z, a.z); a.w = fmaf(w, c.w, a.w);
    }
    const float inv = inv_l[g];
    const uint32_t lo = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.x * inv)) |
                        ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.y * inv)) << 16);
    const uint32_t hi = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.z * inv)) |
                        ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.w * inv)) << 16);
    *reinterpret_cast<uint2*>(orow + i * 4) = make_uint2(lo, hi);
  }
}

// Tensor-core decode attention for one (sequence, kv head, split): the G query
// heads are the rows of m16n8k16 tiles (rows >= G are zero), positions the
// columns of the score tiles and the k dimension of the P.V tiles.  K and V
// rows of the split are staged in shared memory with 16-byte piece c of row t
// at piece c ^ (t & 7), so ldmatrix (K) and ldmatrix.trans (V) read eight rows
// without bank conflicts.  Each warp owns 32 positions.
template <int HD, int G>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ AttnParams p) {
  constexpr int KT = HD / 16;   // k-tiles of the head dimension
  constexpr int NT = HD / 8;    // n-tiles of the output
  constexpr int P16 = HD / 8;   // 16-byte pieces per row
  constexpr int PSH = HD == 128 ? 4 : 3;
  constexpr int NW = kThreads / 32;
  constexpr int RB = HD * 2;    // row bytes
  static_assert(NW * 32 == kMaxChunk, "one warp per 32 positions");
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float red[NW][8];
  __shared__ float stat[2][8];
  __shared__ int last;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.hkv, kvh = bh - b * p.hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, qd = lane & 3;
  const int t0 = split * p.chunk;
  const int len = min(p.n - t0, p.chunk);  // >= 1: the plan leaves no empty split
  // shared: V rows | K rows, the K region reused after the scores for the
  // warps' outputs [NW][G][HD] and the merge's split weights and sums
  const uint32_t vs_s = (uint32_t)__cvta_generic_to_shared(sm);
  const uint32_t ks_s = vs_s + kMaxChunk * RB;
  float* po = reinterpret_cast<float*>(sm + kMaxChunk * RB);
  const uint16_t* kb = p.k + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;
  const uint16_t* vb = p.v + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;

  // the cache and q come from earlier kernels of the step
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  // K rows, then V rows -> shared memory (rows >= len zero-filled), as two
  // copy groups: the scores and the softmax need only K, so they overlap V
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    const uint32_t base = kv == 0 ? ks_s : vs_s;
    const uint16_t* src = kv == 0 ? kb : vb;
    for (int i = tid; i < kMaxChunk * P16; i += kThreads) {
      const int t = i >> PSH, c = i & (P16 - 1);
      const uint32_t off = (uint32_t)(t * RB + ((c ^ (t & 7)) << 4));
      const bool in = t < len;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(base + off),
                   "l"(in ? src + (long long)t * HD + c * 8 : src), "r"(in ? 16u : 0u));
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  // q fragments (A rows = heads): dims kt*16 + 2*qd (+1) and + 8
  uint32_t qa[KT][2];
  const uint16_t* qrow = p.q + (long long)b * p.ld_q + (long long)(kvh * G + (r < G ? r : 0)) * HD;
#pragma unroll
  for (int kt = 0; kt < KT; ++kt) {
    qa[kt][0] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + kt * 16 + 2 * qd) : 0u;
    qa[kt][1] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + kt * 16 + 8 + 2 * qd) : 0u;
  }
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // K landed
  __syncthreads();

  // scores of the warp's 32 positions (4 n-tiles of 8): lane holds head r, positions 2qd, 2qd + 1
  const int wp0 = warp * 32;
  float s[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    const int row = wp0 + nt * 8 + (lane & 7);  // the row this lane addresses for ldmatrix
#pragma unroll
    for (int kt = 0; kt < KT; kt += 2) {
      uint32_t m[4];
      const int c = 2 * kt + (lane >> 3);
      ldsm_x4(ks_s + row * RB + ((c ^ (row & 7)) << 4), m);
      mma16816(s[nt], qa[kt][0], qa[kt][1], m[0], m[1]);
      mma16816(s[nt], qa[kt + 1][0], qa[kt + 1][1], m[2], m[3]);
    }
  }
  // scale, mask, split max per head
  float mx = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = wp0 + nt * 8 + 2 * qd + e;
      s[nt][e] = t < len ? s[nt][e] * p.qscale : -INFINITY;
      mx = fmaxf(mx, s[nt][e]);
    }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  if (qd == 0 && r < G) red[warp][r] = mx;
  __syncthreads();
  if (tid < G) {
    float m = red[0][tid];
#pragma unroll
    for (int w = 1; w < NW; ++w) m = fmaxf(m, red[w][tid]);
    stat[0][tid] = m;
  }
  __syncthreads();
  const float M = r < G ? stat[0][r] : 0.f;
  float l = 0.f;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      s[nt][e] = exp2f(s[nt][e] - M);  // masked positions: exp2(-inf) = 0
      l += s[nt][e];
    }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");  // V landed
  __syncthreads();  // red is reused; V visible to every warp
  if (qd == 0 && r < G) red[warp][r] = l;

  // P.V: the warp's 32 positions are two k-tiles; P re-packed as bf16 A fragments
  float o[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
    const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    const int row = wp0 + kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      uint32_t m[4];
      const int c = 2 * np + (lane >> 4);
      ldsm_x4_t(vs_s + row * RB + ((c ^ (row & 7)) << 4), m);
      mma16816(o[2 * np], a0, a2, m[0], m[1]);
      mma16816(o[2 * np + 1], a0, a2, m[2], m[3]);
    }
  }
  if (r < G) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float2*>(po + (warp * G + r) * HD + nt * 8 + 2 * qd) = make_float2(o[nt][0], o[nt][1]);
  }
  __syncthreads();
  // this split's slot: the warps' outputs summed in warp order, then (max, sum)
  const long long slot = (long long)bh * p.nsplit + split;
  float4* dst = reinterpret_cast<float4*>(p.part + slot * G * HD);
  for (int i = tid; i < G * HD / 4; i += kThreads) {
    float4 acc = reinterpret_cast<const float4*>(po)[i];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
      const float4 c = reinterpret_cast<const float4*>(po + w * G * HD)[i];
      acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w;
    }
    dst[i] = acc;
  }
  if (tid < G) {
    float ls = red[0][tid];
#pragma unroll
    for (int w = 1; w < NW; ++w) ls += red[w][tid];
    p.stats[slot * G + tid] = make_float2(stat[0][tid], ls);
  }
  // the last split of this (b, kv head) to finish merges
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.counter + bh, 1u);
    last = prev == (unsigned)(p.nsplit - 1);
    if (last) p.counter[bh] = 0u;  // ready for the next call
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  merge_splits<HD, G>(p, bh, b, kvh, po + NW * G * HD);
}

// Streaming variant: the split's positions pass through the CTA in stages of
// 64 (16 per warp), double-buffered, so the copy of stage c + 1 overlaps the
// scores and P.V of stage c and a CTA can cover a long split; each warp keeps
// its own running (max, sum, un-normalised output) per head across the stages
// (exp2 rescaling when its max grows), and the four warps are combined once at
// the end into the split's slot, in the format the merge reads.
constexpr int kStage = 64;

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) decode_attn_stream_kernel(const __grid_constant__ AttnParams p) {
  constexpr int KT = HD / 16;
  constexpr int NT = HD / 8;
  constexpr int P16 = HD / 8;
  constexpr int PSH = HD == 128 ? 4 : 3;
  constexpr int NW = kThreads / 32;
  constexpr int RB = HD * 2;
  constexpr int BUF = 2 * kStage * RB;  // one stage: K rows, then V rows
  static_assert(NW * 16 == kStage, "16 positions per warp and stage");
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float wst[NW][8][2];  // per warp and head: running max, sum
  __shared__ float stat[2][8];
  __shared__ int last;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.hkv, kvh = bh - b * p.hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = lane >> 2, qd = lane & 3;
  const int t0 = split * p.chunk;
  const int len = min(p.n - t0, p.chunk);  // >= 1: the plan leaves no empty split
  const int nst = (len + kStage - 1) / kStage;
  const uint32_t sm_s = (uint32_t)__cvta_generic_to_shared(sm);
  const uint16_t* kb = p.k + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;
  const uint16_t* vb = p.v + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;

  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  // stage c -> buffer c & 1: K rows then V rows (rows >= len zero-filled),
  // 16-byte piece j of row t at piece j ^ (t & 7)
  auto issue = [&](int c) {
    const uint32_t base = sm_s + (uint32_t)((c & 1) * BUF);
    const int tb = c * kStage;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const uint16_t* src = kv == 0 ? kb : vb;
      const uint32_t dst = base + (uint32_t)(kv * kStage * RB);
      for (int i = tid; i < kStage * P16; i += kThreads) {
        const int t = i >> PSH, j = i & (P16 - 1);
        const bool in = tb + t < len;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst + (uint32_t)(t * RB + ((j ^ (t & 7)) << 4))),
                     "l"(in ? src + (long long)(tb + t) * HD + j * 8 : src), "r"(in ? 16u : 0u));
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  issue(0);
  if (nst > 1) issue(1);
  uint32_t qa[KT][2];
  const uint16_t* qrow = p.q + (long long)b * p.ld_q + (long long)(kvh * G + (r < G ? r : 0)) * HD;
#pragma unroll
  for (int kt = 0; kt < KT; ++kt) {
    qa[kt][0] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + kt * 16 + 2 * qd) : 0u;
    qa[kt][1] = r < G ? *reinterpret_cast<const uint32_t*>(qrow + kt * 16 + 8 + 2 * qd) : 0u;
  }
  float mw = -INFINITY, lw = 0.f;  // this warp's running max and sum for head r
  float o[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  const int wp0 = warp * 16;
  for (int c = 0; c < nst; ++c) {
    if (c + 1 < nst) asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();  // stage c landed for every thread's copies
    const uint32_t ks = sm_s + (uint32_t)((c & 1) * BUF), vs = ks + (uint32_t)(kStage * RB);
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const int row = wp0 + nt * 8 + (lane & 7);
#pragma unroll
      for (int kt = 0; kt < KT; kt += 2) {
        uint32_t m[4];
        const int j = 2 * kt + (lane >> 3);
        ldsm_x4(ks + row * RB + ((j ^ (row & 7)) << 4), m);
        mma16816(s[nt], qa[kt][0], qa[kt][1], m[0], m[1]);
        mma16816(s[nt], qa[kt + 1][0], qa[kt + 1][1], m[2], m[3]);
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = c * kStage + wp0 + nt * 8 + 2 * qd + e;
        s[nt][e] = t < len ? s[nt][e] * p.qscale : -INFINITY;
        mx = fmaxf(mx, s[nt][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(mw, mx);
    const bool none = mn == -INFINITY;  // nothing valid seen by this warp yet
    const float alpha = none ? 1.f : exp2f(mw - mn);
    float ls = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[nt][e] = none ? 0.f : exp2f(s[nt][e] - mn);  // masked positions: exp2(-inf) = 0
        ls += s[nt][e];
      }
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    lw = fmaf(lw, alpha, ls);
    mw = mn;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      o[nt][0] *= alpha;
      o[nt][1] *= alpha;
    }
    // P.V: the warp's 16 positions are one k-tile; P re-packed as bf16 A fragments
    const uint32_t a0 = pack_bf16x2(s[0][0], s[0][1]);
    const uint32_t a2 = pack_bf16x2(s[1][0], s[1][1]);
    const int row = wp0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      uint32_t m[4];
      const int j = 2 * np + (lane >> 4);
      ldsm_x4_t(vs + row * RB + ((j ^ (row & 7)) << 4), m);
      mma16816(o[2 * np], a0, a2, m[0], m[1]);
      mma16816(o[2 * np + 1], a0, a2, m[2], m[3]);
    }
    __syncthreads();  // every warp is done with buffer c & 1
    if (c + 2 < nst) issue(c + 2);
  }
  // combine the warps: M = max of their maxima, each scaled by exp2(m_w - M)
  if (qd == 0 && r < G) {
    wst[warp][r][0] = mw;
    wst[warp][r][1] = lw;
  }
  __syncthreads();
  if (tid < G) {
    float M = wst[0][tid][0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, wst[w][tid][0]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w)
      if (wst[w][tid][0] != -INFINITY) L = fmaf(exp2f(wst[w][tid][0] - M), wst[w][tid][1], L);
    stat[0][tid] = M;
    stat[1][tid] = L;
  }
  __syncthreads();
  float* po = reinterpret_cast<float*>(sm);  // [NW][G][HD]: the stage buffers are free now
  if (r < G) {
    const float wsc = mw == -INFINITY ? 0.f : exp2f(mw - stat[0][r]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float2*>(po + (warp * G + r) * HD + nt * 8 + 2 * qd) = make_float2(o[nt][0] * wsc, o[nt][1] * wsc);
  }
  __syncthreads();
  const long long slot = (long long)bh * p.nsplit + split;
  float4* dst = reinterpret_cast<float4*>(p.part + slot * G * HD);
  for (int i = tid; i < G * HD / 4; i += kThreads) {
    float4 acc = reinterpret_cast<const float4*>(po)[i];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
      const float4 cc = reinterpret_cast<const float4*>(po + w * G * HD)[i];
      acc.x += cc.x; acc.y += cc.y; acc.z += cc.z; acc.w += cc.w;
    }
    dst[i] = acc;
  }
  if (tid < G) p.stats[slot * G + tid] = make_float2(stat[0][tid], stat[1][tid]);
  // the last split of this (b, kv head) to finish merges
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(p.counter + bh, 1u);
    last = prev == (unsigned)(p.nsplit - 1);
    if (last) p.counter[bh] = 0u;  // ready for the next call
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  merge_splits<HD, G>(p, bh, b, kvh, po + NW * G * HD);
}

// Split count before rounding the chunk to a multiple of 4: the fewest splits
// of at most kMaxChunk positions.  Measured on B200 (8B / 70B shard heads,
// 2048-4096 positions, batch 1-8), more splits than that only lengthen the
// merge, which the last CTA of a (sequence, kv head) runs over every split:
// e.g. 70B heads at tensor parallelism 8 (one kv head, 4096 positions) take
// 9.7 us with 32 splits against 21.7 us with 128.  Non-decreasing in n, so it
// also bounds plan()'s split count for every n' <= n (the chunk rounding in
// plan() only lowers it).
long long split_bound(long long B, int hkv, long long n) {
  (void)B;
  (void)hkv;
  const long long s = (n + kMaxChunk - 1) / kMaxChunk;
  return s < 1 ? 1 : s;
}

void plan(long long B, int hkv, long long n, int* nsplit, int* chunk) {
  long long s = split_bound(B, hkv, n);
  // Many (sequence, kv head) pairs: fewer, longer splits that stream through
  // two stage buffers, about 2.6 CTAs per SM, and past one wave of 3 CTAs per
  // SM not just above a wave boundary.  Measured on B200 (us, this split count
  // against the fewest 128-position splits): 8B heads at 2048 positions, batch
  // 4 / 8 / 32: 11.1 / 15.9 / 51.3 against 11.7 / 16.4 / 56.5; 70B heads at
  // 4096 positions, batch 16 / 64: 49.9 / 181 against 68.1 / 235.
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long bh = B * hkv, want = (long long)sms * 13 / 5, slots = 3LL * sms;
  if (bh * s > want) {
    const long long s0 = s;
    s = (want + bh - 1) / bh;
    while (s < s0 && bh * s > slots && (bh * s) % slots < slots * 2 / 5) ++s;
  }
  long long c = ((n + s - 1) / s + 3) & ~3LL;  // multiple of 4 keeps the shared-memory regions 16-byte aligned
  s = (n + c - 1) / c;
  *nsplit = (int)s;
  *chunk = (int)c;
}

// Scratch of wal_decode_attention_static, for callers that cannot allocate
// device memory: 4 MiB that every GPU loading this library keeps until the
// process exits.  The merge counters occupy a fixed region at the front (each
// call clears the ones it uses); partial outputs and stats follow.  Host code
// must not pass this name to a kernel: it reaches the device address through
// cudaGetSymbolAddress, once per device.
constexpr size_t kStaticScratchBytes = 4u << 20;  // 4 MiB
constexpr size_t kStaticCounters = 4096;         // max B * hkv
constexpr size_t kStaticDataOffset = kStaticCounters * sizeof(unsigned);
static __device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

size_t part_bytes(long long B, int hkv, int nsplit, int G, int hd) {
  return ((size_t)B * hkv * nsplit * G * hd * sizeof(float) + 255) & ~(size_t)255;
}
size_t stats_bytes(long long B, int hkv, int nsplit, int G) {
  return ((size_t)B * hkv * nsplit * G * sizeof(float2) + 255) & ~(size_t)255;
}
// The merge counters sit at the front of a workspace, at an offset that does
// not depend on n: calls of growing n that reuse one workspace find them at
// zero where the previous call left them.
size_t counter_bytes(long long B, int hkv) { return ((size_t)B * hkv * sizeof(unsigned) + 255) & ~(size_t)255; }

// Dynamic shared memory of one CTA: the V rows, then the K rows, which the
// output buffer and the merge's per-split weights (2 floats per head and
// split) reuse once K has been read.
size_t smem_bytes(int hd, int G, long long nsplit) {
  const size_t k_region = (size_t)kMaxChunk * hd * 2, out_region = ((size_t)4 * G * hd + (size_t)2 * G * nsplit) * 4;
  return (size_t)kMaxChunk * hd * 2 + (k_region > out_region ? k_region : out_region);
}
constexpr size_t kMaxSmem = 227u * 1024u;  // opt-in dynamic shared memory per CTA on sm_100

template <int HD, int G>
int launch(const AttnParams& p, long long B, void* stream) {
  // splits of at most 128 positions: one CTA stages all of its K and V at
  // once; longer splits stream through two stage buffers
  auto kern = p.chunk <= kMaxChunk ? decode_attn_kernel<HD, G> : decode_attn_stream_kernel<HD, G>;
  const int smem = (int)smem_bytes(HD, G, p.nsplit);
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * p.hkv), (unsigned)p.nsplit);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return WAL_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

template <int HD>
int launch_g(const AttnParams& p, long long B, int G, void* stream) {
  switch (G) {
    case 1: return launch<HD, 1>(p, B, stream);
    case 2: return launch<HD, 2>(p, B, stream);
    case 4: return launch<HD, 4>(p, B, stream);
    case 8: return launch<HD, 8>(p, B, stream);
    default: return WAL_ERR_UNSUPPORTED;
  }
}

}  // namespace

extern "C" {

size_t wal_decode_attention_workspace(int64_t B, int32_t hq, int32_t hkv, int32_t hd, int64_t n) {
  if (B <= 0 || hq <= 0 || hkv <= 0 || hd <= 0 || n <= 0 || hq % hkv) return 0;
  // sized for the largest split count of any call with up to n positions
  const int nsplit = (int)split_bound(B, hkv, n);
  const int G = hq / hkv;
  return counter_bytes(B, hkv) + part_bytes(B, hkv, nsplit, G, hd) + stats_bytes(B, hkv, nsplit, G);
}

}  // extern "C"

namespace {

// Argument checks and parameters shared by both entry points (scratch pointers left unset).
int prepare(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache, const uint16_t* v_cache, int64_t B, int32_t hq,
            int32_t hkv, int32_t hd, int64_t cache_len, int64_t n, float scale, uint16_t* out, int64_t ld_out,
            AttnParams* p) {
  if (!q || !k_cache || !v_cache || !out) return WAL_ERR_INVALID_ARGUMENT;
  if (B <= 0 || hq <= 0 || hkv <= 0 || n <= 0 || cache_len <= 0 || n > cache_len) return WAL_ERR_SHAPE;
  if (hq % hkv || B * hkv > 0x7fffffff) return WAL_ERR_SHAPE;
  if (hd != 64 && hd != 128) return WAL_ERR_UNSUPPORTED;
  if (ld_q < (int64_t)hq * hd || ld_out < (int64_t)hq * hd) return WAL_ERR_SHAPE;
  if (((uintptr_t)q & 7) || ((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15) || ((uintptr_t)out & 7) ||
      (ld_q % 4) || (ld_out % 4))
    return WAL_ERR_ALIGNMENT;
  p->q = q;
  p->ld_q = ld_q;
  p->k = k_cache;
  p->v = v_cache;
  p->cache_len = cache_len;
  p->n = (int)n;
  p->hq = hq;
  p->hkv = hkv;
  p->hd = hd;
  plan(B, hkv, n, &p->nsplit, &p->chunk);
  if (smem_bytes(hd, hq / hkv, p->nsplit) > kMaxSmem) return WAL_ERR_SHAPE;  // merge weights of too many splits
  p->qscale = scale * 1.4426950408889634f;  // log2(e)
  p->out = out;
  p->ld_out = ld_out;
  return WAL_OK;
}

int run(const AttnParams& p, long long B, void* stream) {
  const int G = p.hq / p.hkv;
  return p.hd == 128 ? launch_g<128>(p, B, G, stream) : launch_g<64>(p, B, G, stream);
}

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices];

}  // namespace

extern "C" {

int wal_decode_attention_ex(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache, const uint16_t* v_cache,
                            int64_t B, int32_t hq, int32_t hkv, int32_t hd, int64_t cache_len, int64_t n, float scale,
                            uint16_t* out, int64_t ld_out, void* workspace, size_t workspace_bytes, int num_splits,
                            void* stream) {
  AttnParams p;
  int st = prepare(q, ld_q, k_cache, v_cache, B, hq, hkv, hd, cache_len, n, scale, out, ld_out, &p);
  if (st != WAL_OK) return st;
  if (!workspace) return WAL_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)workspace & 255) return WAL_ERR_ALIGNMENT;
  const int G = hq / hkv;
  if (num_splits < 0) return WAL_ERR_INVALID_ARGUMENT;
  if (num_splits > 0) {  // explicit split: at least 32 positions per split
    long long sp = num_splits;
    if (sp > (n + 31) / 32) return WAL_ERR_SHAPE;
    long long c = ((n + sp - 1) / sp + 3) & ~3LL;
    p.nsplit = (int)((n + c - 1) / c);
    p.chunk = (int)c;
    if (smem_bytes(hd, G, p.nsplit) > kMaxSmem) return WAL_ERR_SHAPE;
    if (workspace_bytes < counter_bytes(B, hkv) + part_bytes(B, hkv, p.nsplit, G, hd) + stats_bytes(B, hkv, p.nsplit, G))
      return WAL_ERR_BUFFER_TOO_SMALL;
  } else if (workspace_bytes < wal_decode_attention_workspace(B, hq, hkv, hd, n)) {
    return WAL_ERR_BUFFER_TOO_SMALL;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t cb = counter_bytes(B, hkv);
  p.counter = reinterpret_cast<unsigned*>(ws);
  p.part = reinterpret_cast<float*>(ws + cb);
  p.stats = reinterpret_cast<float2*>(ws + cb + part_bytes(B, hkv, p.nsplit, G, hd));
  return run(p, B, stream);
}

int wal_decode_attention(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache, const uint16_t* v_cache, int64_t B,
                         int32_t hq, int32_t hkv, int32_t hd, int64_t cache_len, int64_t n, float scale,
                         uint16_t* out, int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream) {
  return wal_decode_attention_ex(q, ld_q, k_cache, v_cache, B, hq, hkv, hd, cache_len, n, scale, out, ld_out,
                                 workspace, workspace_bytes, 0, stream);
}

int wal_decode_attention_static(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache, const uint16_t* v_cache,
                                int64_t B, int32_t hq, int32_t hkv, int32_t hd, int64_t cache_len, int64_t n,
                                float scale, uint16_t* out, int64_t ld_out, void* stream) {
  AttnParams p;
  int st = prepare(q, ld_q, k_cache, v_cache, B, hq, hkv, hd, cache_len, n, scale, out, ld_out, &p);
  if (st != WAL_OK) return st;
  const int G = hq / hkv;
  const size_t data = part_bytes(B, hkv, p.nsplit, G, hd) + stats_bytes(B, hkv, p.nsplit, G);
  if ((size_t)B * hkv > kStaticCounters || data > kStaticScratchBytes - kStaticDataOffset)
    return WAL_ERR_BUFFER_TOO_SMALL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return WAL_ERR_CUDA;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev] && cudaGetSymbolAddress(&g_scratch_addr[dev], g_attn_scratch) != cudaSuccess) {
      g_scratch_addr[dev] = nullptr;
      return WAL_ERR_CUDA;
    }
    base = g_scratch_addr[dev];
  }
  uint8_t* ws = static_cast<uint8_t*>(base);
  p.counter = reinterpret_cast<unsigned*>(ws);
  p.part = reinterpret_cast<float*>(ws + kStaticDataOffset);
  p.stats = reinterpret_cast<float2*>(ws + kStaticDataOffset + part_bytes(B, hkv, p.nsplit, G, hd));
  // the array keeps whatever the last call left: clear the counters this call
  // uses (the partials and stats are written before they are read)
  if (cudaMemsetAsync(p.counter, 0, (size_t)B * hkv * sizeof(unsigned), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return WAL_ERR_CUDA;
  return run(p, B, stream);
}

}  // extern "C"
