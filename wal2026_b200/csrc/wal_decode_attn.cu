// Decode attention for the Llama-shaped stacks: one new query token per
// sequence, grouped-query heads, softmax(q k^T * scale) v over cache positions
// [0, n).  Replaces the PyTorch scaled_dot_product_attention call (and the copy
// of its output) in the decode step; no reference counterpart (the reference
// runs Hugging Face attention).
//
// Split-K over positions: CTA (b, kv head, split) scores its position range
// for all G = hq / hkv query heads that share the kv head.  The split's V rows
// stream into shared memory (cp.async) while each thread scores one position
// with its whole K row loaded at once (hd / 8 independent 16-byte loads), so
// many rows are in flight per SM; the weighted sum of values then reads V from
// shared memory.  Each CTA keeps (max, sum, un-normalised output) per head in
// fp32 and writes them to a workspace slot.  The last CTA of each (b, kv head)
// to finish (a counter in the workspace, returned to zero) merges the splits in
// split order - deterministic - and writes the bf16 output row in the layout
// the o-projection reads.  Softmax uses base-2 exponentials of scores
// pre-multiplied by scale * log2(e).
#include "../../include/wal_rvq.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace {

constexpr int kThreads = 128;     // 4 warps
constexpr int kMaxChunk = kThreads;  // positions per split: one K row per thread
constexpr int kTargetCtas = 148;   // one CTA per SM when the batch is small

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

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

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ AttnParams p) {
  constexpr int E = HD / 32;   // head-dim elements per lane in the value pass
  constexpr int P16 = HD / 8;  // 16-byte pieces per K/V row
  constexpr int NW = kThreads / 32;
  // shared: q [G][HD] fp32 | scores [G][chunk] fp32 | V rows [chunk][HD] bf16 | warp outputs [NW][G][HD] fp32
  //         | merge weights [nsplit][G] | merge sums [nsplit][G]
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[NW][G];
  __shared__ float stat[2][G];
  __shared__ int last;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.hkv, kvh = bh - b * p.hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = split * p.chunk;
  const int len = min(p.n - t0, p.chunk);  // >= 1: the plan leaves no empty split
  float* qs = sm;
  float* sc = qs + G * HD;
  uint16_t* vs = reinterpret_cast<uint16_t*>(sc + G * p.chunk);
  float* po = reinterpret_cast<float*>(vs + p.chunk * HD);
  const uint16_t* kb = p.k + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;
  const uint16_t* vb = p.v + (((long long)b * p.hkv + kvh) * p.cache_len + t0) * HD;

  // the cache and q come from earlier kernels of the step
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  // this thread's K row: hd / 8 independent 16-byte loads in flight
  uint4 kv[P16];
  if (tid < len) {
    const uint4* kr = reinterpret_cast<const uint4*>(kb + (long long)tid * HD);
#pragma unroll
    for (int j = 0; j < P16; ++j) kv[j] = __ldg(kr + j);
  }
  // V rows of this split -> shared memory
  const uint32_t vs_s = (uint32_t)__cvta_generic_to_shared(vs);
  for (int i = tid; i < len * P16; i += kThreads)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(vs_s + i * 16), "l"(vb + (long long)i * 8));
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  // the G query heads, pre-scaled
  for (int i = tid; i < G * HD; i += kThreads)
    qs[i] = bf16f(p.q[(long long)b * p.ld_q + (long long)kvh * G * HD + i]) * p.qscale;
  __syncthreads();

  // scores of this thread's position for the G heads
  float m_part[G];
  if (tid < len) {
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll
    for (int j = 0; j < P16; ++j) {
      const uint32_t w[4] = {kv[j].x, kv[j].y, kv[j].z, kv[j].w};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qa = *reinterpret_cast<const float4*>(qs + g * HD + j * 8);
        const float4 qb = *reinterpret_cast<const float4*>(qs + g * HD + j * 8 + 4);
        s[g] = fmaf(qa.x, __uint_as_float(w[0] << 16), s[g]);
        s[g] = fmaf(qa.y, __uint_as_float(w[0] & 0xFFFF0000u), s[g]);
        s[g] = fmaf(qa.z, __uint_as_float(w[1] << 16), s[g]);
        s[g] = fmaf(qa.w, __uint_as_float(w[1] & 0xFFFF0000u), s[g]);
        s[g] = fmaf(qb.x, __uint_as_float(w[2] << 16), s[g]);
        s[g] = fmaf(qb.y, __uint_as_float(w[2] & 0xFFFF0000u), s[g]);
        s[g] = fmaf(qb.z, __uint_as_float(w[3] << 16), s[g]);
        s[g] = fmaf(qb.w, __uint_as_float(w[3] & 0xFFFF0000u), s[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sc[g * p.chunk + tid] = s[g];
      m_part[g] = s[g];
    }
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) m_part[g] = -INFINITY;
  }
  // split max per head
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = m_part[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp][g] = m;
  }
  __syncthreads();
  float e_part[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = red[0][g];
#pragma unroll
    for (int w = 1; w < NW; ++w) m = fmaxf(m, red[w][g]);
    if (tid == 0) stat[0][g] = m;
    e_part[g] = 0.f;
    if (tid < len) {
      e_part[g] = exp2f(sc[g * p.chunk + tid] - m);
      sc[g * p.chunk + tid] = e_part[g];
    }
  }
  __syncthreads();  // red is reused below
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float l = e_part[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) red[warp][g] = l;
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncthreads();
  // weighted values from shared memory: warps own positions, lanes own E columns
  float acc[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
  for (int t = warp; t < len; t += NW) {
    float vv[E];
    const uint16_t* vr = vs + t * HD + lane * E;
    if constexpr (E == 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(vr);
      vv[0] = __uint_as_float(raw.x << 16); vv[1] = __uint_as_float(raw.x & 0xFFFF0000u);
      vv[2] = __uint_as_float(raw.y << 16); vv[3] = __uint_as_float(raw.y & 0xFFFF0000u);
    } else {
      const uint32_t raw = *reinterpret_cast<const uint32_t*>(vr);
      vv[0] = __uint_as_float(raw << 16); vv[1] = __uint_as_float(raw & 0xFFFF0000u);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pg = sc[g * p.chunk + t];
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] = fmaf(pg, vv[e], acc[g][e]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) po[(warp * G + g) * HD + lane * E + e] = acc[g][e];
  __syncthreads();
  // this split's slot: the warps' outputs summed in warp order, then (max, sum)
  const long long slot = (long long)bh * p.nsplit + split;
  float4* dst = reinterpret_cast<float4*>(p.part + slot * G * HD);
  for (int i = tid; i < G * HD / 4; i += kThreads) {
    float4 a = reinterpret_cast<const float4*>(po)[i];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
      const float4 c = reinterpret_cast<const float4*>(po + w * G * HD)[i];
      a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
    }
    dst[i] = a;
  }
  if (tid < G) {
    float l = red[0][tid];
#pragma unroll
    for (int w = 1; w < NW; ++w) l += red[w][tid];
    p.stats[slot * G + tid] = make_float2(stat[0][tid], l);
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
  const int ns = p.nsplit;
  float* wgt = po + NW * G * HD;  // [nsplit][G] exp2(m_s - M)
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
    if (lane == 0) stat[1][g] = 1.f / l;
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
    const float inv = stat[1][g];
    const uint32_t lo = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.x * inv)) |
                        ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.y * inv)) << 16);
    const uint32_t hi = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.z * inv)) |
                        ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a.w * inv)) << 16);
    *reinterpret_cast<uint2*>(orow + i * 4) = make_uint2(lo, hi);
  }
}

void plan(long long B, int hkv, long long n, int* nsplit, int* chunk) {
  long long s = (kTargetCtas + B * hkv - 1) / (B * hkv);
  const long long min_split = (n + kMaxChunk - 1) / kMaxChunk;
  if (s < min_split) s = min_split;
  const long long max_split = (n + 31) / 32;  // at least 32 positions per split
  if (s > max_split) s = max_split;
  if (s < 1) s = 1;
  long long c = ((n + s - 1) / s + 3) & ~3LL;  // multiple of 4 keeps the shared-memory regions 16-byte aligned
  s = (n + c - 1) / c;
  *nsplit = (int)s;
  *chunk = (int)c;
}

// Scratch of wal_decode_attention_static, zero-filled at module load: the
// merge counters occupy a fixed region at the front (so they are zero for any
// shape, each call returning them to zero), partial outputs and stats follow.
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

template <int HD, int G>
int launch(const AttnParams& p, long long B, void* stream) {
  auto kern = decode_attn_kernel<HD, G>;
  const int smem = (G * HD + G * p.chunk + 4 * G * HD + 2 * G * p.nsplit) * 4 + p.chunk * HD * 2;
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
  int nsplit = 0, chunk = 0;
  plan(B, hkv, n, &nsplit, &chunk);
  const int G = hq / hkv;
  return part_bytes(B, hkv, nsplit, G, hd) + stats_bytes(B, hkv, nsplit, G) + (size_t)B * hkv * sizeof(unsigned);
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

int wal_decode_attention(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache, const uint16_t* v_cache, int64_t B,
                         int32_t hq, int32_t hkv, int32_t hd, int64_t cache_len, int64_t n, float scale,
                         uint16_t* out, int64_t ld_out, void* workspace, size_t workspace_bytes, void* stream) {
  AttnParams p;
  int st = prepare(q, ld_q, k_cache, v_cache, B, hq, hkv, hd, cache_len, n, scale, out, ld_out, &p);
  if (st != WAL_OK) return st;
  if (!workspace) return WAL_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)workspace & 255) return WAL_ERR_ALIGNMENT;
  if (workspace_bytes < wal_decode_attention_workspace(B, hq, hkv, hd, n)) return WAL_ERR_BUFFER_TOO_SMALL;
  const int G = hq / hkv;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part = reinterpret_cast<float*>(ws);
  p.stats = reinterpret_cast<float2*>(ws + part_bytes(B, hkv, p.nsplit, G, hd));
  p.counter = reinterpret_cast<unsigned*>(ws + part_bytes(B, hkv, p.nsplit, G, hd) + stats_bytes(B, hkv, p.nsplit, G));
  return run(p, B, stream);
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
  return run(p, B, stream);
}

}  // extern "C"
