// Decode-step glue around the Block-RVQ linears of a Llama-shaped decoder, and
// the receiving half of the tensor-parallel exchange.
//
//   residual_rmsnorm_kernel  partial outputs of a row-parallel linear (tagged
//                            words pushed by wal_rvq_gemv_push from every rank,
//                            or one local fp32 output) summed in rank order,
//                            added to the residual stream, then the next
//                            RMSNorm; one CTA per token row.  Each thread spins
//                            on its own words until their tags are current,
//                            bounded (~2 s, %globaltimer); a timeout is reported
//                            through a status word instead of hanging, and the
//                            exchange must then be re-created (its call count
//                            no longer advances).
//   rope_kv_kernel           rotary embedding of q and k for one position and
//                            the KV-cache append, one thread per rotated pair.
//   silu_mul_kernel          SiLU(gate) * up of the fused gate/up output.
//
// Every kernel is launched with programmatic dependent launch: it waits on the
// grid dependency before reading its inputs and immediately allows the next
// kernel (the following GEMV, whose weight prologue needs none of this
// kernel's outputs) to start.  No reference counterpart: the reference runs
// these steps as separate PyTorch operators in Hugging Face decoder layers.
#include "../../include/wal_rvq.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>
#include <cstring>

namespace {

namespace cg = cooperative_groups;

__device__ __forceinline__ void dependency_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void dependents_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // 2 s
constexpr int kNormThreads = 512;
constexpr int kMaxNormN = 16384;

struct NormParams {
  // local form: one fp32 partial (or none)
  const float* partial;
  long long ldp;
  // exchange form: tagged words {value, tag} from num_ranks ranks
  const uint4* recv;  // pairs of words
  int num_ranks;
  long long rank_stride, ld;  // in words
  unsigned* epoch;
  unsigned* done;
  uint16_t* h;
  long long ldh;
  const uint16_t* w;
  float eps;
  uint16_t* x;
  long long ldx;
  int N;
  int* status;
};

__device__ __forceinline__ uint4 ld_volatile_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Two tagged words (4 x u32: value, tag, value, tag); false if the deadline passed first.
__device__ __forceinline__ bool wait_pair(const uint4* src, unsigned tag, unsigned long long deadline, float& a,
                                          float& b) {
  for (;;) {
    const uint4 v = ld_volatile_v4(src);
    if (v.y == tag && v.w == tag) {
      a = __uint_as_float(v.x);
      b = __uint_as_float(v.z);
      return true;
    }
    if (global_ns() > deadline) return false;
  }
}

__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(const __grid_constant__ NormParams p) {
  extern __shared__ float hs[];  // [N] residual values after the add
  __shared__ float red[kNormThreads / 32];
  __shared__ int give_up;
  dependency_wait();
  dependents_launch();
  const int m = blockIdx.x;
  unsigned tag = 0;
  unsigned long long deadline = 0;
  if (p.recv) {
    tag = *reinterpret_cast<const volatile unsigned*>(p.epoch) + 1u;
    deadline = global_ns() + kPeerWaitNs;
  }
  if (threadIdx.x == 0) give_up = 0;
  __syncthreads();

  uint16_t* hrow = p.h + (long long)m * p.ldh;
  float sq = 0.f;
  bool ok = true;
  // 8 columns per thread per step: one 16-byte load of h, 8 values per source
  for (int c = threadIdx.x * 8; c < p.N; c += kNormThreads * 8) {
    uint4 hv = *reinterpret_cast<const uint4*>(hrow + c);
    uint16_t hb[8];
    memcpy(hb, &hv, 16);
    bool have = false;
    float s[8];
    if (p.recv) {
      const uint4* row = p.recv + ((long long)m * p.ld + c) / 2;
      for (int r = 0; r < p.num_ranks && ok; ++r) {
        const uint4* src = row + r * (p.rank_stride / 2);
        float v[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) ok = ok && wait_pair(src + j, tag, deadline, v[2 * j], v[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = r == 0 ? v[j] : s[j] + v[j];
      }
      have = ok;
    } else if (p.partial) {
      const float* src = p.partial + (long long)m * p.ldp + c;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      s[0] = a.x; s[1] = a.y; s[2] = a.z; s[3] = a.w; s[4] = b.x; s[5] = b.y; s[6] = b.z; s[7] = b.w;
      have = true;
    }
    if (!ok) break;
    if (have) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = bf16_to_f32(f32_to_bf16(s[j]));  // the linear's bf16 output
        hb[j] = f32_to_bf16(bf16_to_f32(hb[j]) + v);     // bf16 residual add
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float hn = bf16_to_f32(hb[j]);
      hs[c + j] = hn;
      sq = fmaf(hn, hn, sq);
    }
  }
  if (!ok) give_up = 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (give_up) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, (int)WAL_ERR_PEER_TIMEOUT);
    return;  // h, x and the call count stay as they were
  }
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)p.N + p.eps);
  uint16_t* xrow = p.x + (long long)m * p.ldx;
  for (int c = threadIdx.x * 8; c < p.N; c += kNormThreads * 8) {
    const uint4 wv = *reinterpret_cast<const uint4*>(p.w + c);
    uint16_t wb[8], ob[8], hb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) hb[j] = f32_to_bf16(hs[c + j]);
    if (p.recv || p.partial) {
      uint4 hv;
      memcpy(&hv, hb, 16);
      *reinterpret_cast<uint4*>(hrow + c) = hv;
    }
    memcpy(wb, &wv, 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = f32_to_bf16((hs[c + j] * rstd) * bf16_to_f32(wb[j]));
    uint4 ov;
    memcpy(&ov, ob, 16);
    *reinterpret_cast<uint4*>(xrow + c) = ov;
  }
  if (p.recv) {  // the last CTA advances the slot's call count, after every CTA read it
    __syncthreads();
    if (threadIdx.x == 0) {
      if (atomicAdd(p.done, 1u) == gridDim.x - 1) {
        *p.done = 0u;
        *p.epoch = tag;
      }
    }
  }
}

// Cluster form of the same operation for wide rows: one cluster of kNormCluster
// CTAs per token row, each CTA owning N / kNormCluster columns.  Every thread
// issues the loads of all ranks' words of its 8 columns at once and re-reads
// (bounded) only the words whose tag is not yet current, so the exchange costs
// one memory round trip instead of one per rank; the CTAs' sums of squares
// meet through distributed shared memory and are added in CTA order, so every
// CTA (and every rank) derives the same scale.
constexpr int kNormCluster = 8;

__global__ void __launch_bounds__(256) residual_rmsnorm_cluster_kernel(const __grid_constant__ NormParams p) {
  extern __shared__ float hs[];  // this CTA's columns after the residual add
  __shared__ float red[8];
  __shared__ float cta_sum;
  __shared__ int cta_fail;
  cg::cluster_group cluster = cg::this_cluster();
  const int cr = (int)cluster.block_rank();
  dependency_wait();
  dependents_launch();
  const int m = blockIdx.y;
  const int cols = p.N / kNormCluster;
  const int c_begin = cr * cols;
  unsigned tag = 0;
  unsigned long long deadline = 0;
  if (p.recv) {
    tag = *reinterpret_cast<const volatile unsigned*>(p.epoch) + 1u;
    deadline = global_ns() + kPeerWaitNs;
  }
  if (threadIdx.x == 0) cta_fail = 0;
  __syncthreads();
  uint16_t* hrow = p.h + (long long)m * p.ldh;
  float sq = 0.f;
  bool ok = true;
  for (int lc = threadIdx.x * 8; lc < cols; lc += blockDim.x * 8) {
    const int c = c_begin + lc;
    uint4 hv = *reinterpret_cast<const uint4*>(hrow + c);
    uint16_t hb[8];
    memcpy(hb, &hv, 16);
    float s[8];
    bool have = false;
    if (p.recv) {
      const uint4* row = p.recv + ((long long)m * p.ld + c) / 2;
      uint4 v[WAL_MAX_RANKS][4];
#pragma unroll
      for (int r = 0; r < WAL_MAX_RANKS; ++r)
        if (r < p.num_ranks)
#pragma unroll
          for (int j = 0; j < 4; ++j) v[r][j] = ld_volatile_v4(row + r * (p.rank_stride / 2) + j);
#pragma unroll
      for (int r = 0; r < WAL_MAX_RANKS; ++r) {
        if (r >= p.num_ranks) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // re-read only words that are not current yet, until the deadline
          while (ok && (v[r][j].y != tag || v[r][j].w != tag)) {
            if (global_ns() > deadline) {
              ok = false;
              break;
            }
            v[r][j] = ld_volatile_v4(row + r * (p.rank_stride / 2) + j);
          }
          const float a = __uint_as_float(v[r][j].x), b = __uint_as_float(v[r][j].z);
          s[2 * j] = r == 0 ? a : s[2 * j] + a;
          s[2 * j + 1] = r == 0 ? b : s[2 * j + 1] + b;
        }
      }
      have = ok;
    } else if (p.partial) {
      const float* src = p.partial + (long long)m * p.ldp + c;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      s[0] = a.x; s[1] = a.y; s[2] = a.z; s[3] = a.w; s[4] = b.x; s[5] = b.y; s[6] = b.z; s[7] = b.w;
      have = true;
    }
    if (!ok) break;
    if (have) {
#pragma unroll
      for (int j = 0; j < 8; ++j) hb[j] = f32_to_bf16(bf16_to_f32(hb[j]) + bf16_to_f32(f32_to_bf16(s[j])));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float hn = bf16_to_f32(hb[j]);
      hs[lc + j] = hn;
      sq = fmaf(hn, hn, sq);
    }
  }
  if (!ok) cta_fail = 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    cta_sum = t;
  }
  cluster.sync();  // every CTA's partial sum and failure flag are published
  float tot = 0.f;
  int fail = 0;
  for (int k = 0; k < kNormCluster; ++k) {
    tot += *cluster.map_shared_rank(&cta_sum, k);
    fail |= *cluster.map_shared_rank(&cta_fail, k);
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
  if (fail) {
    if (threadIdx.x == 0 && cr == 0 && p.status) atomicExch(p.status, (int)WAL_ERR_PEER_TIMEOUT);
    return;  // this row's h and x stay as they were; the call count does not advance
  }
  const float rstd = rsqrtf(tot / (float)p.N + p.eps);
  uint16_t* xrow = p.x + (long long)m * p.ldx;
  for (int lc = threadIdx.x * 8; lc < cols; lc += blockDim.x * 8) {
    const int c = c_begin + lc;
    const uint4 wv = *reinterpret_cast<const uint4*>(p.w + c);
    uint16_t wb[8], ob[8], hb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) hb[j] = f32_to_bf16(hs[lc + j]);
    if (p.recv || p.partial) {
      uint4 hv;
      memcpy(&hv, hb, 16);
      *reinterpret_cast<uint4*>(hrow + c) = hv;
    }
    memcpy(wb, &wv, 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = f32_to_bf16((hs[lc + j] * rstd) * bf16_to_f32(wb[j]));
    uint4 ov;
    memcpy(&ov, ob, 16);
    *reinterpret_cast<uint4*>(xrow + c) = ov;
  }
  if (p.recv) {  // the last CTA of the grid advances the slot's call count
    __syncthreads();
    if (threadIdx.x == 0) {
      if (atomicAdd(p.done, 1u) == gridDim.x * gridDim.y - 1) {
        *p.done = 0u;
        *p.epoch = tag;
      }
    }
  }
}

struct RopeParams {
  const uint16_t* qkv;
  long long ld_qkv;
  int M, hq, hkv, hd;
  const float* cos;
  const float* sin;
  long long pos, cache_len;
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
};

__global__ void __launch_bounds__(256) rope_kv_kernel(const __grid_constant__ RopeParams p) {
  dependency_wait();
  dependents_launch();
  const int half = p.hd / 2;
  const long long n_rot = (long long)p.M * (p.hq + p.hkv) * half;
  const long long n_v = (long long)p.M * p.hkv * p.hd;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_rot + n_v;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < n_rot) {
      const int j = (int)(i % half);
      const long long t = i / half;
      const int head = (int)(t % (p.hq + p.hkv));
      const int m = (int)(t / (p.hq + p.hkv));
      const uint16_t* src = p.qkv + (long long)m * p.ld_qkv + (long long)head * p.hd;
      const float x1 = bf16_to_f32(src[j]), x2 = bf16_to_f32(src[j + half]);
      // x * cos + rotate_half(x) * sin, each product rounded, then the sum
      const float o1 = __fadd_rn(__fmul_rn(x1, p.cos[j]), __fmul_rn(-x2, p.sin[j]));
      const float o2 = __fadd_rn(__fmul_rn(x2, p.cos[j + half]), __fmul_rn(x1, p.sin[j + half]));
      uint16_t* dst;
      if (head < p.hq) {
        dst = p.q_out + (long long)m * p.hq * p.hd + (long long)head * p.hd;
      } else {
        dst = p.k_cache + (((long long)m * p.hkv + (head - p.hq)) * p.cache_len + p.pos) * p.hd;
      }
      dst[j] = f32_to_bf16(o1);
      dst[j + half] = f32_to_bf16(o2);
    } else {
      const long long v = i - n_rot;
      const int j = (int)(v % p.hd);
      const long long t = v / p.hd;
      const int kvh = (int)(t % p.hkv);
      const int m = (int)(t / p.hkv);
      const uint16_t* src = p.qkv + (long long)m * p.ld_qkv + (long long)(p.hq + p.hkv + kvh) * p.hd;
      p.v_cache[(((long long)m * p.hkv + kvh) * p.cache_len + p.pos) * p.hd + j] = src[j];
    }
  }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(const uint16_t* __restrict__ gu, long long ld_gu, int M,
                                                       long long I, uint16_t* __restrict__ out, long long ld_out) {
  dependency_wait();
  dependents_launch();
  const long long total = (long long)M * I;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / I, c = i - m * I;
    const float g = bf16_to_f32(gu[m * ld_gu + c]);
    const float u = bf16_to_f32(gu[m * ld_gu + I + c]);
    const float s = bf16_to_f32(f32_to_bf16(g / (1.0f + expf(-g))));
    out[m * ld_out + c] = f32_to_bf16(s * u);
  }
}

template <typename Kern, typename... Args>
int launch_pdl(Kern kern, int grid, int block, int smem, void* stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) return WAL_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

int grid_for(long long work, int block) {
  long long g = (work + block - 1) / block;
  if (g > 148 * 8) g = 148 * 8;
  return (int)(g < 1 ? 1 : g);
}

// Sending half of the exchange for an output that some other kernel already
// produced (e.g. a dense library GEMM): every pair of adjacent fp32 values of
// rows < M becomes one 16-byte store {v0, tag, v1, tag} into every rank's
// receive rows (as NCCL's LL protocol, each 8-byte {value, tag} half arrives
// whole).  tag = *epoch + 1, read after the grid dependency.
struct PushRowsParams {
  const void* y;
  long long ldy;
  int y_dtype;
  int M;
  long long N;  // even
  int num_ranks;
  uint4* dst[WAL_MAX_RANKS];
  long long ld_dst;  // words, even
  const unsigned* epoch;
};

__global__ void __launch_bounds__(256) push_rows_kernel(const __grid_constant__ PushRowsParams p) {
  dependency_wait();
  const unsigned tag = *reinterpret_cast<const volatile unsigned*>(p.epoch) + 1u;
  const long long pairs_per_row = p.N / 2, total = pairs_per_row * p.M;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / pairs_per_row);
    const long long c = (i - (long long)m * pairs_per_row) * 2;
    float v0, v1;
    if (p.y_dtype == WAL_F32) {
      const float2 v = *reinterpret_cast<const float2*>(static_cast<const float*>(p.y) + m * p.ldy + c);
      v0 = v.x;
      v1 = v.y;
    } else {
      const uint32_t b = *reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(p.y) + m * p.ldy + c);
      v0 = __uint_as_float(b << 16);
      v1 = __uint_as_float(b & 0xffff0000u);
    }
    const long long w = (m * p.ld_dst + c) / 2;
#pragma unroll
    for (int r = 0; r < WAL_MAX_RANKS; ++r)
      if (r < p.num_ranks)
        asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"l"(p.dst[r] + w),
                     "r"(__float_as_uint(v0)), "r"(tag), "r"(__float_as_uint(v1)), "r"(tag)
                     : "memory");
  }
  dependents_launch();
}

}  // namespace

extern "C" {

static int launch_norm(NormParams& p, int64_t M, int64_t N, void* stream) {
  if (!p.h || !p.w || !p.x) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0 || N <= 0) return WAL_ERR_SHAPE;
  if (N % 8 || N > kMaxNormN || M > 65535) return WAL_ERR_UNSUPPORTED;
  if (p.ldh < N || p.ldx < N) return WAL_ERR_SHAPE;
  if ((p.ldh % 8) || (p.ldx % 8) || ((uintptr_t)p.h & 15) || ((uintptr_t)p.x & 15) || ((uintptr_t)p.w & 15))
    return WAL_ERR_ALIGNMENT;
  p.N = (int)N;
  if (N % (8 * kNormCluster) == 0 && N >= 1024) {
    // one cluster of kNormCluster CTAs per row, 8 columns per thread
    const int cols = (int)N / kNormCluster;
    int threads = ((cols / 8 + 31) / 32) * 32;
    if (threads > 256) threads = 256;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kNormCluster, (unsigned)M);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = cols * 4;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kNormCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, residual_rmsnorm_cluster_kernel, p) != cudaSuccess) return WAL_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
  }
  const int smem = (int)N * 4;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(residual_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  return launch_pdl(residual_rmsnorm_kernel, (int)M, kNormThreads, smem, stream, p);
}

int wal_residual_rmsnorm(const float* partial, int64_t ldp, uint16_t* h, int64_t ldh, const uint16_t* norm_weight,
                         float eps, uint16_t* x_out, int64_t ldx, int64_t M, int64_t N, void* stream) {
  NormParams p = {};
  if (partial) {
    if (ldp < N) return WAL_ERR_SHAPE;
    if ((ldp % 4) || ((uintptr_t)partial & 15)) return WAL_ERR_ALIGNMENT;
  }
  p.partial = partial;
  p.ldp = ldp;
  p.h = h;
  p.ldh = ldh;
  p.w = norm_weight;
  p.eps = eps;
  p.x = x_out;
  p.ldx = ldx;
  return launch_norm(p, M, N, stream);
}

int wal_tp_reduce_rmsnorm(const void* recv, int32_t num_ranks, int64_t rank_stride, int64_t ld, uint32_t* epoch,
                          uint32_t* done, uint16_t* h, int64_t ldh, const uint16_t* norm_weight, float eps,
                          uint16_t* x_out, int64_t ldx, int64_t M, int64_t N, int* status, void* stream) {
  if (!recv || !epoch || !done) return WAL_ERR_INVALID_ARGUMENT;
  if (num_ranks < 1 || num_ranks > WAL_MAX_RANKS) return WAL_ERR_INVALID_ARGUMENT;
  if (ld < N || (num_ranks > 1 && rank_stride < M * ld)) return WAL_ERR_SHAPE;
  if ((ld % 2) || (rank_stride % 2) || ((uintptr_t)recv & 15)) return WAL_ERR_ALIGNMENT;
  NormParams p = {};
  p.recv = static_cast<const uint4*>(recv);
  p.num_ranks = num_ranks;
  p.rank_stride = rank_stride;
  p.ld = ld;
  p.epoch = epoch;
  p.done = done;
  p.h = h;
  p.ldh = ldh;
  p.w = norm_weight;
  p.eps = eps;
  p.x = x_out;
  p.ldx = ldx;
  p.status = status;
  return launch_norm(p, M, N, stream);
}

int wal_rope_kv_append(const uint16_t* qkv, int64_t ld_qkv, int64_t M, int32_t hq, int32_t hkv, int32_t hd,
                       const float* cos, const float* sin, int64_t pos, uint16_t* q_out, uint16_t* k_cache,
                       uint16_t* v_cache, int64_t cache_len, void* stream) {
  if (!qkv || !cos || !sin || !q_out || !k_cache || !v_cache) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0 || hq <= 0 || hkv <= 0 || hd <= 0 || hd % 2 || cache_len <= 0) return WAL_ERR_SHAPE;
  if (pos < 0 || pos >= cache_len) return WAL_ERR_SHAPE;
  if (ld_qkv < (int64_t)(hq + 2 * hkv) * hd) return WAL_ERR_SHAPE;
  RopeParams p;
  p.qkv = qkv;
  p.ld_qkv = ld_qkv;
  p.M = (int)M;
  p.hq = hq;
  p.hkv = hkv;
  p.hd = hd;
  p.cos = cos;
  p.sin = sin;
  p.pos = pos;
  p.cache_len = cache_len;
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  const long long work = M * (long long)(hq + hkv) * (hd / 2) + M * (long long)hkv * hd;
  return launch_pdl(rope_kv_kernel, grid_for(work, 256), 256, 0, stream, p);
}

int wal_silu_mul(const uint16_t* gu, int64_t ld_gu, int64_t M, int64_t I, uint16_t* out, int64_t ld_out,
                 void* stream) {
  if (!gu || !out) return WAL_ERR_INVALID_ARGUMENT;
  if (M <= 0 || I <= 0 || ld_gu < 2 * I || ld_out < I || M > 0x7fffffff) return WAL_ERR_SHAPE;
  return launch_pdl(silu_mul_kernel, grid_for(M * I, 256), 256, 0, stream, gu, (long long)ld_gu, (int)M,
                    (long long)I, out, (long long)ld_out);
}

int wal_tp_push_rows(const void* y, int64_t ldy, int y_dtype, int64_t M, int64_t N, const wal_tp_push* push,
                     void* stream) {
  if (!y || !push || !push->epoch) return WAL_ERR_INVALID_ARGUMENT;
  if (push->num_ranks < 1 || push->num_ranks > WAL_MAX_RANKS || push->rank < 0 || push->rank >= push->num_ranks)
    return WAL_ERR_INVALID_ARGUMENT;
  if (y_dtype != WAL_F32 && y_dtype != WAL_BF16) return WAL_ERR_UNSUPPORTED;
  if (M <= 0 || N <= 0 || M > 0x7fffffff || ldy < N || push->ld_dst < N) return WAL_ERR_SHAPE;
  if ((N % 2) || (ldy % 2) || (push->ld_dst % 2)) return WAL_ERR_ALIGNMENT;
  if ((uintptr_t)y & (y_dtype == WAL_F32 ? 7 : 3)) return WAL_ERR_ALIGNMENT;
  PushRowsParams p = {};
  p.y = y;
  p.ldy = ldy;
  p.y_dtype = y_dtype;
  p.M = (int)M;
  p.N = N;
  p.num_ranks = push->num_ranks;
  for (int r = 0; r < push->num_ranks; ++r) {
    if (!push->dst[r]) return WAL_ERR_INVALID_ARGUMENT;
    if ((uintptr_t)push->dst[r] & 15) return WAL_ERR_ALIGNMENT;
    p.dst[r] = static_cast<uint4*>(push->dst[r]);
  }
  p.ld_dst = push->ld_dst;
  p.epoch = push->epoch;
  return launch_pdl(push_rows_kernel, grid_for(M * (N / 2), 256), 256, 0, stream, p);
}

int wal_peer_region_create(size_t bytes, void** dev_ptr, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) <= WAL_IPC_HANDLE_BYTES, "IPC handle does not fit");
  if (!dev_ptr || !handle_out || bytes == 0) return WAL_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return WAL_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return WAL_ERR_CUDA;
  }
  std::memset(handle_out, 0, WAL_IPC_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return WAL_OK;
}

int wal_peer_region_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return WAL_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return WAL_ERR_CUDA;
  *dev_ptr = p;
  return WAL_OK;
}

int wal_peer_region_close(void* dev_ptr) {
  if (!dev_ptr) return WAL_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

int wal_peer_region_free(void* dev_ptr) {
  if (!dev_ptr) return WAL_ERR_INVALID_ARGUMENT;
  return cudaFree(dev_ptr) == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

}  // extern "C"
