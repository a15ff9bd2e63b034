// Encoder side of Block-RVQ: nearest-codebook-entry assignment, the hot loop
// of the reference's k-means fit and of every stage's full assignment
// (reference src/block_vq.py:180-196, _assign_to_codebook): for each block
// x (d values), the entry c minimising
//     dist = ||x||^2 + ||c||^2 - 2 x.c          (fp32, the reference's form)
// with the lowest index among equal distances (torch.min's first minimum).
//
// One thread per block: its d values stay in registers, the codebook (fp32,
// with its squared norms) is staged in shared memory once per CTA and read by
// every thread of a warp at the same address (broadcast, no bank conflicts);
// squared norms are rounded squares summed in order (the reference's
// square().sum()), the d-term dot products run in ascending order with fused
// multiply-adds.
// The reference forms x.c inside a CPU matrix product whose summation order
// is its own, so a block whose two best entries are within a few fp32 units
// of each other can be assigned differently; every other block gets the same
// id and the same minimum distance up to those units.
#include "../../include/wal_rvq.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kThreads = 256;
constexpr int kMaxSmem = 227 * 1024;  // the codebook (fp32 [C][d] and its norms) lives in shared memory

template <int D>
__global__ void __launch_bounds__(kThreads) assign_kernel(const float* __restrict__ blocks, long long n,
                                                          const float* __restrict__ codebook, int C,
                                                          int32_t* __restrict__ ids, float* __restrict__ min_dist) {
  extern __shared__ float sm[];
  float* cb = sm;           // [C][D]
  float* csq = sm + C * D;  // [C]
  for (int i = threadIdx.x; i < C * D; i += blockDim.x) cb[i] = codebook[i];
  __syncthreads();
  for (int e = threadIdx.x; e < C; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) s = __fadd_rn(s, __fmul_rn(cb[e * D + j], cb[e * D + j]));  // square, then sum
    csq[e] = s;
  }
  __syncthreads();
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < n; b += (long long)gridDim.x * blockDim.x) {
    float x[D];
#pragma unroll
    for (int j = 0; j < D; ++j) x[j] = blocks[b * D + j];
    float xsq = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) xsq = __fadd_rn(xsq, __fmul_rn(x[j], x[j]));
    float best = __int_as_float(0x7f800000);  // +inf
    int arg = 0;
    for (int e = 0; e < C; ++e) {
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < D; ++j) dot = fmaf(x[j], cb[e * D + j], dot);
      const float dist = __fsub_rn(__fadd_rn(xsq, csq[e]), __fmul_rn(2.0f, dot));
      if (dist < best) {  // strict: the first of equal minima wins
        best = dist;
        arg = e;
      }
    }
    ids[b] = arg;
    if (min_dist) min_dist[b] = best;
  }
}

template <int D>
int launch(const float* blocks, long long n, const float* codebook, int C, int32_t* ids, float* min_dist,
           cudaStream_t s) {
  const int smem = (C * D + C) * (int)sizeof(float);
  auto kern = assign_kernel<D>;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return WAL_ERR_CUDA;
  long long grid = (n + kThreads - 1) / kThreads;
  if (grid > 148 * 16) grid = 148 * 16;
  kern<<<(unsigned)grid, kThreads, smem, s>>>(blocks, n, codebook, C, ids, min_dist);
  return cudaGetLastError() == cudaSuccess ? WAL_OK : WAL_ERR_CUDA;
}

}  // namespace

extern "C" int wal_rvq_assign(const float* blocks, int64_t n, int32_t d, const float* codebook, int32_t num_entries,
                              int32_t* ids, float* min_dist, void* stream) {
  if (!blocks || !codebook || !ids) return WAL_ERR_INVALID_ARGUMENT;
  if (n <= 0 || num_entries <= 0) return WAL_ERR_SHAPE;
  if ((long long)(num_entries * (long long)d + num_entries) * (long long)sizeof(float) > kMaxSmem)
    return WAL_ERR_UNSUPPORTED;
  if (((uintptr_t)blocks & 3) || ((uintptr_t)codebook & 3) || ((uintptr_t)ids & 3) || ((uintptr_t)min_dist & 3))
    return WAL_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (d) {
    case 4: return launch<4>(blocks, n, codebook, num_entries, ids, min_dist, s);
    case 8: return launch<8>(blocks, n, codebook, num_entries, ids, min_dist, s);
    case 16: return launch<16>(blocks, n, codebook, num_entries, ids, min_dist, s);
    case 32: return launch<32>(blocks, n, codebook, num_entries, ids, min_dist, s);
    default: return WAL_ERR_UNSUPPORTED;
  }
}
