/*
 * CPU oracle of the Block-RVQ runtime linear: TEST INFRASTRUCTURE ONLY.
 *
 * A C restatement of the reference's dequantise-then-matmul forward
 * (matmul_strategy="per_group"), used as the timed CPU baseline and as a fast
 * checker at full sizes.  Nothing in the product links it.
 *
 * Restated reference lines:
 *   src/runtime.py:381-388  fp32 accumulator from +0.0, recon += fp32(codebook[ids]) per stage in order
 *   src/runtime.py:413-414  slice to in_features, .to(bf16), * row_scale.to(bf16) (bf16 result)
 *   src/runtime.py:1501-1507 per-group F.linear(x, weight, bias), fp32 accumulation, groups concatenated
 * Like the reference, every call materialises the whole bf16 weight before the
 * product (the weight buffer is per call, rows are processed in parallel).
 *
 * bf16 rounding follows PyTorch's float->bfloat16 conversion (round to nearest
 * even on the fp32 bits, NaN -> 0x7FC0).  fp16 -> fp32 is exact.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (isnan(f)) return 0x7FC0u;
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static inline float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* w[rows][K] (bf16 bits) for one group; ids[s] is [rows][blocks] with idw bytes per id. */
static void reconstruct_rows(const void* const* ids, int idw, const uint16_t* books, int R, int entries, int d,
                             const uint16_t* rho, int64_t row_begin, int64_t row_end, int64_t K, int64_t blocks,
                             uint16_t* w) {
  float* acc = (float*)malloc(sizeof(float) * (size_t)(blocks * d));
  for (int64_t n = row_begin; n < row_end; ++n) {
    for (int64_t i = 0; i < blocks * d; ++i) acc[i] = 0.0f;
    for (int s = 0; s < R; ++s) {
      const uint16_t* book = books + (size_t)s * entries * d;
      for (int64_t b = 0; b < blocks; ++b) {
        const uint32_t id = idw == 1 ? ((const uint8_t*)ids[s])[n * blocks + b]
                                     : ((const uint16_t*)ids[s])[n * blocks + b];
        const uint16_t* e = book + (size_t)id * d;
        for (int j = 0; j < d; ++j) acc[b * d + j] += f16_to_f32(e[j]);
      }
    }
    const float rb = bf16_to_f32(f32_to_bf16(f16_to_f32(rho[n])));
    for (int64_t k = 0; k < K; ++k) {
      const float wb = bf16_to_f32(f32_to_bf16(acc[k]));
      w[(n - row_begin) * K + k] = f32_to_bf16(wb * rb);
    }
  }
  free(acc);
}

typedef struct job {
  const void* const* ids;
  int idw;
  const uint16_t* books;
  int R, entries, d;
  const uint16_t* rho;
  int64_t rows, K, blocks;
  const uint16_t* x;
  int64_t M;
  const uint16_t* bias;
  float* y;
  int64_t ldy, row0;
  uint16_t* w; /* [rows][K] */
  int64_t begin, end;
  int gemv;
} job;

static void* run_job(void* arg) {
  job* j = (job*)arg;
  reconstruct_rows(j->ids, j->idw, j->books, j->R, j->entries, j->d, j->rho, j->begin, j->end, j->K, j->blocks,
                   j->w + j->begin * j->K);
  if (j->gemv) {
    for (int64_t n = j->begin; n < j->end; ++n) {
      for (int64_t m = 0; m < j->M; ++m) {
        float s = 0.0f;
        const uint16_t* xr = j->x + m * j->K;
        const uint16_t* wr = j->w + n * j->K;
        for (int64_t k = 0; k < j->K; ++k) s += bf16_to_f32(xr[k]) * bf16_to_f32(wr[k]);
        if (j->bias) s += bf16_to_f32(j->bias[j->row0 + n]);
        j->y[m * j->ldy + j->row0 + n] = s;
      }
    }
  }
  return NULL;
}

int rvq_oracle_max_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static int run_parallel(job base, int threads) {
  if (threads <= 0) threads = rvq_oracle_max_threads();
  if (threads > 256) threads = 256;
  if (threads > base.rows) threads = (int)base.rows;
  if (threads < 1) threads = 1;
  job jobs[256];
  pthread_t tids[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = base;
    jobs[t].begin = base.rows * t / threads;
    jobs[t].end = base.rows * (t + 1) / threads;
  }
  for (int t = 1; t < threads; ++t)
    if (pthread_create(&tids[t], NULL, run_job, &jobs[t]) != 0) return 2;
  run_job(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
  return 0;
}

/*
 * One group's forward: y[M][ldy] (columns row0..row0+rows-1) = x[M][K] @ w^T (+ bias), fp32.
 * x and bias are bf16 bits; threads <= 0 means all online CPUs.
 */
int rvq_oracle_forward_group(const void* const* ids, int idw, const uint16_t* books, int R, int entries, int d,
                             const uint16_t* rho, int64_t rows, int64_t K, const uint16_t* x, int64_t M,
                             const uint16_t* bias, float* y, int64_t ldy, int64_t row0, int threads) {
  uint16_t* w = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(rows * K));
  if (!w) return 1;
  job base = {ids, idw, books, R, entries, d, rho, rows, K, (K + d - 1) / d, x, M, bias, y, ldy, row0, w, 0, 0, 1};
  const int st = run_parallel(base, threads);
  free(w);
  return st;
}

/* Weight only (bf16 bits, [rows][K]) for the bit-exactness checks. */
int rvq_oracle_reconstruct_group(const void* const* ids, int idw, const uint16_t* books, int R, int entries, int d,
                                 const uint16_t* rho, int64_t rows, int64_t K, uint16_t* w, int threads) {
  job base = {ids, idw, books, R, entries, d, rho, rows, K, (K + d - 1) / d, NULL, 0, NULL, NULL, 0, 0, w, 0, 0, 0};
  return run_parallel(base, threads);
}
