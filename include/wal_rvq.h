/*
 * wal_rvq.h - C ABI of the B200 Block-RVQ / route-codebook runtime linear.
 *
 * A Block-RVQ linear stores an N x K weight as, for every (row, block of d
 * columns) unit and every stage s < R, an id into a per-stage fp16 codebook
 * of `num_entries` rows of d values, plus one fp16 scale per output row.
 * Rows may be split into groups that carry their own codebooks.  The weight
 * this library decodes is, bit for bit, the one the reference's
 * dequantise-then-matmul path builds for a bf16 forward:
 *
 *   w[n, k] = bf16( bf16( sum_s fp32(C_s[id_s(n, k / d)][k % d]) ) * bf16(rho[n]) )
 *
 * (reference src/runtime.py:379-414, PackedBlockRVQGroup.reconstruct_weight),
 * and the GEMV computes y = x @ w^T (+ bias) with fp32 accumulation
 * (reference src/runtime.py:1501-1507, PackedGroupedBlockRVQLinear.forward,
 * default "per_group" strategy).  The dense weight is never materialised by
 * the GEMV.
 *
 * Conventions: every entry point returns a wal_status (0 = success) and never
 * throws.  Device pointers are CUDA device memory of the current device;
 * `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Host pointers are ordinary CPU memory.  bf16/fp16 values are passed as
 * uint16_t bit patterns.  No entry point synchronises the stream.
 */
#ifndef WAL_RVQ_H
#define WAL_RVQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WAL_API __attribute__((visibility("default")))
#else
#define WAL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wal_status {
  WAL_OK = 0,
  WAL_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size            */
  WAL_ERR_SHAPE = 2,            /* inconsistent or unsupported dimensions     */
  WAL_ERR_ALIGNMENT = 3,        /* pointer or leading dimension misaligned    */
  WAL_ERR_ID_RANGE = 4,         /* an id or route is >= its codebook size     */
  WAL_ERR_UNSUPPORTED = 5,      /* valid input this build does not implement  */
  WAL_ERR_CUDA = 6,             /* a CUDA runtime call failed                  */
  WAL_ERR_BUFFER_TOO_SMALL = 7, /* caller buffer smaller than required        */
  WAL_ERR_PEER_TIMEOUT = 8      /* a peer's data did not arrive in time       */
} wal_status;

typedef enum wal_dtype { WAL_BF16 = 0, WAL_F32 = 1, WAL_F16 = 2 } wal_dtype;

/* How the stage values become a weight (wal_rvq_layer.sum_mode).
 * WAL_SUM_EXACT: the reference's per_group reconstruction (src/runtime.py:379-414):
 *   w = T( T( sum_s fp32(C_s[id]) ) * T(rho) ), the stage sum in fp32 from +0.0.
 * WAL_SUM_FAST: the reference's reconstruct_weight_fast (src/runtime.py:431-448,
 *   :568-598), used by its *_fast and hot strategies: every stage table is
 *   rounded to T once (times T(stage scale), rounded, when scales exist) and
 *   the stages are added in T, in order: w = T( T(T(C_0[id]) + T(C_1[id])) * T(rho) ).
 * T is the weight type: bf16 for bf16 activations, fp16 for fp16 ones, fp32
 * for fp32 ones (where both modes differ only in the sign of zero sums). */
#define WAL_SUM_EXACT 0
#define WAL_SUM_FAST 1

/* Rows per packed tile and blocks per packed chunk (layout constants). */
#define WAL_TILE_ROWS 16
#define WAL_CHUNK_BLOCKS 16

/* Shape of one packed linear. */
typedef struct wal_rvq_geometry {
  int64_t out_features; /* N (sum of group rows)                                  */
  int64_t in_features;  /* K, a multiple of 4                                      */
  int32_t block_size;   /* d in {8, 16, 32}                                         */
  int32_t num_stages;   /* R in 1..4                                                */
  int32_t num_entries;  /* codebook rows per stage: <= 256 (1-byte ids) or, for     */
                        /* R == 1, <= 32767 (2-byte ids, e.g. route*256 + code)     */
  int32_t num_groups;   /* row groups, each with its own R codebooks               */
} wal_rvq_geometry;

/* Device-resident packed linear.  All pointers are device pointers except
 * group_rows, a host array (read during the call only). */
typedef struct wal_rvq_layer {
  wal_rvq_geometry geom;
  int64_t num_tiles;          /* from wal_rvq_packed_size                            */
  const void* packed_ids;     /* packed id stream (layout in wal_rvq_pack)           */
  const int32_t* tile_table;  /* 4 x int32 per tile: group, first row, rows, 0       */
  const uint16_t* codebooks;  /* fp16 [num_groups][R][num_entries][d]                */
  const uint16_t* row_scale;  /* fp16 [N]                                            */
  const uint16_t* bias;       /* bf16 [N] or NULL                                    */
  const int64_t* group_rows;  /* HOST [num_groups] rows per group; NULL if 1 group   */
  const float* stage_scales;  /* fp32 [num_groups][R] per-stage scales or NULL: each */
                              /* stage value is RN(fp32(c) * scale) before the sum   */
                              /* (reference src/block_vq.py:264-268)                 */
  int32_t sum_mode;           /* WAL_SUM_EXACT or WAL_SUM_FAST                       */
} wal_rvq_layer;

/* Human-readable text for a status code (static storage). */
WAL_API const char* wal_status_string(int status);

/* Library version as an integer (major * 10000 + minor * 100 + patch). */
WAL_API int wal_version(void);

/*
 * Size of the packed id stream and tile count for a geometry whose groups
 * have the given row counts (host array of num_groups values summing to N).
 * Replaces the buffer registration of reference src/runtime.py:262-265
 * (stage_ids_{i} buffers) with one tile-major stream.
 */
WAL_API int wal_rvq_packed_size(const wal_rvq_geometry* geom, const int64_t* group_rows,
                        size_t* packed_bytes, int64_t* num_tiles);

/*
 * Host re-layout of per-group, per-stage id matrices into the packed stream.
 * stage_ids[g * R + s] points to a host [rows_g, blocks] row-major matrix of
 * uint8 (num_entries <= 256) or uint16/int16 ids, blocks = ceil(K / d).
 * Every id is checked against num_entries (WAL_ERR_ID_RANGE).
 *
 * Layout: tiles of 16 rows (groups padded to whole tiles with id 0), each tile
 * split into chunks of 16 blocks; chunk = 16 rows x R stages x 16 ids, id
 * width 1 or 2 bytes little-endian, i.e. 16*R*idw bytes per row-chunk, so a
 * row-chunk is whole 16-byte vectors and each 8-row half of a chunk is one
 * contiguous, 128-byte-aligned run.  tile_table receives (group, first output
 * row, valid rows, 0) per tile.
 * Replaces reference src/runtime.py:249-344 (PackedBlockRVQGroup.__init__
 * buffer registration) and src/runtime.py:855-876 (_triton_state id stacking).
 */
WAL_API int wal_rvq_pack(const wal_rvq_geometry* geom, const int64_t* group_rows,
                 const void* const* stage_ids, void* packed, size_t packed_bytes,
                 int32_t* tile_table);

/*
 * Route-codebook packing: a uint8 route (< num_routes) and a uint8 code per
 * unit, host [N, blocks] each, become single-stage 2-byte ids
 * route * 256 + code into a flattened [num_routes * 256, d] codebook.
 * geom must have num_stages == 1, num_groups == 1 and
 * num_entries == num_routes * 256.  No reference module exists for this
 * format; it is the one-stage special case of reference src/runtime.py:379-414.
 */
WAL_API int wal_route_pack(const wal_rvq_geometry* geom, const uint8_t* route, const uint8_t* code,
                   void* packed, size_t packed_bytes, int32_t* tile_table);

/*
 * Decode GEMV (any M; up to 32 tokens per kernel launch, larger M in slabs of
 * 32): y[M, N] = x[M, K] @ w^T (+ bias).
 * x: device bf16, row stride ldx elements (ldx >= K, ldx % 4 == 0, 8-byte
 * aligned base; ldx % 8 == 0 with a 16-byte aligned base is fastest).  y: device, row stride ldy elements, dtype y_dtype
 * (WAL_BF16: one rounding of the fp32 result; WAL_F32: the fp32 result).
 * Replaces reference src/runtime.py:1362-1507 (PackedGroupedBlockRVQLinear.forward)
 * and src/triton_id_matmul.py:220-306 (rvq_group_linear_matmul).
 */
WAL_API int wal_rvq_gemv(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                 void* y, int64_t ldy, int y_dtype, void* stream);

/*
 * Decode GEMV with the activation type explicit: x_dtype WAL_BF16 or WAL_F16
 * (weights decoded and multiplied in that type, as the reference's forward in
 * x.dtype does, src/runtime.py:1501-1507 with reconstruct_weight(x.dtype));
 * y_dtype WAL_BF16, WAL_F16 or WAL_F32.  x_dtype WAL_F32 runs fp32 weights
 * (w = fp32(sum) * fp32(rho)) with fp32 fused multiply-adds on the CUDA
 * cores and needs y_dtype WAL_F32.  warps_per_tile and num_ctas as in
 * wal_rvq_gemv_ex (0 = library default).
 */
WAL_API int wal_rvq_gemv_typed(const wal_rvq_layer* layer, const void* x, int x_dtype, int64_t M, int64_t ldx,
                       void* y, int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas, void* stream);

/*
 * Prefill GEMM (large M): y[M, N] = x[M, K] @ w^T (+ bias) on the tcgen05
 * tensor cores, two SMs per tile (a cluster of 2 CTAs issuing cta_group::2
 * MMAs).  Weight tiles are decoded exactly (same arithmetic as the GEMV) into
 * shared memory per 64-column stage; x tiles arrive by TMA (no multicast).
 * Supports d = 8, R in {1, 2}, <= 256 entries; row groups must start at a
 * multiple of 128 rows.  x: bf16, ldx % 8 == 0, 16-byte aligned base.
 * y_dtype: WAL_BF16 or WAL_F32; y takes 16-byte stores of whole output
 * pieces when its base and its row stride (ldy elements) are multiples of 16
 * bytes, scalar stores otherwise (any ldy >= N works; the elements of a row
 * past N are not written).  status: optional device int, set to 1 if a
 * pipeline wait timed out (the CTA then stops and frees its resources), NULL
 * to skip.  Returns WAL_ERR_UNSUPPORTED for other configurations (callers use
 * wal_rvq_gemv).  Replaces reference src/runtime.py:1501-1507 for large M (the
 * module uses it from 128 tokens).
 */
WAL_API int wal_rvq_gemm(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                 void* y, int64_t ldy, int y_dtype, int* status, void* stream);

/*
 * Prefill GEMM with the activation type explicit: x_dtype WAL_BF16 or
 * WAL_F16 (weights decoded in that type, MMA operands of that type, fp32
 * accumulation); y_dtype WAL_BF16, WAL_F16 or WAL_F32.  Supports the
 * configurations of wal_rvq_gemm in both sum modes, plus one-stage tables with
 * a stage scale and fast-mode tables with stage scales; otherwise (and for
 * x_dtype WAL_F32) returns WAL_ERR_UNSUPPORTED.
 */
WAL_API int wal_rvq_gemm_typed(const wal_rvq_layer* layer, const void* x, int x_dtype, int64_t M, int64_t ldx,
                       void* y, int64_t ldy, int y_dtype, int* status, void* stream);

/*
 * Same as wal_rvq_gemv with an explicit split of each 16-row tile's blocks
 * over `warps_per_tile` warps (1, 2, 4 or 8; 0 = library default) and an
 * explicit CTA count (0 = one persistent wave).  For tuning and tests.
 */
WAL_API int wal_rvq_gemv_ex(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                    void* y, int64_t ldy, int y_dtype, int warps_per_tile, int num_ctas,
                    void* stream);

/*
 * Materialise the bf16 weight [N, K] (row stride ldw) from the packed form,
 * bit-identical to reference src/runtime.py:1234-1236
 * (PackedGroupedBlockRVQLinear.reconstruct_weight(torch.bfloat16)).
 */
WAL_API int wal_rvq_dequant(const wal_rvq_layer* layer, uint16_t* w, int64_t ldw, void* stream);

/*
 * The weight [N, K] in w_dtype (WAL_BF16, WAL_F16 or WAL_F32), bit-identical
 * to reference src/runtime.py:1234-1236 reconstruct_weight(out_dtype) for
 * WAL_SUM_EXACT and to reconstruct_weight_fast(out_dtype) (:1238-1240) for
 * WAL_SUM_FAST.
 */
WAL_API int wal_rvq_dequant_typed(const wal_rvq_layer* layer, void* w, int64_t ldw, int w_dtype, void* stream);

/*
 * Read the packed stream back into per-stage id matrices on the device:
 * ids [R][N][blocks] with 1-byte (num_entries <= 256) or 2-byte elements.
 * Used to prove the re-layout is lossless (ids must round-trip bit-exactly).
 */
WAL_API int wal_rvq_unpack_ids(const wal_rvq_layer* layer, void* ids, void* stream);

/* ------------------------------------------------------------------------
 * Per-block corrections (reference src/runtime.py:389-412): after the fp32
 * stage sum S of a block (one unit, d columns), in this order
 *   WAL_CORR_SIGN         S += (sigma * residual_scale[u]) @ sign_matrix, sigma_i = +1
 *                         when bit i of residual_signs[u] is set, else -1
 *   WAL_CORR_BLOCK_SCALE  S *= block_scale[u]
 *   WAL_CORR_POLAR        S = inverse polar transform of S (radius, then angle
 *                         groups of widths 1, 2, 4, ..., angles in units of pi)
 *   WAL_CORR_MATRIX       S = S @ transform[g]          (otherwise, if set)
 *   WAL_CORR_BIAS         S += transform_bias[g]
 * then w = T(T(S) * T(rho)).  Unit u = row * blocks + block over the layer's
 * rows (groups concatenated).  The matrix products run in ascending index
 * order with fused multiply-adds; the reference's CPU matrix product may sum
 * in another order, so a weight can differ in the last fp32 bit before its
 * rounding (visible after rounding in about one weight in 10^4).
 * ------------------------------------------------------------------------ */
#define WAL_CORR_SIGN 1
#define WAL_CORR_BLOCK_SCALE 2
#define WAL_CORR_MATRIX 4
#define WAL_CORR_POLAR 8
#define WAL_CORR_BIAS 16

typedef struct wal_rvq_corrections {
  const int32_t* group_flags;     /* device int32 [num_groups]: WAL_CORR_* bits          */
  const int32_t* residual_signs;  /* device int32 [N * blocks] (sign bits) or NULL      */
  const uint16_t* residual_scale; /* device fp16 [N * blocks] or NULL                   */
  const uint16_t* block_scale;    /* device fp16 [N * blocks] or NULL                   */
  const float* sign_matrix;       /* device fp32 [d][d] or NULL                         */
  const float* transform;         /* device fp32 [num_groups][d][d] or NULL             */
  const float* transform_bias;    /* device fp32 [num_groups][d] or NULL                */
} wal_rvq_corrections;

/*
 * y[M, N] = x[M, K] @ w^T (+ bias) for a layer with corrections, x_dtype
 * WAL_BF16 / WAL_F16 / WAL_F32 (weights in that type), y_dtype any of the
 * three; CUDA-core fp32 accumulation, 8 tokens per launch.  The layer's
 * sum_mode must be WAL_SUM_EXACT (the reference's fast reconstruction does not
 * take corrections).  Replaces reference src/runtime.py:1501-1507 for such
 * encodings, which the reference's fused kernels refuse (src/runtime.py:837-853).
 */
WAL_API int wal_rvq_gemv_corrected(const wal_rvq_layer* layer, const wal_rvq_corrections* corr, const void* x,
                           int x_dtype, int64_t M, int64_t ldx, void* y, int64_t ldy, int y_dtype, void* stream);

/* The corrected weight [N, K] in w_dtype (reference reconstruct_weight(out_dtype)). */
WAL_API int wal_rvq_dequant_corrected(const wal_rvq_layer* layer, const wal_rvq_corrections* corr, void* w,
                              int64_t ldw, int w_dtype, void* stream);

/* ------------------------------------------------------------------------
 * Encoder: nearest codebook entry (reference src/block_vq.py:180-196,
 * _assign_to_codebook, the hot loop of its k-means fit and of every stage's
 * assignment).  blocks: device fp32 [n][d]; codebook: device fp32
 * [num_entries][d]; ids: device int32 [n] receives the entry minimising
 * ||x||^2 + ||c||^2 - 2 x.c (fp32; the first of equal minima), min_dist
 * (device fp32 [n] or NULL) that distance.  d in {4, 8, 16, 32}; the codebook
 * must fit in shared memory ((num_entries * (d + 1)) * 4 <= 227 KB).  A block
 * whose two best entries lie within a few fp32 units of each other can be
 * assigned differently from the reference's CPU matrix product.
 * ------------------------------------------------------------------------ */
WAL_API int wal_rvq_assign(const float* blocks, int64_t n, int32_t d, const float* codebook, int32_t num_entries,
                   int32_t* ids, float* min_dist, void* stream);

/* ------------------------------------------------------------------------
 * ID-route linear (reference src/runtime.py:52-97, PackedIDRouteLinear; fused
 * Triton kernel src/triton_id_matmul.py:19-67): one int16 id per weight into
 * a scalar fp16 route table codebook_sum[num_routes].  The weight is, bit for
 * bit, the reference's bf16 weight
 *   w[n, k] = bf16_rn( fp16_rn( codebook_sum[ids[n, k]] * row_scale[n] ) ).
 * Packed ids: tiles of 16 rows, chunks of 128 columns of 4 KB each (eight
 * 512-byte warp-wide vectors; order in wal_idroute_pack), padding ids 0.
 * ------------------------------------------------------------------------ */
typedef struct wal_idroute_layer {
  int64_t out_features;          /* N                                             */
  int64_t in_features;           /* K, a multiple of 8                            */
  int32_t num_routes;            /* table entries, <= 32767                       */
  const void* packed_ids;        /* device, from wal_idroute_pack                 */
  const uint16_t* codebook_sum;  /* device fp16 [num_routes]                      */
  const uint16_t* row_scale;     /* device fp16 [N]                               */
  const uint16_t* bias;          /* device bf16 [N] or NULL                       */
} wal_idroute_layer;

/* Bytes of the packed id stream for an N x K weight. */
WAL_API int wal_idroute_packed_size(int64_t out_features, int64_t in_features, size_t* packed_bytes);

/*
 * Host re-layout of int16 ids [N][K] (row-major) into the packed stream:
 * chunk (tile t, columns 128c..128c+127) at byte (t * chunks + c) * 4096;
 * inside it, row 8h + r (h = 0, 1), columns 32g + 16u + 4q + j (g < 4, u < 2,
 * q < 4, j < 4) at byte (h * 4 + g) * 512 + (r * 4 + q) * 16 + u * 8 + j * 2.
 * Every id is checked against num_routes (WAL_ERR_ID_RANGE).  Replaces the
 * int16 `ids` buffer of reference src/runtime.py:59-62.
 */
WAL_API int wal_idroute_pack(int64_t out_features, int64_t in_features, int32_t num_routes,
                     const int16_t* ids, void* packed, size_t packed_bytes);

/*
 * y[M, N] = x[M, K] @ w^T (+ bias), x bf16 (ldx % 4 == 0, 8-byte aligned),
 * y bf16 or fp32, fp32 accumulation, up to 16 tokens per launch (slabs
 * beyond).  Replaces reference src/runtime.py:95-97 (forward) and
 * src/triton_id_matmul.py:70-150 (id_route_linear_matmul).
 */
WAL_API int wal_idroute_gemv(const wal_idroute_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                     void* y, int64_t ldy, int y_dtype, void* stream);

/* The weight [N, K] (row stride ldw): w_dtype WAL_F16 gives reference
 * src/runtime.py:89-93 (reconstruct_weight) bit for bit, WAL_BF16 the same
 * followed by .to(torch.bfloat16) (the forward's weight). */
WAL_API int wal_idroute_dequant(const wal_idroute_layer* layer, uint16_t* w, int64_t ldw, int w_dtype,
                        void* stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel decode.  No reference counterpart: the reference runs one
 * device.  A row-parallel linear (o_proj, down_proj split along K) produces
 * an fp32 partial output on every rank.  wal_rvq_gemv_push stores each
 * element of its partial straight into a receive slot in every rank's memory
 * (peer pointers over NVLink, mapped with wal_peer_region_open) as one 8-byte
 * word {fp32 value, uint32 tag}; the tag is the slot's call count + 1, so a
 * word is fresh exactly when its tag matches and no fence or flag is needed
 * (an aligned 8-byte store arrives whole).  wal_tp_reduce_rmsnorm on every
 * rank waits (bounded) for all ranks' words, sums them in rank order (every
 * rank then holds identical values), adds the residual, applies the next
 * RMSNorm and advances the slot's call count.
 * ------------------------------------------------------------------------ */
#define WAL_MAX_RANKS 8
#define WAL_IPC_HANDLE_BYTES 64

typedef struct wal_tp_push {
  int32_t num_ranks;            /* P in 1..WAL_MAX_RANKS                                    */
  int32_t rank;                 /* this rank                                                */
  void* dst[WAL_MAX_RANKS];     /* dst[p]: rank p's receive rows for this rank, 8-byte words */
  int64_t ld_dst;               /* row stride of every dst[p] in words (>= N)               */
  const uint32_t* epoch;        /* this rank's call count of the slot (device)              */
} wal_tp_push;

/*
 * Decode GEMV whose fp32 output rows are stored, tagged with *epoch + 1,
 * into dst[p] for every rank p.  Bias is not added (row-parallel partials).
 */
WAL_API int wal_rvq_gemv_push(const wal_rvq_layer* layer, const uint16_t* x, int64_t M, int64_t ldx,
                      const wal_tp_push* push, void* stream);

/*
 * Receiving half of the exchange.  recv: this rank's receive slot, words
 * [num_ranks][rank_stride] with rows ld words apart; epoch/done: this rank's
 * call count and CTA counter of the slot (device, start at zero).  Waits
 * until every word of rows < M carries tag *epoch + 1 (bounded, about 2 s),
 * then h <- bf16(h + bf16(sum_p value_p)) (fp32 sum in rank order),
 * x_out <- bf16(RMSNorm(h) * norm_weight), and *epoch += 1.  On timeout writes
 * WAL_ERR_PEER_TIMEOUT to *status (if not NULL) and leaves h, x_out and the
 * call count unchanged.  h, norm_weight, x_out: bf16; N % 8 == 0, N <= 16384.
 */
WAL_API int wal_tp_reduce_rmsnorm(const void* recv, int32_t num_ranks, int64_t rank_stride, int64_t ld,
                          uint32_t* epoch, uint32_t* done, uint16_t* h, int64_t ldh,
                          const uint16_t* norm_weight, float eps, uint16_t* x_out, int64_t ldx,
                          int64_t M, int64_t N, int* status, void* stream);

/*
 * Sending half of the exchange for an output another kernel produced (a dense
 * library GEMM, say): y (WAL_F32 or WAL_BF16, rows < M, N columns, row stride
 * ldy) is stored into dst[p] of every rank p as {value, tag} words, two words
 * per 16-byte store, tag = *epoch + 1; wal_tp_reduce_rmsnorm receives it
 * exactly like the words of wal_rvq_gemv_push.  N, ldy and push->ld_dst even;
 * every dst[p] 16-byte aligned.
 */
WAL_API int wal_tp_push_rows(const void* y, int64_t ldy, int y_dtype, int64_t M, int64_t N, const wal_tp_push* push,
                     void* stream);

/*
 * Local form: h <- bf16(h + bf16(partial)) when partial (fp32, rows ldp apart)
 * is not NULL, then x_out <- bf16(h * rsqrt(mean(h^2) + eps) * norm_weight).
 */
WAL_API int wal_residual_rmsnorm(const float* partial, int64_t ldp, uint16_t* h, int64_t ldh,
                         const uint16_t* norm_weight, float eps, uint16_t* x_out, int64_t ldx,
                         int64_t M, int64_t N, void* stream);

/*
 * Rotary embedding (rotate-half) of q and k for one position plus the KV
 * cache append.  qkv: bf16 [M, ld_qkv] holding q (hq heads), k, v (hkv heads
 * each) of head_dim hd.  cos/sin: fp32 [hd].  q_out: bf16 [M, hq * hd].
 * k_cache/v_cache: bf16 [M, hkv, cache_len, hd] (contiguous); position pos
 * is written.  Rounding as x.float() * cos + rotate_half(x).float() * sin
 * with separately rounded products, then one bf16 rounding.
 */
WAL_API int wal_rope_kv_append(const uint16_t* qkv, int64_t ld_qkv, int64_t M, int32_t hq, int32_t hkv,
                       int32_t hd, const float* cos, const float* sin, int64_t pos, uint16_t* q_out,
                       uint16_t* k_cache, uint16_t* v_cache, int64_t cache_len, void* stream);

/* out[m, i] = bf16(bf16(silu(g[m, i])) * u[m, i]) with g = gu[m, 0:I], u = gu[m, I:2I] (bf16). */
WAL_API int wal_silu_mul(const uint16_t* gu, int64_t ld_gu, int64_t M, int64_t I, uint16_t* out,
                 int64_t ld_out, void* stream);

/*
 * Decode attention (one query token per sequence, grouped-query heads):
 * out[b, h*hd:(h+1)*hd] = softmax(q[b, h] . k[b, h/G, t] * scale) v[b, h/G, t]
 * over positions t < n, G = hq / hkv.  q: bf16 rows ld_q apart (q heads
 * contiguous, 8-byte aligned); k_cache/v_cache: bf16 [B, hkv, cache_len, hd]
 * contiguous, 16-byte aligned; out: bf16 rows ld_out apart.  hd in {64, 128},
 * G in {1, 2, 4, 8}.
 * workspace: device scratch of at least wal_decode_attention_workspace(B, hq,
 * hkv, hd, max_n) bytes for calls with n <= max_n positions (the size covers
 * the largest split count of any such n), 256-byte aligned and zero-filled
 * before its first use.  Its merge counters sit at a fixed offset at the
 * front and every call leaves them at zero, so one workspace serves a whole
 * decode loop whose n grows; calls sharing one workspace must not overlap in
 * time.  Split-K over positions with an exact (log-sum-exp) merge in split
 * order: deterministic.  Few (sequence, kv head) pairs get the fewest splits
 * of at most 128 positions, each staged in one round; many pairs get fewer,
 * longer splits (about 2.6 CTAs per SM) that stream through two 64-position
 * stage buffers.  The merge keeps 8 * G bytes per split in shared
 * memory: a call whose splits (about n / 128 at large n) do not fit in 227 KB
 * returns WAL_ERR_SHAPE (hd = 128, G = 8: n <= 366,592 positions).  No
 * reference counterpart (the reference runs Hugging Face attention).
 */
WAL_API size_t wal_decode_attention_workspace(int64_t B, int32_t hq, int32_t hkv, int32_t hd, int64_t n);
WAL_API int wal_decode_attention(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache,
                         const uint16_t* v_cache, int64_t B, int32_t hq, int32_t hkv, int32_t hd,
                         int64_t cache_len, int64_t n, float scale, uint16_t* out, int64_t ld_out,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * wal_decode_attention with an explicit split count (0 = library default):
 * num_splits splits of at least 32 positions each (num_splits <= ceil(n /
 * 32), else WAL_ERR_SHAPE; splits longer than 128 positions stream); the
 * workspace must hold that many splits' partials (WAL_ERR_BUFFER_TOO_SMALL
 * otherwise).  For tuning and tests.
 */
WAL_API int wal_decode_attention_ex(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache,
                         const uint16_t* v_cache, int64_t B, int32_t hq, int32_t hkv, int32_t hd,
                         int64_t cache_len, int64_t n, float scale, uint16_t* out, int64_t ld_out,
                         void* workspace, size_t workspace_bytes, int num_splits, void* stream);

/*
 * Decode attention that allocates nothing, for callers that cannot call
 * cudaMalloc: a plugin run by a host engine that owns all device memory and
 * hands it inputs and outputs but no workspace, or a serving loop that must
 * not stall on the device-wide synchronisation a cudaMalloc/cudaFree pair
 * brings.  Arguments and results (bit-identical) are those of
 * wal_decode_attention without the workspace: the scratch is a 4 MiB array
 * compiled into this library, which every GPU that loads the library keeps
 * until the process exits.  Limit: B * hkv <= 4096 and the call's split
 * partials and statistics (B * hkv * nsplit * G * (hd + 2) * 4 bytes) within
 * 4 MiB - 16 KiB (Llama-3-8B heads at 2048 positions fit up to batch 55);
 * larger calls return WAL_ERR_BUFFER_TOO_SMALL and launch nothing.  Each call clears the merge counters it uses with an
 * asynchronous memset on the stream before its kernel.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress, that
 * device current); make that first call before any stream capture.  Every
 * call on a device uses the same array, so calls that can overlap on the GPU
 * (other streams, other host threads) race and corrupt each other's results.
 * No counterpart in the reference.
 */
WAL_API int wal_decode_attention_static(const uint16_t* q, int64_t ld_q, const uint16_t* k_cache,
                         const uint16_t* v_cache, int64_t B, int32_t hq, int32_t hkv, int32_t hd,
                         int64_t cache_len, int64_t n, float scale, uint16_t* out, int64_t ld_out,
                         void* stream);

/*
 * Device memory shared with peer processes: create (cudaMalloc, zero-filled,
 * IPC handle of WAL_IPC_HANDLE_BYTES written to handle_out), open a peer's
 * handle (mapped with peer access), close a mapping, free own memory.
 */
WAL_API int wal_peer_region_create(size_t bytes, void** dev_ptr, void* handle_out);
WAL_API int wal_peer_region_open(const void* handle, void** dev_ptr);
WAL_API int wal_peer_region_close(void* dev_ptr);
WAL_API int wal_peer_region_free(void* dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* WAL_RVQ_H */
