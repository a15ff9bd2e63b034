// Host-side part of the C ABI: status strings, packed-size computation and
// the re-layout of per-stage id matrices into the tile-major packed stream.
//
// The packed stream replaces the per-stage [rows, blocks] id buffers the
// reference registers on its runtime module (src/runtime.py:262-265) and the
// [stages, rows, blocks] stack it builds for its fused kernel
// (src/runtime.py:855-876).  Layout (all offsets in bytes):
//
//   tile t (16 rows) -> chunk c (16 blocks) -> vector v (V = R * idw vectors)
//   -> row rr (16 rows) -> 16 bytes
//
//   offset(t, c, v, rr) = ((t * NC + c) * V + v) * 256 + rr * 16
//
// where vector v = s * idw + h holds ids of stage s for blocks
// 16c + [16h/idw, 16(h+1)/idw) of that row, little-endian, idw bytes each.
// Each 128-byte run (8 rows of one vector) is what one warp-wide 16-byte load
// of eight row-owners reads, so every code load is a full, aligned line.
#include "../../include/wal_rvq.h"

#include <cstring>
#include <vector>

namespace {

int id_width(const wal_rvq_geometry* g) { return g->num_entries <= 256 ? 1 : 2; }

int check_geometry(const wal_rvq_geometry* g) {
  if (!g) return WAL_ERR_INVALID_ARGUMENT;
  if (g->out_features <= 0 || g->in_features <= 0 || g->num_groups <= 0) return WAL_ERR_SHAPE;
  if (g->block_size != 8 && g->block_size != 16 && g->block_size != 32) return WAL_ERR_UNSUPPORTED;
  if (g->num_stages < 1 || g->num_stages > 4) return WAL_ERR_UNSUPPORTED;
  if (g->num_entries < 1 || g->num_entries > 32767) return WAL_ERR_SHAPE;
  if (g->num_stages > 1 && g->num_entries > 256) return WAL_ERR_UNSUPPORTED;
  if (g->in_features % 4 != 0) return WAL_ERR_UNSUPPORTED;
  return WAL_OK;
}

struct Dims {
  int64_t blocks, chunks, vectors, tile_bytes;
};

Dims dims_of(const wal_rvq_geometry* g) {
  Dims d;
  d.blocks = (g->in_features + g->block_size - 1) / g->block_size;
  d.chunks = (d.blocks + WAL_CHUNK_BLOCKS - 1) / WAL_CHUNK_BLOCKS;
  d.vectors = (int64_t)g->num_stages * id_width(g);
  d.tile_bytes = d.chunks * d.vectors * 256;
  return d;
}

int count_tiles(const wal_rvq_geometry* g, const int64_t* group_rows, int64_t* tiles) {
  if (!group_rows) return WAL_ERR_INVALID_ARGUMENT;
  int64_t total_rows = 0, t = 0;
  for (int i = 0; i < g->num_groups; ++i) {
    if (group_rows[i] <= 0) return WAL_ERR_SHAPE;
    total_rows += group_rows[i];
    t += (group_rows[i] + WAL_TILE_ROWS - 1) / WAL_TILE_ROWS;
  }
  if (total_rows != g->out_features) return WAL_ERR_SHAPE;
  *tiles = t;
  return WAL_OK;
}

inline uint8_t* id_ptr(uint8_t* packed, const Dims& d, int idw, int64_t t, int64_t block, int s, int rr) {
  const int64_t c = block / WAL_CHUNK_BLOCKS;
  const int64_t j = block % WAL_CHUNK_BLOCKS;
  const int64_t byte_in_row = j * idw;  // 0..16*idw-1
  const int64_t v = (int64_t)s * idw + byte_in_row / 16;
  return packed + ((t * d.chunks + c) * d.vectors + v) * 256 + rr * 16 + byte_in_row % 16;
}

}  // namespace

extern "C" {

const char* wal_status_string(int status) {
  switch (status) {
    case WAL_OK: return "ok";
    case WAL_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or non-positive size)";
    case WAL_ERR_SHAPE: return "inconsistent or unsupported shape";
    case WAL_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case WAL_ERR_ID_RANGE: return "id or route out of range of its codebook";
    case WAL_ERR_UNSUPPORTED: return "configuration not implemented by this build";
    case WAL_ERR_CUDA: return "CUDA runtime error";
    case WAL_ERR_BUFFER_TOO_SMALL: return "caller buffer too small";
    case WAL_ERR_PEER_TIMEOUT: return "a peer rank's data did not arrive within the wait limit";
    default: return "unknown status";
  }
}

int wal_version(void) { return 100; }

int wal_rvq_packed_size(const wal_rvq_geometry* geom, const int64_t* group_rows, size_t* packed_bytes,
                        int64_t* num_tiles) {
  int st = check_geometry(geom);
  if (st != WAL_OK) return st;
  if (!packed_bytes || !num_tiles) return WAL_ERR_INVALID_ARGUMENT;
  int64_t tiles = 0;
  st = count_tiles(geom, group_rows, &tiles);
  if (st != WAL_OK) return st;
  const Dims d = dims_of(geom);
  *packed_bytes = (size_t)(tiles * d.tile_bytes);
  *num_tiles = tiles;
  return WAL_OK;
}

int wal_rvq_pack(const wal_rvq_geometry* geom, const int64_t* group_rows, const void* const* stage_ids,
                 void* packed, size_t packed_bytes, int32_t* tile_table) {
  size_t need = 0;
  int64_t tiles = 0;
  int st = wal_rvq_packed_size(geom, group_rows, &need, &tiles);
  if (st != WAL_OK) return st;
  if (!stage_ids || !packed || !tile_table) return WAL_ERR_INVALID_ARGUMENT;
  if (packed_bytes < need) return WAL_ERR_BUFFER_TOO_SMALL;
  const Dims d = dims_of(geom);
  const int idw = id_width(geom);
  const int R = geom->num_stages;
  const int64_t B = d.blocks;
  std::memset(packed, 0, need);
  uint8_t* out = static_cast<uint8_t*>(packed);
  int64_t t0 = 0, row0 = 0;
  for (int g = 0; g < geom->num_groups; ++g) {
    const int64_t rows = group_rows[g];
    for (int s = 0; s < R; ++s)
      if (!stage_ids[(size_t)g * R + s]) return WAL_ERR_INVALID_ARGUMENT;
    const int64_t nt = (rows + WAL_TILE_ROWS - 1) / WAL_TILE_ROWS;
    for (int64_t lt = 0; lt < nt; ++lt) {
      const int64_t t = t0 + lt;
      const int64_t first = lt * WAL_TILE_ROWS;
      const int64_t valid = rows - first < WAL_TILE_ROWS ? rows - first : WAL_TILE_ROWS;
      tile_table[4 * t + 0] = g;
      tile_table[4 * t + 1] = (int32_t)(row0 + first);
      tile_table[4 * t + 2] = (int32_t)valid;
      tile_table[4 * t + 3] = 0;
      for (int s = 0; s < R; ++s) {
        const void* src = stage_ids[(size_t)g * R + s];
        for (int64_t rr = 0; rr < valid; ++rr) {
          const int64_t row = first + rr;
          for (int64_t b = 0; b < B; ++b) {
            uint32_t id;
            if (idw == 1) {
              id = static_cast<const uint8_t*>(src)[row * B + b];
            } else {
              id = static_cast<const uint16_t*>(src)[row * B + b];
            }
            if (id >= (uint32_t)geom->num_entries) return WAL_ERR_ID_RANGE;
            uint8_t* p = id_ptr(out, d, idw, t, b, s, (int)rr);
            p[0] = (uint8_t)(id & 0xFF);
            if (idw == 2) p[1] = (uint8_t)(id >> 8);
          }
        }
      }
    }
    t0 += nt;
    row0 += rows;
  }
  return WAL_OK;
}

int wal_route_pack(const wal_rvq_geometry* geom, const uint8_t* route, const uint8_t* code, void* packed,
                   size_t packed_bytes, int32_t* tile_table) {
  int st = check_geometry(geom);
  if (st != WAL_OK) return st;
  if (!route || !code) return WAL_ERR_INVALID_ARGUMENT;
  if (geom->num_stages != 1 || geom->num_groups != 1 || geom->num_entries % 256 != 0 ||
      geom->num_entries <= 256)
    return WAL_ERR_SHAPE;
  const int num_routes = geom->num_entries / 256;
  const int64_t N = geom->out_features;
  const int64_t B = (geom->in_features + geom->block_size - 1) / geom->block_size;
  std::vector<uint16_t> ids((size_t)(N * B));
  for (int64_t i = 0; i < N * B; ++i) {
    if (route[i] >= num_routes) return WAL_ERR_ID_RANGE;
    ids[(size_t)i] = (uint16_t)(route[i] * 256 + code[i]);
  }
  const void* stage[1] = {ids.data()};
  const int64_t rows[1] = {N};
  return wal_rvq_pack(geom, rows, stage, packed, packed_bytes, tile_table);
}

}  // extern "C"
