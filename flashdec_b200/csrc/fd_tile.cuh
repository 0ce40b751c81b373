// Shared-memory layout of one K/V tile as the TMA writes it (128B swizzle),
// shared by the decode kernels of fd_attention.cu and fd_wave_decode.cu.
#pragma once

#include <cstdint>

namespace fd {

constexpr int kTile = 32;  // tokens per tile

// Column of element (row, col) in a merge buffer of 128-float-aligned rows:
// XOR with 8 * (row % 4) so that consecutive rows start on different banks.
__device__ __forceinline__ int merge_col(int row, int col) { return col ^ ((row & 3) << 3); }

// Stage tiles (one 32-token tile of K or V).  Default layout (kPageRows 0):
// D/64 halves of [32 rows][64 dims], one TMA box per (page, half).  With
// kPageRows = 16 or 8 (head_dim 128, pages of that many tokens, one box per
// page plane): [page][half][kPageRows rows][64 dims].  Both carry the TMA
// 128B swizzle, which depends only on the shared-memory address (16-byte
// chunk index XOR address bits 7-9 = row % 8; every half of a page starts on
// a 1 KB boundary).
template <int kPageRows>
__device__ __forceinline__ uint32_t stage_row_base(int row, int half) {
  if constexpr (kPageRows > 0) {
    return (row / kPageRows) * (kPageRows * 256) + half * (kPageRows * 128) +
           (row % kPageRows) * 128;
  } else {
    return half * (kTile * 128) + row * 128;
  }
}
// Byte distance of 16 tile rows and of one 64-dim half in a stage, for the
// per-lane ldmatrix offsets that are hoisted out of the tile loop: row
// r + 16 np of half h of chunk (8 h + c8) sits at
//   stage_row_base(r, 0) + np * kRows16Bytes + h * kHalfStride + ((c8 ^ (r % 8)) << 4)
// for r < 16 (a multiple-of-8 row shift keeps r % 8, hence the swizzle).
template <int kPageRows>
struct StageStrides {
  static constexpr uint32_t kRows16Bytes = kPageRows > 0 ? (16 / kPageRows) * (kPageRows * 256) : 16 * 128;
  static constexpr uint32_t kHalfStride = kPageRows > 0 ? kPageRows * 128 : kTile * 128;
};

template <int kPageRows>
__device__ __forceinline__ uint32_t stage_tile_offset(int row, int dim) {
  const int dd = dim & 63;
  return stage_row_base<kPageRows>(row, dim >> 6) + (((dd >> 3) ^ (row & 7)) << 4) +
         ((dd & 7) << 1);
}
template <int kPageRows>
__device__ __forceinline__ uint32_t stage_chunk_offset(int row, int chunk) {
  return stage_row_base<kPageRows>(row, chunk >> 3) + (((chunk & 7) ^ (row & 7)) << 4);
}

// Byte offset of element (row, dim) in a [32][D] tile stored as D/64 halves
// of [32][64] with the TMA 128B swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t tile_offset(int row, int dim) {
  const int dd = dim & 63;
  return (dim >> 6) * (kTile * 128) + row * 128 + (((dd >> 3) ^ (row & 7)) << 4) + ((dd & 7) << 1);
}

// Byte offset of 16-byte chunk `chunk` (8 dims) of `row`.
__device__ __forceinline__ uint32_t chunk_offset(int row, int chunk) {
  return (chunk >> 3) * (kTile * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

__device__ __forceinline__ int tmap_coord(int axis, int kv_head, int blk) {
  return axis == 1 ? kv_head : (axis == 2 ? blk : 0);  // token and half start at 0
}

}  // namespace fd
