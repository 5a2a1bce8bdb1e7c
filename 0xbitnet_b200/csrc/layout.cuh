// layout.cuh — the device weight layout ("T16") and its index arithmetic.
//
// GGUF I2_S stores each output row m as in_dim/4 bytes: 128-element blocks of
// 32 bytes, byte gp of a block holding elements gp, 32+gp, 64+gp, 96+gp in bits
// 7:6, 5:4, 3:2, 1:0 (code c = weight + 1). Splitting a block into two 16-byte
// halves h, the 16 bytes of half h hold, for each group g, the 16 consecutive
// elements 32g+16h .. 32g+16h+15, one 2-bit field per byte. That is what makes
// the format SIMD-friendly: (word >> (6-2g)) & 0x03030303 yields four int8
// codes of four consecutive elements.
//
// The repack keeps every 16-byte half intact and only moves it:
//
//   rows are padded to a multiple of 128 with code 1 (weight 0); then
//   byte offset of (row m, block b, half h) =
//       ((m/16) * KB + b) * 512 + h * 256 + (m%16) * 16,   KB = in_dim / 128.
//
// A 16-row subtile is one contiguous KB * 512-byte run (a single bulk copy for a
// GEMV CTA); inside it each block is 512 bytes ordered [half][row][16 B], so a
// warp reads a subtile's block with one fully coalesced 512-byte access (lane =
// half*16 + row). The tensor-core GEMM fetches a 128-row x 2-block stage with a
// single 3D TMA copy (box: 512 bytes x 2 blocks x 8 subtiles).
#pragma once

#include <cstdint>

namespace obn {

constexpr int kTileRows = 128;      // row padding (one GEMM weight tile)
constexpr int kSubRows = 16;        // rows per subtile
constexpr int kBlockK = 128;        // elements per I2_S block
constexpr int kSubtileBytes = 512;  // one block of one subtile: 16 rows x 32 bytes

__host__ __device__ inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

// Byte offset of block b of subtile S (= m / 16).
__host__ __device__ inline size_t subtile_offset(int S, int b, int KB) {
  return (static_cast<size_t>(S) * KB + b) * kSubtileBytes;
}

// Byte offset of the 16-byte half (row m, block b, half h).
__host__ __device__ inline size_t half_offset(int m, int b, int h, int KB) {
  return subtile_offset(m / 16, b, KB) + static_cast<size_t>(h) * 256 + (m % 16) * 16;
}

}  // namespace obn
