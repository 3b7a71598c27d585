// Layout helpers of the tiled int8 activation operand shared by the prefill GEMM (ivb_gemm.cu) and the
// prefill orchestration (ivb_prefill.cu).
#pragma once

#include <cstddef>

namespace ivb {

constexpr int kGemmTile = 16384;  // bytes of one 128-token x 128-input activation tile

// Position of input i inside the GEMM activation layout: each 16-input block is a 4 x 4 byte transpose
// (byte 4f + b holds input 4b + f), which matches the codes a packed weight word yields by masking
// (w >> 2f) & 0x03030303 for f = 0..3.
__host__ __device__ __forceinline__ int gemm_slot(int i) { return (i & ~15) + ((i & 3) << 2) + ((i >> 2) & 3); }

// One 16-byte chunk (c) of row r in a K-major core-matrix tile: core matrices of 8 rows x 16 bytes,
// 8 chunks (128 inputs) per row group. LBO (next K chunk) = 128 B, SBO (next 8-row group) = 1024 B.
__host__ __device__ __forceinline__ int tile_off(int r, int c) { return (((r >> 3) << 3) + c) * 128 + ((r & 7) << 4); }

// Byte offset of (token t, 16-input chunk k) in the tiled activation buffer of row length ldq:
// 16 KB blocks per (token tile, 128-input group), each a core-matrix tile.
__host__ __device__ __forceinline__ size_t q8_chunk_offset(int t, int k, int ldq) {
  return (static_cast<size_t>(t >> 7) * (ldq >> 7) + (k >> 3)) * kGemmTile + tile_off(t & 127, k & 7);
}

}  // namespace ivb
