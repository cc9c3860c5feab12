// Tiled HBM layout of quantized weights (the "slx tile" format).
//
// The slot pool stores every expert in the byte order the GEMV kernels
// stream, so one 16-row tile arrives in a handful of large bulk copies (the
// copy engine's cost is per request; small requests cap bandwidth):
//
//   pair tile   (gate/up rows r..r+15 of one expert, or rows r..r+15 and
//                r+16..r+31 of a dense matrix):
//                [P: 16 rows x RB bytes][Q: 16 rows x RB bytes]
//                [SB: nG x 32 words, word (G, m, row) = scale | bias << 16]
//   single tile (down rows r..r+15 of one expert):
//                [16 rows x RB bytes][SB: nG x 16 words]
//
// RB = in*bits/8 packed bytes per row (MLX affine codes, unchanged), nG =
// in/64.  Inside a row, 16-byte unit u is stored at u ^ (row & 7) when RB is
// a multiple of 128 (XOR swizzle: the fragment reads of 8 rows then hit 8
// different bank quads).  Scale/bias words are ordered so the 32 lanes of a
// warp read 32 consecutive words.
//
// Expert slot = (I/16) pair tiles over in = H, then (H/16) single tiles over
// in = I; same total bytes as the MLX layout.  A dense [out, in] matrix =
// ceil(out/32) pair tiles (rows past `out` are zero).
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __CUDACC__
#define SLX_TILE_FN __host__ __device__ __forceinline__
#else
#define SLX_TILE_FN inline
#endif

namespace slx {

SLX_TILE_FN int tile_rb(int in, int bits) { return in * bits / 8; }
SLX_TILE_FN int tile_ng(int in) { return in / 64; }
SLX_TILE_FN bool tile_swizzled(int in, int bits) {
  return (tile_rb(in, bits) % 128) == 0;
}
SLX_TILE_FN size_t pair_tile_bytes(int in, int bits) {
  return (size_t)32 * tile_rb(in, bits) + (size_t)128 * tile_ng(in);
}
SLX_TILE_FN size_t single_tile_bytes(int in, int bits) {
  return (size_t)16 * tile_rb(in, bits) + (size_t)64 * tile_ng(in);
}
// bytes of region A (gate/up pair tiles) of one expert
SLX_TILE_FN size_t expert_a_bytes(int H, int I, int bits) {
  return (size_t)(I / 16) * pair_tile_bytes(H, bits);
}
SLX_TILE_FN size_t expert_tiled_bytes(int H, int I, int bits) {
  return expert_a_bytes(H, I, bits) + (size_t)(H / 16) * single_tile_bytes(I, bits);
}
SLX_TILE_FN size_t dense_tiled_bytes(int out, int in, int bits) {
  return (size_t)((out + 31) / 32) * pair_tile_bytes(in, bits);
}
// byte offset of (row, byte b of the packed row) inside a tile's row block
SLX_TILE_FN int swz_offset(int row, int b, int RB, bool swz) {
  const int u = b >> 4;
  return row * RB + (((swz ? (u ^ (row & 7)) : u)) << 4) + (b & 15);
}

}  // namespace slx
