// Device side of the MLX-affine -> tile-format repack (slx_tiles.cuh),
// shared by the pack kernels (slx_pack.cu) and the decode SwitchGLU's
// in-kernel slot fill (slx_qgemv.cu).  Every function is called by all
// threads of a block and strides over the block.
#pragma once
#include "slx_common.cuh"
#include "slx_tiles.cuh"

namespace slx {

struct QSrc {
  const uint8_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

// rows p0.. of P and q0.. of Q (rows >= nrows are zero) -> one pair tile
SLX_DEV void pack_pair(uint8_t* dst, QSrc P, int p0, QSrc Q, int q0,
                       int nrows, int in, int bits) {
  const int RB = tile_rb(in, bits), nG = tile_ng(in);
  const bool swz = tile_swizzled(in, bits);
  const int units = RB / 16;
  for (int i = threadIdx.x; i < 32 * units; i += blockDim.x) {
    const int r32 = i / units, u = i % units;
    const int m = r32 >> 4, r = r32 & 15;
    const int srow = (m ? q0 : p0) + r;
    const QSrc src = m ? Q : P;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (srow < nrows)
      v = *reinterpret_cast<const uint4*>(src.w + (size_t)srow * RB + 16 * u);
    *reinterpret_cast<uint4*>(dst + m * 16 * RB + swz_offset(r, 16 * u, RB, swz)) = v;
  }
  uint32_t* sb = reinterpret_cast<uint32_t*>(dst + 32 * RB);
  for (int i = threadIdx.x; i < nG * 32; i += blockDim.x) {
    const int G = i >> 5, m = (i >> 4) & 1, r = i & 15;
    const int srow = (m ? q0 : p0) + r;
    const QSrc src = m ? Q : P;
    uint32_t word = 0;
    if (srow < nrows)
      word = (uint32_t)src.s[(size_t)srow * nG + G] |
             ((uint32_t)src.b[(size_t)srow * nG + G] << 16);
    sb[i] = word;
  }
}

SLX_DEV void pack_single(uint8_t* dst, QSrc D, int r0, int in, int bits) {
  const int RB = tile_rb(in, bits), nG = tile_ng(in);
  const bool swz = tile_swizzled(in, bits);
  const int units = RB / 16;
  for (int i = threadIdx.x; i < 16 * units; i += blockDim.x) {
    const int r = i / units, u = i % units;
    const uint4 v =
        *reinterpret_cast<const uint4*>(D.w + (size_t)(r0 + r) * RB + 16 * u);
    *reinterpret_cast<uint4*>(dst + swz_offset(r, 16 * u, RB, swz)) = v;
  }
  uint32_t* sb = reinterpret_cast<uint32_t*>(dst + 16 * RB);
  for (int i = threadIdx.x; i < nG * 16; i += blockDim.x) {
    const int G = i >> 4, r = i & 15;
    sb[i] = (uint32_t)D.s[(size_t)(r0 + r) * nG + G] |
            ((uint32_t)D.b[(size_t)(r0 + r) * nG + G] << 16);
  }
}

}  // namespace slx
