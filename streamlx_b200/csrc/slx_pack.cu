// Repack MLX-affine quantized weights (as stored in the safetensors shards,
// streamlx/stindex.py:22-39 row ranges) into the tile format of
// slx_tiles.cuh.  Runs when a pool slot is filled, after the raw expert
// bytes have been copied host -> device; one extra HBM pass per expert.
#include "slx_kernels.cuh"
#include "slx_tiles.cuh"

namespace slx {

struct QSrc {
  const uint8_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

constexpr int kPackMax = 32;
struct PackArgs {
  QSrc gate[kPackMax], up[kPackMax], down[kPackMax];
  uint8_t* dst[kPackMax];
  int n, H, I, bits;
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

__global__ void __launch_bounds__(256) k_pack_experts(const __grid_constant__ PackArgs a) {
  const int e = blockIdx.y, t = blockIdx.x;
  const int na = a.I / 16;
  uint8_t* base = a.dst[e];
  if (t < na) {
    pack_pair(base + (size_t)t * pair_tile_bytes(a.H, a.bits), a.gate[e],
              16 * t, a.up[e], 16 * t, a.I, a.H, a.bits);
  } else {
    const int rb = t - na;
    pack_single(base + expert_a_bytes(a.H, a.I, a.bits) +
                    (size_t)rb * single_tile_bytes(a.I, a.bits),
                a.down[e], 16 * rb, a.I, a.bits);
  }
}

__global__ void __launch_bounds__(256) k_pack_dense(QSrc W, int out, int in, int bits,
                                                    uint8_t* dst) {
  const int t = blockIdx.x;
  pack_pair(dst + (size_t)t * pair_tile_bytes(in, bits), W, 32 * t, W,
            32 * t + 16, out, in, bits);
}

int launch_pack_experts(const void* const* gw, const void* const* gs,
                        const void* const* gb, const void* const* uw,
                        const void* const* us, const void* const* ub,
                        const void* const* dw, const void* const* ds,
                        const void* const* db, void* const* dst, int n, int H,
                        int I, int bits, cudaStream_t stream) {
  for (int e0 = 0; e0 < n; e0 += kPackMax) {
    PackArgs a = {};
    a.n = n - e0 < kPackMax ? n - e0 : kPackMax;
    a.H = H;
    a.I = I;
    a.bits = bits;
    for (int i = 0; i < a.n; ++i) {
      const int e = e0 + i;
      a.gate[i] = {(const uint8_t*)gw[e], (const uint16_t*)gs[e], (const uint16_t*)gb[e]};
      a.up[i] = {(const uint8_t*)uw[e], (const uint16_t*)us[e], (const uint16_t*)ub[e]};
      a.down[i] = {(const uint8_t*)dw[e], (const uint16_t*)ds[e], (const uint16_t*)db[e]};
      a.dst[i] = (uint8_t*)dst[e];
    }
    dim3 grid(I / 16 + H / 16, a.n);
    k_pack_experts<<<grid, 256, 0, stream>>>(a);
    if (cudaGetLastError() != cudaSuccess) return SLX_ERR_CUDA;
  }
  return SLX_OK;
}

int launch_pack_dense(const void* w, const void* s, const void* b, int out,
                      int in, int bits, void* dst, cudaStream_t stream) {
  QSrc W = {(const uint8_t*)w, (const uint16_t*)s, (const uint16_t*)b};
  k_pack_dense<<<(out + 31) / 32, 256, 0, stream>>>(W, out, in, bits,
                                                    (uint8_t*)dst);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace slx
