// Repack MLX-affine quantized weights (as stored in the safetensors shards,
// streamlx/stindex.py:22-39 row ranges) into the tile format of
// slx_tiles.cuh.  Runs when a pool slot is filled, after the raw expert
// bytes have been copied host -> device; one extra HBM pass per expert.
#include "slx_kernels.cuh"
#include "slx_tiles.cuh"
#include "slx_pack.cuh"

namespace slx {

constexpr int kPackMax = 32;
struct PackArgs {
  QSrc gate[kPackMax], up[kPackMax], down[kPackMax];
  uint8_t* dst[kPackMax];
  int n, H, I, bits;
};

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
