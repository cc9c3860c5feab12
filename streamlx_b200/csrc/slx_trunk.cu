// Decoder-trunk kernels around the expert path (sm_100a): RMSNorm (with the
// residual add fused), per-head q/k RMSNorm + RoPE + KV-cache append, batch-1
// decode attention (GQA), and greedy argmax.  The trunk is not part of the
// reference (mlx-lm owns it); these exist so decode tok/s can be measured on
// the synthetic decoders, and they read their position from device memory so
// a whole decode step can be captured in a CUDA graph.
#include "slx_kernels.cuh"

namespace slx {

template <typename T, typename Op>
SLX_DEV T breduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T r = red[0];
  for (int i = 1; i < nw; ++i) r = op(r, red[i]);
  return r;
}

// h_out = bf16(h_in + d) (if d, else h_in), y = bf16(h_out * rsqrt(mean(
// h_out^2) + eps) * w).  One CTA per token, 8 bf16 per thread per chunk (one
// 16-byte load each), the row kept in registers between the two passes.
// h_out may alias h_in.
constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;   // H <= 8 * 256 * 4

__global__ void __launch_bounds__(kNormThreads) k_add_rmsnorm(
    const uint16_t* h_in, const uint16_t* d, const uint16_t* w, int H,
    float eps, uint16_t* h_out, uint16_t* y) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const uint16_t* hr = h_in + (size_t)t * H;
  const uint16_t* dr = d ? d + (size_t)t * H : nullptr;
  uint4 v[kNormMaxChunks];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c >= H) break;
    uint4 a = *reinterpret_cast<const uint4*>(hr + c);
    if (dr) {
      const uint4 b = *reinterpret_cast<const uint4*>(dr + c);
      uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = round_bf16(bf16_lo(pa[q]) + bf16_lo(pb[q]));
        const float hi = round_bf16(bf16_hi(pa[q]) + bf16_hi(pb[q]));
        pa[q] = (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
      }
    }
    if (dr || h_out != h_in)
      *reinterpret_cast<uint4*>(h_out + (size_t)t * H + c) = a;
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = bf16_lo(pa[q]), hi = bf16_hi(pa[q]);
      ss += lo * lo + hi * hi;
    }
    v[j] = a;
  }
  ss = breduce(ss, red, [](float a, float b) { return a + b; });
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c >= H) break;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&v[j]);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint16_t lo = f32_to_bf16(bf16_lo(pa[q]) * inv * bf16_lo(pw[q]));
      const uint16_t hi = f32_to_bf16(bf16_hi(pa[q]) * inv * bf16_hi(pw[q]));
      po[q] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(y + (size_t)t * H + c) = o;
  }
}

// qkv row layout: [nq*hd | nkv*hd | nkv*hd].  Per head: RMSNorm over hd with
// q_norm / k_norm, then rotate-half RoPE at pos[t]; q written back in place,
// k and v appended to the caches at row pos[t].
__global__ void k_qk_rope_cache(uint16_t* qkv, int nq, int nkv, int hd,
                                const uint16_t* qn, const uint16_t* kn,
                                float eps, const float* inv_freq,
                                const int32_t* pos, int max_len,
                                uint16_t* kcache, uint16_t* vcache,
                                int32_t* status) {
  __shared__ float red[32];
  const int t = blockIdx.x, hidx = blockIdx.y;
  const int half = hd / 2, i = threadIdx.x;  // blockDim.x == half
  const int p = pos[t];
  if (p < 0 || p >= max_len) {
    if (i == 0) set_status(status, SLX_ERR_OUT_OF_RANGE);
    return;
  }
  const int row = (nq + 2 * nkv) * hd;
  uint16_t* base = qkv + (size_t)t * row;
  if (hidx >= nq + nkv) {  // v head: copy into cache
    const int vh = hidx - nq - nkv;
    const uint16_t* src = base + (nq + nkv) * hd + vh * hd;
    uint16_t* dst = vcache + ((size_t)p * nkv + vh) * hd;
    dst[i] = src[i];
    dst[i + half] = src[i + half];
    return;
  }
  const bool isq = hidx < nq;
  uint16_t* v = base + hidx * hd;
  const uint16_t* nw = isq ? qn : kn;
  float a = bf16_to_f32(v[i]), b = bf16_to_f32(v[i + half]);
  float ss = breduce(a * a + b * b, red, [](float x, float y) { return x + y; });
  const float inv = rsqrtf(ss / (float)hd + eps);
  a = round_bf16(a * inv * bf16_to_f32(nw[i]));
  b = round_bf16(b * inv * bf16_to_f32(nw[i + half]));
  const float ang = (float)p * inv_freq[i];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const uint16_t ra = f32_to_bf16(a * cs - b * sn);
  const uint16_t rb = f32_to_bf16(a * sn + b * cs);
  if (isq) {
    v[i] = ra;
    v[i + half] = rb;
  } else {
    uint16_t* dst = kcache + ((size_t)p * nkv + (hidx - nq)) * hd;
    dst[i] = ra;
    dst[i + half] = rb;
  }
}

// One CTA per (token, q head).  Scores over positions 0..pos[t], softmax in
// fp32, output bf16.  Dynamic smem: max_len floats.
__global__ void __launch_bounds__(128) k_attn_decode(
    const uint16_t* qkv, int nq, int nkv, int hd, const uint16_t* kcache,
    const uint16_t* vcache, const int32_t* pos, int max_len, float scale,
    uint16_t* out) {
  extern __shared__ float sc[];
  __shared__ float red[32];
  const int t = blockIdx.x, hq = blockIdx.y;
  const int hk = hq / (nq / nkv);
  const int n = pos[t] + 1;
  if (n <= 0 || n > max_len) return;
  const uint16_t* q = qkv + (size_t)t * (nq + 2 * nkv) * hd + hq * hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  // each lane owns hd/32 dims (hd = 128 -> 4)
  float qv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] = bf16_to_f32(q[lane * 4 + j]);
  for (int p = warp; p < n; p += nw) {
    const uint16_t* kr = kcache + ((size_t)p * nkv + hk) * hd + lane * 4;
    const uint2 kw = *reinterpret_cast<const uint2*>(kr);
    float s = qv[0] * bf16_lo(kw.x) + qv[1] * bf16_hi(kw.x) +
              qv[2] * bf16_lo(kw.y) + qv[3] * bf16_hi(kw.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sc[p] = s * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int p = threadIdx.x; p < n; p += blockDim.x) mx = fmaxf(mx, sc[p]);
  mx = breduce(mx, red, [](float a, float b) { return fmaxf(a, b); });
  float se = 0.f;
  for (int p = threadIdx.x; p < n; p += blockDim.x) {
    const float e = expf(sc[p] - mx);
    sc[p] = e;
    se += e;
  }
  se = breduce(se, red, [](float a, float b) { return a + b; });
  __syncthreads();
  const int d = threadIdx.x;  // blockDim.x == hd
  float acc = 0.f;
  for (int p = 0; p < n; ++p)
    acc += sc[p] * bf16_to_f32(vcache[((size_t)p * nkv + hk) * hd + d]);
  out[((size_t)t * nq + hq) * hd + d] = f32_to_bf16(acc / se);
}

// greedy argmax over bf16 logits, ties -> lowest index
__global__ void __launch_bounds__(1024) k_argmax(const uint16_t* logits,
                                                  int V, int32_t* out) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  const int t = blockIdx.x;
  const uint16_t* l = logits + (size_t)t * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = bf16_to_f32(l[i]);
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { rv[warp] = best; ri[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (rv[w] > best || (rv[w] == best && ri[w] < bi)) { best = rv[w]; bi = ri[w]; }
    out[t] = bi;
  }
}

int launch_add_rmsnorm(const uint16_t* h_in, const uint16_t* d,
                       const uint16_t* w, int T, int H, float eps,
                       uint16_t* h_out, uint16_t* y, cudaStream_t s) {
  if (H % 8 || H > 8 * kNormThreads * kNormMaxChunks) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  k_add_rmsnorm<<<T, kNormThreads, 0, s>>>(h_in, d, w, H, eps, h_out, y);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_qk_rope_cache(uint16_t* qkv, int T, int nq, int nkv, int hd,
                         const uint16_t* qn, const uint16_t* kn, float eps,
                         const float* inv_freq, const int32_t* pos,
                         int max_len, uint16_t* kc, uint16_t* vc,
                         int32_t* status, cudaStream_t s) {
  if (hd != 128) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  dim3 grid(T, nq + 2 * nkv);
  k_qk_rope_cache<<<grid, hd / 2, 0, s>>>(qkv, nq, nkv, hd, qn, kn, eps,
                                          inv_freq, pos, max_len, kc, vc,
                                          status);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_attn_decode(const uint16_t* qkv, int T, int nq, int nkv, int hd,
                       const uint16_t* kc, const uint16_t* vc,
                       const int32_t* pos, int max_len, uint16_t* out,
                       cudaStream_t s) {
  if (hd != 128 || nq % nkv) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  const int smem = max_len * 4;
  if (smem > 200 * 1024) return SLX_ERR_UNSUPPORTED;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(k_attn_decode,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(T, nq);
  k_attn_decode<<<grid, hd, smem, s>>>(qkv, nq, nkv, hd, kc, vc, pos, max_len,
                                       1.0f / sqrtf((float)hd), out);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_argmax(const uint16_t* logits, int T, int V, int32_t* out,
                  cudaStream_t s) {
  if (T <= 0) return SLX_OK;
  k_argmax<<<T, 1024, 0, s>>>(logits, V, out);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace slx
