// Decoder-trunk kernels around the expert path (sm_100a): RMSNorm (with the
// residual add fused), per-head q/k RMSNorm + RoPE + KV-cache append, batch-1
// decode attention (GQA), and greedy argmax.  The trunk is not part of the
// reference (mlx-lm owns it); these exist so decode tok/s can be measured on
// the synthetic decoders, and they read their position from device memory so
// a whole decode step can be captured in a CUDA graph.
#include <cooperative_groups.h>

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
  pdl_launch_dependents();
  uint4 wv[kNormMaxChunks];  // immutable norm weights, in flight before the wait
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    wv[j] = c < H ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0, 0, 0, 0);
  }
  pdl_wait_primary();
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
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&v[j]);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv[j]);
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

// Expert-parallel combine (slx_ep_exchange): wait until every rank has
// counted every CTA of its SwitchGLU launch for this step and layer, then
// delta = bf16(sum_j fma(score_j, row_j) (+ shared row)) -- the same fp32
// operations in the same unit order as the single-GPU fused kernel -- and
// the residual add + RMSNorm of k_add_rmsnorm on it (same arithmetic).
constexpr int kEpMaxK = SLX_FILL_MAX_K;  // routed units per token

__global__ void __launch_bounds__(kNormThreads) k_ep_combine_rmsnorm(
    const slx_ep_exchange ep, const float* scores, int k, int H,
    int has_shared, const uint16_t* h_in, const uint16_t* w, float eps,
    uint16_t* h_out, uint16_t* y, int32_t* status) {
  __shared__ float red[32];
  __shared__ int s_ok;
  __shared__ float s_sc[kEpMaxK];
  pdl_launch_dependents();
  uint4 wv[kNormMaxChunks];  // immutable norm weights, in flight before the wait
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    wv[j] = c < H ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0, 0, 0, 0);
  }
  pdl_wait_primary();
  const int stamp = *ep.stamp;
  if (threadIdx.x < k && threadIdx.x < kEpMaxK) s_sc[threadIdx.x] = scores[threadIdx.x];
  if (threadIdx.x == 0) {
    s_ok = 1;
    if (ep.grid > 0) {
      // counters per (stamp parity, layer): this parity's steps so far,
      // each counted by every CTA of every rank
      const unsigned int want = (unsigned int)((stamp + 1) >> 1) *
                                (unsigned int)(ep.n_ranks * ep.grid);
      const unsigned int* cnt =
          ep.count[ep.rank] + (stamp & 1) * ep.n_layers + ep.layer;
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t i = 0;; ++i) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
                     : "=r"(v) : "l"(cnt) : "memory");
        if ((int)(v - want) >= 0) break;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > (uint64_t)ep.wait_ns) {
          set_status(status, SLX_ERR_DEVICE_TIMEOUT);
          s_ok = 0;
          break;
        }
        if (i > 256) __nanosleep(64);
      }
    }
  }
  __syncthreads();
  const uint16_t* blk =
      reinterpret_cast<const uint16_t*>(ep.recv[ep.rank]) +
      ((size_t)(stamp & 1) * ep.n_layers + ep.layer) * (size_t)(k + 1) * H;
  uint4 v[kNormMaxChunks];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int c = (j * kNormThreads + threadIdx.x) * 8;
    if (c >= H) break;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (s_ok) {
      // every unit's row first (one round trip), then the combine in unit
      // order
      uint4 rows[kEpMaxK];
#pragma unroll
      for (int u = 0; u < kEpMaxK; ++u)
        if (u < k)
          rows[u] = __ldcg(reinterpret_cast<const uint4*>(blk + (size_t)u * H + c));
#pragma unroll
      for (int u = 0; u < kEpMaxK; ++u) {
        if (u >= k) break;
        const float sc = s_sc[u];
        const uint32_t rw[4] = {rows[u].x, rows[u].y, rows[u].z, rows[u].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = fmaf(sc, bf16_lo(rw[q]), acc[2 * q]);
          acc[2 * q + 1] = fmaf(sc, bf16_hi(rw[q]), acc[2 * q + 1]);
        }
      }
      if (has_shared) {
        const uint4 r = __ldcg(reinterpret_cast<const uint4*>(
            blk + (size_t)k * H + c));
        const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = acc[2 * q] + bf16_lo(rw[q]);
          acc[2 * q + 1] = acc[2 * q + 1] + bf16_hi(rw[q]);
        }
      }
    }
    uint4 a = *reinterpret_cast<const uint4*>(h_in + c);
    uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float dlo = round_bf16(acc[2 * q]), dhi = round_bf16(acc[2 * q + 1]);
      const float lo = round_bf16(bf16_lo(pa[q]) + dlo);
      const float hi = round_bf16(bf16_hi(pa[q]) + dhi);
      pa[q] = (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
    }
    *reinterpret_cast<uint4*>(h_out + c) = a;
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
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&v[j]);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv[j]);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint16_t lo = f32_to_bf16(bf16_lo(pa[q]) * inv * bf16_lo(pw[q]));
      const uint16_t hi = f32_to_bf16(bf16_hi(pa[q]) * inv * bf16_hi(pw[q]));
      po[q] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(y + c) = o;
  }
}

int launch_ep_combine_rmsnorm(const slx_ep_exchange& ep, const float* scores,
                              int k, int H, int has_shared,
                              const uint16_t* h_in, const uint16_t* w,
                              float eps, uint16_t* h_out, uint16_t* y,
                              int32_t* status, cudaStream_t s) {
  if (H % 8 || H > 8 * kNormThreads * kNormMaxChunks || k < 1 || k > kEpMaxK)
    return SLX_ERR_UNSUPPORTED;
  return launch_k(k_ep_combine_rmsnorm, dim3(1), dim3(kNormThreads), 0, s, ep,
                  scores, k, H, has_shared, h_in, w, eps, h_out, y, status) ==
                 cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
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
  pdl_launch_dependents();
  pdl_wait_primary();
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

// Split-K decode attention (GQA) on a thread-block cluster.  The 8 CTAs of
// a cluster serve one (token, kv head) and every q head that shares it; CTA
// r takes the 64-position chunks r, r+8, ...: it stages a chunk's K and V
// rows (2 x 16 KB) in shared memory with one round of 16-byte loads, scores
// every (head, position) pair (4 threads per position), and folds the chunk
// into a running softmax (max, sum, unnormalised O) per head.  Each CTA then
// writes its (O, max, sum) into CTA 0's shared memory (distributed shared
// memory); after one cluster barrier CTA 0 merges them and writes out.
constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 64;
constexpr int kAttnMaxRep = 8;
constexpr int kAttnCluster = 8;
constexpr int kAttnPart = 128 + 2;  // O, max, sum
// dynamic shared memory: K, V chunk (bf16) | q (fp32) | p | partials
constexpr int kAttnSmem = 2 * kAttnChunk * 128 * 2 + kAttnMaxRep * 128 * 4 +
                          kAttnMaxRep * kAttnChunk * 4 +
                          kAttnCluster * kAttnMaxRep * kAttnPart * 4;

// One head vector of the token (128 bf16 at v) through the q/k RMSNorm and
// rotate-half RoPE by one warp, with the arithmetic and summation order of
// k_qk_rope_cache (lane l holds pairs l and l + 32 of the 64, each half of
// the sum reduced as one 32-thread block would): rotated values (bf16) at
// dst[i] and dst[i + 64].
// The lane's norm weights (pairs lane and lane + 32: dims i and i + 64) and
// inverse frequencies, fixed inputs loaded before the kernel waits.
struct RopeLane {
  float w[2][2];  // [pair][dim i, dim i + 64]
  float f[2];
};

SLX_DEV RopeLane rope_lane(const uint16_t* nw, const float* inv_freq,
                           int lane) {
  RopeLane r;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    r.w[h][0] = bf16_to_f32(__ldg(nw + i));
    r.w[h][1] = bf16_to_f32(__ldg(nw + i + 64));
    r.f[h] = __ldg(inv_freq + i);
  }
  return r;
}

SLX_DEV void rope_head(const uint16_t* v, const RopeLane& rl, float eps, int p,
                       uint16_t* dst, int lane) {
  float a[2], b[2], s2[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    a[h] = bf16_to_f32(v[i]);
    b[h] = bf16_to_f32(v[i + 64]);
    float x = a[h] * a[h] + b[h] * b[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    s2[h] = x;
  }
  const float inv = rsqrtf((s2[0] + s2[1]) / 128.f + eps);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = lane + 32 * h;
    const float an = round_bf16(a[h] * inv * rl.w[h][0]);
    const float bn = round_bf16(b[h] * inv * rl.w[h][1]);
    const float ang = (float)p * rl.f[h];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    dst[i] = f32_to_bf16(an * cs - bn * sn);
    dst[i + 64] = f32_to_bf16(an * sn + bn * cs);
  }
}

// K and V rows c0 .. c0 + np - 1 of kv head hk into Ks / Vs (64 x 128
// bf16 each; rows from np on, and row `skip`, zero).  All threads call this.
SLX_DEV void stage_chunk(uint16_t* Ks, uint16_t* Vs, const uint16_t* kcache,
                         const uint16_t* vcache, size_t kstride, int hk,
                         int hd, int c0, int np, int skip) {
  for (int u = threadIdx.x; u < kAttnChunk * 16; u += kAttnThreads) {
    const int r = u >> 4, cu = u & 15;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (r < np && c0 + r != skip) {
      const size_t off = (size_t)(c0 + r) * kstride + (size_t)hk * hd;
      kv = reinterpret_cast<const uint4*>(kcache + off)[cu];
      vv = reinterpret_cast<const uint4*>(vcache + off)[cu];
    }
    reinterpret_cast<uint4*>(Ks)[u] = kv;
    reinterpret_cast<uint4*>(Vs)[u] = vv;
  }
}

struct AttnRope {  // ROPE form: the token's q/k norm, RoPE and cache append
  const uint16_t* qn;
  const uint16_t* kn;
  float eps;
  const float* inv_freq;
  uint16_t* kcache;
  uint16_t* vcache;
  int32_t* status;
};

template <bool ROPE>
__global__ void __cluster_dims__(kAttnCluster, 1, 1)
    __launch_bounds__(kAttnThreads) k_attn_decode(
        const uint16_t* qkv, int nq, int nkv, int hd, const uint16_t* kcache,
        const uint16_t* vcache, const int32_t* pos, int max_len, float scale,
        uint16_t* out, const AttnRope R) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) uint8_t attn_smem[];
  uint16_t* Ks = reinterpret_cast<uint16_t*>(attn_smem);
  uint16_t* Vs = Ks + kAttnChunk * 128;
  float* qs = reinterpret_cast<float*>(Vs + kAttnChunk * 128);
  float* ps = qs + kAttnMaxRep * 128;                 // [rep][64]
  float* parts = ps + kAttnMaxRep * kAttnChunk;       // [8][rep][130]
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  pdl_launch_dependents();
  const int hk = blockIdx.y, t = blockIdx.z;
  const int rep = nq / nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t kstride = (size_t)nkv * hd;
  // ROPE: the position and the cache rows before the token's own (n - 1)
  // are inputs of earlier steps, not of the preceding kernel, so this CTA's
  // first chunk is staged before the wait (the token's row is filled in
  // after it), as are the fixed norm weights and frequencies
  int n = ROPE ? pos[t] + 1 : 0;
  bool ok_n = n > 0 && n <= max_len;
  int nchunks = ok_n ? (n + kAttnChunk - 1) / kAttnChunk : 0;
  RopeLane rq, rk;
  const bool early = ROPE && rank < nchunks;
  if constexpr (ROPE) {
    rq = rope_lane(R.qn, R.inv_freq, lane);
    rk = rope_lane(R.kn, R.inv_freq, lane);
    if (early) stage_chunk(Ks, Vs, kcache, vcache, kstride, hk, hd,
                           rank * kAttnChunk, min(kAttnChunk, n - rank * kAttnChunk),
                           n - 1);
  }
  pdl_wait_primary();
  if constexpr (!ROPE) {
    n = pos[t] + 1;
    ok_n = n > 0 && n <= max_len;
    nchunks = ok_n ? (n + kAttnChunk - 1) / kAttnChunk : 0;
  }
  const uint16_t* q = qkv + (size_t)t * (nq + 2 * nkv) * hd +
                      (size_t)hk * rep * hd;
  // ROPE: the token's own key and value row (position n - 1), computed here
  // and substituted when its chunk is staged; cluster rank 0 appends them
  // to the cache for the later steps
  __shared__ __align__(16) uint16_t knew[128], vnew[128];
  __shared__ __align__(16) uint16_t qrot[kAttnMaxRep * 128];
  if constexpr (ROPE) {
    const uint16_t* base = qkv + (size_t)t * (nq + 2 * nkv) * hd;
    if (!ok_n) {
      if (threadIdx.x == 0 && rank == 0) set_status(R.status, SLX_ERR_OUT_OF_RANGE);
    } else {
      for (int h = warp; h <= rep; h += kAttnThreads / 32) {
        if (h < rep)
          rope_head(q + (size_t)h * hd, rq, R.eps, n - 1, qrot + h * 128,
                    lane);
        else
          rope_head(base + (size_t)(nq + hk) * hd, rk, R.eps, n - 1, knew,
                    lane);
      }
      if (threadIdx.x < 128) vnew[threadIdx.x] = base[(size_t)(nq + nkv + hk) * hd + threadIdx.x];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rep * 128; i += kAttnThreads)
      qs[i] = bf16_to_f32(qrot[i]);
    if (rank == 0 && ok_n && threadIdx.x < 32) {
      const size_t off = (size_t)(n - 1) * kstride + (size_t)hk * hd;
      if (threadIdx.x < 16)
        reinterpret_cast<uint4*>(R.kcache + off)[threadIdx.x] =
            reinterpret_cast<const uint4*>(knew)[threadIdx.x];
      else
        reinterpret_cast<uint4*>(R.vcache + off)[threadIdx.x - 16] =
            reinterpret_cast<const uint4*>(vnew)[threadIdx.x - 16];
    }
  } else {
    for (int i = threadIdx.x; i < rep * 128; i += kAttnThreads)
      qs[i] = bf16_to_f32(q[i]);
  }
  // running state: warp r < rep owns head r's (m, l); thread (d2, rg) owns
  // O of heads rg*2, rg*2+1 at dims 2*d2, 2*d2+1
  float m_run = -INFINITY, l_run = 0.f;
  const int d2 = threadIdx.x & 63, rg = threadIdx.x >> 6;
  float oa0 = 0.f, oa1 = 0.f, ob0 = 0.f, ob1 = 0.f;
  for (int c = rank; c < nchunks; c += kAttnCluster) {
    const int c0 = c * kAttnChunk;
    const int np = min(kAttnChunk, n - c0);
    __syncthreads();  // previous chunk's K/V/p reads are done
    if (!(early && c == rank))
      stage_chunk(Ks, Vs, kcache, vcache, kstride, hk, hd, c0, np,
                  ROPE ? n - 1 : -1);
    if (ROPE && c0 <= n - 1 && n - 1 < c0 + np && threadIdx.x < 16) {
      const int r = n - 1 - c0;  // the token's own row
      reinterpret_cast<uint4*>(Ks + r * 128)[threadIdx.x] =
          reinterpret_cast<const uint4*>(knew)[threadIdx.x];
      reinterpret_cast<uint4*>(Vs + r * 128)[threadIdx.x] =
          reinterpret_cast<const uint4*>(vnew)[threadIdx.x];
    }
    __syncthreads();
    {  // scores: thread = (position, quarter of the 128 dims)
      const int p = threadIdx.x >> 2, qt = threadIdx.x & 3;
      uint4 kr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        kr[u] = reinterpret_cast<const uint4*>(Ks + p * 128 + qt * 32)[u];
      for (int r = 0; r < rep; ++r) {
        const float* qr = qs + r * 128 + qt * 32;
        float sacc = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 qa = *reinterpret_cast<const float4*>(qr + u * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qr + u * 8 + 4);
          sacc += qa.x * bf16_lo(kr[u].x) + qa.y * bf16_hi(kr[u].x) +
                  qa.z * bf16_lo(kr[u].y) + qa.w * bf16_hi(kr[u].y) +
                  qb.x * bf16_lo(kr[u].z) + qb.y * bf16_hi(kr[u].z) +
                  qb.z * bf16_lo(kr[u].w) + qb.w * bf16_hi(kr[u].w);
        }
        sacc += __shfl_xor_sync(0xffffffffu, sacc, 1);
        sacc += __shfl_xor_sync(0xffffffffu, sacc, 2);
        if (qt == 0) ps[r * kAttnChunk + p] = p < np ? sacc * scale : -INFINITY;
      }
    }
    __syncthreads();
    __shared__ float s_scale[kAttnMaxRep];
    if (warp < rep) {  // chunk softmax folded into head warp's running state
      const float a0 = ps[warp * kAttnChunk + lane];
      const float a1 = ps[warp * kAttnChunk + lane + 32];
      float m = fmaxf(a0, a1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float m_new = fmaxf(m_run, m);
      const float e0 = lane < np ? expf(a0 - m_new) : 0.f;
      const float e1 = lane + 32 < np ? expf(a1 - m_new) : 0.f;
      ps[warp * kAttnChunk + lane] = e0;
      ps[warp * kAttnChunk + lane + 32] = e1;
      float l = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      const float f = expf(m_run - m_new);  // 0 on the first chunk
      l_run = l_run * f + l;
      m_run = m_new;
      if (lane == 0) s_scale[warp] = f;
    }
    __syncthreads();
    {  // O = O * f + P.V for this thread's heads and dims
      const int r = rg * 2;
      if (r < rep) {
        const bool two = r + 1 < rep;
        const float fa = s_scale[r], fb = two ? s_scale[r + 1] : 0.f;
        oa0 *= fa; oa1 *= fa; ob0 *= fb; ob1 *= fb;
        for (int p = 0; p < np; ++p) {
          const uint32_t v = reinterpret_cast<const uint32_t*>(Vs + p * 128)[d2];
          const float vl = bf16_lo(v), vh = bf16_hi(v);
          const float w0 = ps[r * kAttnChunk + p];
          oa0 += w0 * vl;
          oa1 += w0 * vh;
          if (two) {
            const float w1 = ps[(r + 1) * kAttnChunk + p];
            ob0 += w1 * vl;
            ob1 += w1 * vh;
          }
        }
      }
    }
  }
  // partials into CTA 0's shared memory
  float* lp = cluster.map_shared_rank(parts, 0) +
              (size_t)rank * kAttnMaxRep * kAttnPart;
  {
    const int r = rg * 2;
    if (r < rep) {
      lp[r * kAttnPart + 2 * d2] = oa0;
      lp[r * kAttnPart + 2 * d2 + 1] = oa1;
      if (r + 1 < rep) {
        lp[(r + 1) * kAttnPart + 2 * d2] = ob0;
        lp[(r + 1) * kAttnPart + 2 * d2 + 1] = ob1;
      }
    }
  }
  if (warp < rep && lane == 0) {
    lp[warp * kAttnPart + 128] = m_run;
    lp[warp * kAttnPart + 129] = l_run;
  }
  cluster.sync();
  if (rank != 0 || !ok_n) return;
  const int nv = min(nchunks, kAttnCluster);  // CTAs that saw positions
  for (int r = warp; r < rep; r += kAttnThreads / 32) {
    float M = -INFINITY;
    for (int cc = 0; cc < nv; ++cc)
      M = fmaxf(M, parts[(cc * kAttnMaxRep + r) * kAttnPart + 128]);
    float Lsum = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int cc = 0; cc < nv; ++cc) {
      const float* pp = parts + (size_t)(cc * kAttnMaxRep + r) * kAttnPart;
      const float f = expf(pp[128] - M);
      Lsum += f * pp[129];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] += f * pp[lane * 4 + j];
    }
    uint16_t* dst = out + ((size_t)t * nq + hk * rep + r) * hd + lane * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = f32_to_bf16(o[j] / Lsum);
  }
}

// greedy argmax over bf16 logits, ties -> lowest index.  One CTA per token;
// 16-byte loads, four in flight per thread, then a (value, index) reduction.
SLX_DEV void argmax_take(float v, int i, float& best, int& bi) {
  if (v > best || (v == best && i < bi)) {
    best = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(1024) k_argmax(const uint16_t* logits,
                                                  int V, int32_t* out) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  pdl_launch_dependents();
  pdl_wait_primary();
  const int t = blockIdx.x;
  const uint16_t* l = logits + (size_t)t * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = (V % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(l) & 15u) == 0);
  if (vec) {
    const uint4* l4 = reinterpret_cast<const uint4*>(l);
    const int n4 = V / 8;
    for (int b = threadIdx.x; b < n4; b += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = b + u * blockDim.x;
        v[u] = q < n4 ? __ldcs(l4 + q) : make_uint4(0xff80ff80u, 0xff80ff80u,
                                                   0xff80ff80u, 0xff80ff80u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = b + u * blockDim.x;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          argmax_take(bf16_lo(w[j]), q * 8 + 2 * j, best, bi);
          argmax_take(bf16_hi(w[j]), q * 8 + 2 * j + 1, best, bi);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x)
      argmax_take(bf16_to_f32(l[i]), i, best, bi);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_take(ov, oi, best, bi);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    rv[warp] = best;
    ri[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      argmax_take(rv[w], ri[w], best, bi);
    out[t] = bi < V ? bi : 0;
  }
}

int launch_add_rmsnorm(const uint16_t* h_in, const uint16_t* d,
                       const uint16_t* w, int T, int H, float eps,
                       uint16_t* h_out, uint16_t* y, cudaStream_t s) {
  if (H % 8 || H > 8 * kNormThreads * kNormMaxChunks) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  return launch_k(k_add_rmsnorm, dim3(T), dim3(kNormThreads), 0, s, h_in, d, w,
                  H, eps, h_out, y) == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_qk_rope_cache(uint16_t* qkv, int T, int nq, int nkv, int hd,
                         const uint16_t* qn, const uint16_t* kn, float eps,
                         const float* inv_freq, const int32_t* pos,
                         int max_len, uint16_t* kc, uint16_t* vc,
                         int32_t* status, cudaStream_t s) {
  if (hd != 128) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  dim3 grid(T, nq + 2 * nkv);
  const cudaError_t e = launch_k(k_qk_rope_cache, grid, dim3(hd / 2), 0, s,
                                 qkv, nq, nkv, hd, qn, kn, eps, inv_freq, pos,
                                 max_len, kc, vc, status);
  if (e != cudaSuccess) return SLX_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_attn_decode(const uint16_t* qkv, int T, int nq, int nkv, int hd,
                       const uint16_t* kc, const uint16_t* vc,
                       const int32_t* pos, int max_len, uint16_t* out,
                       cudaStream_t s) {
  if (hd != 128 || nq % nkv || nq / nkv > kAttnMaxRep) return SLX_ERR_UNSUPPORTED;
  if (T <= 0) return SLX_OK;
  if (T > 65535 || nkv > 65535) return SLX_ERR_INVALID;
  static PerDevice configured;
  std::atomic<int>& slot = configured.here();
  if (!slot.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(k_attn_decode<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kAttnSmem) != cudaSuccess)
      return SLX_ERR_CUDA;
    slot.store(1, std::memory_order_relaxed);
  }
  dim3 grid(kAttnCluster, nkv, T);
  const AttnRope R = {};
  const cudaError_t e = launch_k(k_attn_decode<false>, grid, dim3(kAttnThreads),
                                 (size_t)kAttnSmem, s, qkv, nq, nkv, hd, kc, vc,
                                 pos, max_len, 1.0f / sqrtf((float)hd), out, R);
  return e == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_attn_rope_decode(const uint16_t* qkv, int nq, int nkv, int hd,
                            const uint16_t* qn, const uint16_t* kn, float eps,
                            const float* inv_freq, const int32_t* pos,
                            int max_len, uint16_t* kc, uint16_t* vc,
                            uint16_t* out, int32_t* status, cudaStream_t s) {
  if (hd != 128 || nq % nkv || nq / nkv > kAttnMaxRep) return SLX_ERR_UNSUPPORTED;
  if (nkv > 65535) return SLX_ERR_INVALID;
  static PerDevice configured;
  std::atomic<int>& slot = configured.here();
  if (!slot.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(k_attn_decode<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kAttnSmem) != cudaSuccess)
      return SLX_ERR_CUDA;
    slot.store(1, std::memory_order_relaxed);
  }
  dim3 grid(kAttnCluster, nkv, 1);
  const AttnRope R = {qn, kn, eps, inv_freq, kc, vc, status};
  const cudaError_t e = launch_k(k_attn_decode<true>, grid, dim3(kAttnThreads),
                                 (size_t)kAttnSmem, s, qkv, nq, nkv, hd,
                                 (const uint16_t*)kc, (const uint16_t*)vc, pos,
                                 max_len, 1.0f / sqrtf((float)hd), out, R);
  return e == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_argmax(const uint16_t* logits, int T, int V, int32_t* out,
                  cudaStream_t s) {
  if (T <= 0) return SLX_OK;
  return launch_k(k_argmax, dim3(T), dim3(1024), 0, s, logits, V, out) ==
                 cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace slx
