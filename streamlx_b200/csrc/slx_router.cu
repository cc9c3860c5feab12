// Router GEMV + softmax + top-k (K1) for sm_100a.
//
// Replaces the mlx-lm MoE block's router that the reference wraps
// (streamlx/integrate.py:5-7) and the next-layer predictor it builds from the
// same gate (streamlx/integrate.py:60-88: x * (w_next / w_this) -> gate ->
// argpartition -> take_along_axis).
//
// Determinism contract (what makes routing bit-exact against the CPU
// oracle): each logit is the fp64 sum of exact bf16*bf16 products, rounded
// once to fp32, plus an fp32 bias.  While that fp64 sum is exact (true for
// activation/weight ranges spanning < 2^37) the result does not depend on
// summation order.  Top-k is ranked on the logits (softmax is monotonic):
// descending, ties to the lower expert id.  Scores are the softmax
// probabilities of the selected experts, optionally renormalised.
//
// Layout: grid (ceil(E/8), T); warp w of CTA c computes expert 8c+w.  The
// last CTA to finish a token (ticket counter in caller scratch, reset by
// that CTA) ranks the token's logits.  No CTA ever waits on another.
#include "slx_kernels.cuh"

namespace slx {

constexpr int kRouterWarps = 8;
constexpr int kMaxExperts = 1024;

SLX_DEV double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, typename Op>
SLX_DEV T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T r = red[0];
  for (int i = 1; i < nw; ++i) r = op(r, red[i]);
  return r;
}

__global__ void __launch_bounds__(256) k_router(const RouterArgs a) {
  __shared__ float s_logit[kMaxExperts];
  __shared__ float s_red[32];
  __shared__ int s_last;
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouterWarps + warp;
  const uint16_t* xr = a.x + (size_t)t * a.H;
  if (e < a.E) {
    const uint16_t* wr = a.w + (size_t)e * a.H;
    double acc = 0.0;
    for (int c = lane * 8; c < a.H; c += 256) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
      uint4 rv = make_uint4(0, 0, 0, 0);
      if (a.ratio) rv = *reinterpret_cast<const uint4*>(a.ratio + c);
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
      const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t rs[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x0 = bf16_lo(xs[i]), x1 = bf16_hi(xs[i]);
        if (a.ratio) {
          x0 = round_bf16(x0 * bf16_lo(rs[i]));
          x1 = round_bf16(x1 * bf16_hi(rs[i]));
        }
        acc = fma((double)x0, (double)bf16_lo(ws[i]), acc);
        acc = fma((double)x1, (double)bf16_hi(ws[i]), acc);
      }
    }
    acc = warp_sum_f64(acc);
    if (lane == 0) {
      float lg = (float)acc;
      if (a.bias) lg = lg + a.bias[e];
      a.logits[(size_t)t * a.E + e] = lg;
    }
  }
  // last-arriving CTA of this token ranks it
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&a.tickets[t], 1);
    s_last = ticket == (int)gridDim.x - 1;
    if (s_last) a.tickets[t] = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < a.E; i += blockDim.x)
    s_logit[i] = __ldcg(a.logits + (size_t)t * a.E + i);
  __syncthreads();
  // softmax statistics (deterministic block reductions)
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < a.E; i += blockDim.x) mx = fmaxf(mx, s_logit[i]);
  mx = block_reduce(mx, s_red, [](float u, float v) { return fmaxf(u, v); });
  float se = 0.f;
  for (int i = threadIdx.x; i < a.E; i += blockDim.x) se += expf(s_logit[i] - mx);
  se = block_reduce(se, s_red, [](float u, float v) { return u + v; });
  const bool forced = a.force && a.force[t];
  __shared__ int s_ids[64];
  if (!forced) {
    for (int i = threadIdx.x; i < a.E; i += blockDim.x) {
      const float li = s_logit[i];
      int rank = 0;
      for (int j = 0; j < a.E; ++j) {
        const float lj = s_logit[j];
        rank += (lj > li) || (lj == li && j < i);
      }
      if (rank < a.k) s_ids[rank] = i;
    }
  } else if (threadIdx.x < a.k) {
    int id = a.forced_ids[(size_t)t * a.k + threadIdx.x];
    if (id < 0 || id >= a.E) {
      set_status(a.status, SLX_ERR_OUT_OF_RANGE);
      id = 0;
    }
    s_ids[threadIdx.x] = id;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sel[64];
    float ssum = 0.f;
    for (int j = 0; j < a.k; ++j) {
      sel[j] = expf(s_logit[s_ids[j]] - mx) / se;
      ssum += sel[j];
    }
    for (int j = 0; j < a.k; ++j) {
      a.out_ids[(size_t)t * a.k + j] = s_ids[j];
      a.out_scores[(size_t)t * a.k + j] = a.norm_topk ? sel[j] / ssum : sel[j];
    }
  }
}

int launch_router(const RouterArgs& a, cudaStream_t stream) {
  if (a.E > kMaxExperts || a.k > 64 || a.k < 1 || a.k > a.E || a.H % 8)
    return SLX_ERR_UNSUPPORTED;
  if (a.T <= 0) return SLX_OK;
  if (a.T > 65535) return SLX_ERR_INVALID;
  dim3 grid((a.E + kRouterWarps - 1) / kRouterWarps, a.T);
  k_router<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace slx
