// Router GEMV + softmax + top-k (K1) for sm_100a.
//
// Replaces the mlx-lm MoE block's router that the reference wraps
// (streamlx/integrate.py:5-7) and the next-layer predictor it builds from the
// same gate (streamlx/integrate.py:60-88: x * (w_next / w_this) -> gate ->
// argpartition -> take_along_axis).  One launch serves up to two "heads"
// over the same activations (the layer's router, its next-layer predictor).
//
// Determinism contract (what makes routing bit-exact against the CPU
// oracle): the reference logit is the fp64 sum of exact bf16*bf16 products,
// rounded once to fp32, plus an fp32 bias; while that fp64 sum is exact it
// does not depend on summation order.  Top-k is ranked on the logits
// (softmax is monotonic): descending, ties to the lower expert id.  Scores
// are the softmax probabilities of the selected experts, optionally
// renormalised.
//
// How: the dots run in fp32 (the fp64 issue rate is far too low to do E x H
// of them on a few SMs), each with a rigorous bound on its distance to the
// reference logit (from the sum of |products|, the summation depth and the
// fp32 roundings of both paths).  The ranking is certified when every
// adjacent pair of the top k, and the k-th against every other expert, are
// further apart than their bounds; otherwise the rows that could still
// matter are recomputed exactly in fp64 and ranked again.  Scores use the
// fp32 logits.
//
// Layout: one thread-block cluster of 8 CTAs per (head, token); CTA r of
// the cluster computes experts [r*E/8, (r+1)*E/8), two rows per warp in
// flight, and stores each logit and its bound straight into CTA 0's shared
// memory (distributed shared memory), so the hand-off to the ranking is one
// cluster barrier instead of global-memory round trips.  In CTA 0 one warp
// ranks by k rounds of a warp-wide (max key, min id); the logits are also
// left in the caller's scratch.
#include <cooperative_groups.h>

#include "slx_kernels.cuh"

#ifdef SLX_TRACE
static __device__ unsigned long long g_slx_trace[3][160][16];
#endif

namespace slx {

constexpr int kRouterCluster = 8;  // CTAs per (head, token)
constexpr int kRouterWarps = 16;
constexpr int kRouterThreads = kRouterWarps * 32;
constexpr int kMaxExperts = 1024;
constexpr int kRouterMaxK = 64;
constexpr int kRouterMaxH = 4096;
constexpr int kRouterBatch = 8;  // 16-byte chunks per row in flight per lane
constexpr int kLaneKeys = 8;     // ranking keys held in registers per lane

struct RouterLaunch {
  RouterArgs h[2];
  int n_heads;
};

SLX_DEV double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

SLX_DEV float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// order-preserving map of a float onto uint32 (larger float -> larger key);
// 0 is below every number and marks "no key"
SLX_DEV uint32_t ordered_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// s[j] += x[j] * w[j], a[j] += |x[j] * w[j]| for 8 consecutive columns
// (eight independent chains per row; every product is exact in fp32)
SLX_DEV void dot8(const float* xs, const uint4& wv, float (&s)[8],
                  float (&a)[8]) {
  const float4 xa = *reinterpret_cast<const float4*>(xs);
  const float4 xb = *reinterpret_cast<const float4*>(xs + 4);
  const float x[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
  const float w[8] = {bf16_lo(wv.x), bf16_hi(wv.x), bf16_lo(wv.y),
                      bf16_hi(wv.y), bf16_lo(wv.z), bf16_hi(wv.z),
                      bf16_lo(wv.w), bf16_hi(wv.w)};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    s[j] = fmaf(x[j], w[j], s[j]);
    a[j] = fmaf(fabsf(x[j]), fabsf(w[j]), a[j]);
  }
}

SLX_DEV float sum8(const float (&v)[8]) {
  return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

// Bound on |fp32 logit - reference logit|.  A sum of exact products added
// along at most `depth` roundings is within depth * 2^-24 / (1 - depth *
// 2^-24) of the exact sum relative to sum(|p|), which the computed |p| sum
// `a` underestimates by at most that factor; both paths round once more to
// fp32 before and once when adding the bias (2^-24 relative each); the
// absolute term covers fp32 underflow.  Every factor carries a margin.
SLX_DEV float logit_bound(float s, float a, float logit, int depth) {
  const float g = (float)(depth + 4) * 5.9604645e-08f * 1.0625f;
  return g * a * 1.0625f + 2.3841858e-07f * (fabsf(s) + fabsf(logit)) +
         1e-30f;
}

// Ranking and outputs of one (head, token) from the logits and bounds in
// shared memory (s_x: the token's staged activations, for the exact
// recompute).  Every thread of the CTA calls this.
__device__ __noinline__ void rank_and_write(const RouterArgs& a, int t,
                                            const float* s_x, float* s_logit,
                                            float* s_bound, uint8_t* s_gone,
                                            int* s_cand, int& s_ncand,
                                            int& s_cert) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, H = a.H, k = a.k;
  const bool forced = a.force && a.force[t];
  int id1 = -1, id2 = -1;  // rank `lane` and rank `lane + 32`
  // k rounds of a warp-wide (max key, min id) over the experts (only the
  // exactly known ones when exact_only); lane l holds ids l, l+32, ... (up
  // to kLaneKeys in registers, the rest re-read).  Returns the largest
  // upper bound (logit + bound) among the experts left out.
  auto rank_topk = [&](bool exact_only) {
    for (int e = 32 * kLaneKeys + lane; e < E; e += 32) s_gone[e] = 0;
    __syncwarp();
    uint32_t key[kLaneKeys];
#pragma unroll
    for (int j = 0; j < kLaneKeys; ++j) {
      const int e = lane + 32 * j;
      key[j] = (e < E && (!exact_only || s_bound[e] == 0.f))
                   ? ordered_bits(s_logit[e]) : 0u;
    }
    const bool spill = E > 32 * kLaneKeys;
    for (int r = 0; r < k; ++r) {
      uint32_t b = 0;
      int bid = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < kLaneKeys; ++j)
        if (key[j] > b) {
          b = key[j];
          bid = lane + 32 * j;
        }
      if (spill)
        for (int e = lane + 32 * kLaneKeys; e < E; e += 32) {
          const uint32_t o = (s_gone[e] || (exact_only && s_bound[e] != 0.f))
                                 ? 0u : ordered_bits(s_logit[e]);
          if (o > b) {
            b = o;
            bid = e;
          }
        }
      const uint32_t mx = __reduce_max_sync(0xffffffffu, b);
      const uint32_t win = __reduce_min_sync(
          0xffffffffu, (b == mx) ? (uint32_t)bid : 0xffffffffu);
      if ((int)win < 32 * kLaneKeys) {
        if ((int)(win & 31u) == lane) {
#pragma unroll
          for (int j = 0; j < kLaneKeys; ++j)
            if ((int)win == lane + 32 * j) key[j] = 0;
        }
      } else if (lane == 0) {
        s_gone[win] = 1;
      }
      __syncwarp();
      if (lane == r) id1 = (int)win;
      if (lane + 32 == r) id2 = (int)win;
    }
    float u = -INFINITY;
#pragma unroll
    for (int j = 0; j < kLaneKeys; ++j) {
      const int e = lane + 32 * j;
      if (key[j] != 0u) u = fmaxf(u, s_logit[e] + s_bound[e]);
    }
    if (spill)
      for (int e = lane + 32 * kLaneKeys; e < E; e += 32)
        if (!s_gone[e] && !(exact_only && s_bound[e] != 0.f))
          u = fmaxf(u, s_logit[e] + s_bound[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      u = fmaxf(u, __shfl_xor_sync(0xffffffffu, u, o));
    return u;
  };

  bool certified = true;
  if (warp == 0 && !forced) {
    const float u_rest = rank_topk(false);
    // certify: the picks strictly ordered beyond their bounds and the k-th
    // above every other expert's upper bound (exact ties are never
    // certified: they need the exact values and the id order)
    const float lo1 = lane < k ? s_logit[id1] - s_bound[id1] : INFINITY;
    const float lo2 = lane + 32 < k ? s_logit[id2] - s_bound[id2] : INFINITY;
    const float hi1 = lane < k ? s_logit[id1] + s_bound[id1] : -INFINITY;
    const float hi2 = lane + 32 < k ? s_logit[id2] + s_bound[id2] : -INFINITY;
    const float next_hi1 = __shfl_down_sync(0xffffffffu, hi1, 1);
    const float hi2_lane0 = __shfl_sync(0xffffffffu, hi2, 0);
    const float next_hi2 = __shfl_down_sync(0xffffffffu, hi2, 1);
    bool ok = true;
    if (lane + 1 < k) ok &= lo1 > (lane == 31 ? hi2_lane0 : next_hi1);
    if (lane + 33 < k) ok &= lo2 > next_hi2;
    const int last = k - 1;
    const float lo_last = last < 32
                              ? __shfl_sync(0xffffffffu, lo1, last)
                              : __shfl_sync(0xffffffffu, lo2, last - 32);
    ok &= lo_last > u_rest;
    certified = __all_sync(0xffffffffu, ok);
    if (!certified) {
      // rows that could still be in the top k: upper bound at or above the
      // lowest lower bound among the picks
      float thr = fminf(lo1, lo2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        thr = fminf(thr, __shfl_xor_sync(0xffffffffu, thr, o));
      int n = 0;
      for (int base = 0; base < E; base += 32) {
        const int e = base + lane;
        const bool c = e < E && s_logit[e] + s_bound[e] >= thr;
        const uint32_t m = __ballot_sync(0xffffffffu, c);
        if (c) s_cand[n + __popc(m & ((1u << lane) - 1u))] = e;
        n += __popc(m);
      }
      if (lane == 0) s_ncand = n;
    }
    if (lane == 0) s_cert = certified ? 1 : 0;
  } else if (threadIdx.x == 0) {
    s_cert = 1;
  }
  __syncthreads();
  if (!s_cert) {
    // exact fp64 recompute of the candidate rows, one warp per row
    for (int ci = warp; ci < s_ncand; ci += kRouterWarps) {
      const int e = s_cand[ci];
      double acc = 0.0;
      for (int c = lane; c < H; c += 32)
        acc = fma((double)s_x[c], (double)bf16_to_f32(a.w[(size_t)e * H + c]),
                  acc);
      acc = warp_sum_f64(acc);
      if (lane == 0) {
        float l = (float)acc;
        if (a.bias) l = l + a.bias[e];
        s_logit[e] = l;
        s_bound[e] = 0.f;
      }
    }
    __syncthreads();
    // every row left out is below all the picks: rank the exact rows
    if (warp == 0) rank_topk(true);
  }
  if (warp != 0) return;
  SLX_TRACE_AT(0, 4, slx::globaltimer_ns());

  // ---- outputs ----
  uint32_t mk = 0;
  for (int e = lane; e < E; e += 32) {
    const float l = s_logit[e];
    a.logits[(size_t)t * E + e] = l;
    const uint32_t o = ordered_bits(l);
    mk = o > mk ? o : mk;
  }
  mk = __reduce_max_sync(0xffffffffu, mk);
  const float M =
      __uint_as_float((mk & 0x80000000u) ? (mk & 0x7fffffffu) : ~mk);
  float se = 0.f;
  for (int e = lane; e < E; e += 32) se += expf(s_logit[e] - M);
  const float SE = warp_sum_f32(se);
  if (forced) {
    bool bad = false;
    if (lane < k) {
      id1 = a.forced_ids[(size_t)t * k + lane];
      if (id1 < 0 || id1 >= E) {
        bad = true;
        id1 = 0;
      }
    }
    if (lane + 32 < k) {
      id2 = a.forced_ids[(size_t)t * k + lane + 32];
      if (id2 < 0 || id2 >= E) {
        bad = true;
        id2 = 0;
      }
    }
    if (bad) set_status(a.status, SLX_ERR_OUT_OF_RANGE);
  }
  SLX_TRACE_AT(0, 5, slx::globaltimer_ns());
  float p1 = lane < k ? expf(s_logit[id1] - M) / SE : 0.f;
  float p2 = lane + 32 < k ? expf(s_logit[id2] - M) / SE : 0.f;
  if (a.norm_topk) {
    const float sum = warp_sum_f32(p1 + p2);
    p1 /= sum;
    p2 /= sum;
  }
  if (lane < k) {
    a.out_ids[(size_t)t * k + lane] = id1;
    a.out_scores[(size_t)t * k + lane] = p1;
  }
  if (lane + 32 < k) {
    a.out_ids[(size_t)t * k + lane + 32] = id2;
    a.out_scores[(size_t)t * k + lane + 32] = p2;
  }
  SLX_TRACE_AT(0, 6, slx::globaltimer_ns());
}

__global__ void __cluster_dims__(kRouterCluster, 1, 1)
    __launch_bounds__(kRouterThreads, 1) k_router(const RouterLaunch L) {
  namespace cg = cooperative_groups;
  __shared__ __align__(16) float s_x[kRouterMaxH];
  __shared__ float s_logit[kMaxExperts];   // cluster rank 0: the logits
  __shared__ float s_bound[kMaxExperts];   // and their bounds (0 = exact)
  __shared__ uint8_t s_gone[kMaxExperts];  // picked ids beyond the registers
  __shared__ int s_cand[kMaxExperts];      // rows to recompute exactly
  __shared__ int s_ncand;
  __shared__ int s_cert;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int head = blockIdx.x / kRouterCluster;
  const RouterArgs& a = head ? L.h[1] : L.h[0];
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, H = a.H;
  const int epc = (E + kRouterCluster - 1) / kRouterCluster;
  const int e_lo = rank * epc, e_hi = min(E, e_lo + epc);
  // adds along one logit: the lane's chain, the 8-way tree, the butterfly
  const int depth = (H + 255) / 256 + 3 + 5;
  SLX_TRACE_POINT(0, 0);
  pdl_launch_dependents();

  // this warp's first row pair: gate rows are weights, in flight before
  // the wait on the kernel that produced x
  const int ea0 = e_lo + warp, eb0 = ea0 + kRouterWarps;
  uint4 wa[kRouterBatch], wb[kRouterBatch];
#pragma unroll
  for (int i = 0; i < kRouterBatch; ++i) {
    const int c = i * 256 + lane * 8;
    wa[i] = (ea0 < e_hi && c < H)
                ? __ldg(reinterpret_cast<const uint4*>(a.w + (size_t)ea0 * H + c))
                : make_uint4(0, 0, 0, 0);
    wb[i] = (eb0 < e_hi && c < H)
                ? __ldg(reinterpret_cast<const uint4*>(a.w + (size_t)eb0 * H + c))
                : make_uint4(0, 0, 0, 0);
  }
  pdl_wait_primary();
  // stage x (times the ratio, rounded to bf16, for the predictor) as fp32
  const uint16_t* xr = a.x + (size_t)t * H;
  for (int c = threadIdx.x * 8; c < H; c += kRouterThreads * 8) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t rw[4] = {0, 0, 0, 0};
    if (a.ratio) {
      const uint4 rv = *reinterpret_cast<const uint4*>(a.ratio + c);
      rw[0] = rv.x; rw[1] = rv.y; rw[2] = rv.z; rw[3] = rv.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float x0 = bf16_lo(xw[q]), x1 = bf16_hi(xw[q]);
      if (a.ratio) {
        x0 = round_bf16(x0 * bf16_lo(rw[q]));
        x1 = round_bf16(x1 * bf16_hi(rw[q]));
      }
      s_x[c + 2 * q] = x0;
      s_x[c + 2 * q + 1] = x1;
    }
  }
  __syncthreads();
  SLX_TRACE_POINT(0, 1);
  float* leader_logit = cluster.map_shared_rank(s_logit, 0);
  float* leader_bound = cluster.map_shared_rank(s_bound, 0);
  for (int ea = ea0; ea < e_hi; ea += 2 * kRouterWarps) {
    const int eb = ea + kRouterWarps;
    const bool hb = eb < e_hi;
    float sA[8] = {0, 0, 0, 0, 0, 0, 0, 0}, aA[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sB[8] = {0, 0, 0, 0, 0, 0, 0, 0}, aB[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int base = 0; base < H; base += 256 * kRouterBatch) {
      if (base > 0 || ea != ea0) {
#pragma unroll
        for (int i = 0; i < kRouterBatch; ++i) {
          const int c = base + i * 256 + lane * 8;
          wa[i] = c < H ? __ldg(reinterpret_cast<const uint4*>(
                              a.w + (size_t)ea * H + c))
                        : make_uint4(0, 0, 0, 0);
          wb[i] = (hb && c < H) ? __ldg(reinterpret_cast<const uint4*>(
                                      a.w + (size_t)eb * H + c))
                                : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int i = 0; i < kRouterBatch; ++i) {
        const int c = base + i * 256 + lane * 8;
        if (c < H) {
          dot8(s_x + c, wa[i], sA, aA);
          dot8(s_x + c, wb[i], sB, aB);
        }
      }
    }
    const float ssa = warp_sum_f32(sum8(sA)), asa = warp_sum_f32(sum8(aA));
    const float ssb = warp_sum_f32(sum8(sB)), asb = warp_sum_f32(sum8(aB));
    if (lane == 0) {
      const float la = a.bias ? ssa + a.bias[ea] : ssa;
      leader_logit[ea] = la;
      leader_bound[ea] = logit_bound(ssa, asa, la, depth);
      if (hb) {
        const float lb = a.bias ? ssb + a.bias[eb] : ssb;
        leader_logit[eb] = lb;
        leader_bound[eb] = logit_bound(ssb, asb, lb, depth);
      }
    }
  }
  SLX_TRACE_POINT(0, 2);
  cluster.sync();  // every logit and bound is in rank 0's shared memory
  SLX_TRACE_POINT(0, 3);
  if (rank != 0) return;

  rank_and_write(a, t, s_x, s_logit, s_bound, s_gone, s_cand, s_ncand, s_cert);
}

// One-token form over many SMs: CTA c of a head owns kWideRows gate rows,
// brought into shared memory by one bulk copy issued before the kernel
// waits on its predecessor (the gate is immutable); four warps per row each
// take a quarter of the columns.  Each CTA leaves its rows' logits and
// bounds in the head's scratch and takes a ticket; the CTA that takes the
// last one ranks the head (rank_and_write) and puts the ticket back to 0.
constexpr int kWideRows = 4;
constexpr int kWideSplit = kRouterWarps / kWideRows;  // warps per row

struct WideLaunch {
  RouterArgs h[2];
  float* bound[2];  // [E] per head
  int n_heads, ctas_per_head;
  RouterNorm norm;  // norm.w != null: x = RMSNorm(h_in + delta) first
};

// The token's x = bf16(bf16(h_in + delta) * rsqrt(mean + eps) * w) into
// s_x (times the ratio, rounded, when `ratio`), with the arithmetic and the
// summation order of k_add_rmsnorm (256 threads of 8-value chunks, chunk c
// of thread t = (j * 256 + t) * 8, each warp's sum by butterfly, the warps'
// sums added in order); CTA 0 also stores h_in + delta and x.  All threads
// of the CTA call this.
constexpr int kNormT = 256, kNormJ = 4;

// The thread's chunks of the norm weight and the ratio: fixed weights,
// loaded before the kernel waits on its predecessor.
struct NormWeights {
  uint4 w[kNormJ];
  uint4 r[kNormJ];
};

SLX_DEV void norm_weights(const RouterNorm& nm, int H, const uint16_t* ratio,
                          NormWeights& nw) {
  const int t = threadIdx.x;
  if (t >= kNormT) return;
#pragma unroll
  for (int j = 0; j < kNormJ; ++j) {
    const int c = (j * kNormT + t) * 8;
    if (c >= H) break;
    nw.w[j] = __ldg(reinterpret_cast<const uint4*>(nm.w + c));
    if (ratio) nw.r[j] = __ldg(reinterpret_cast<const uint4*>(ratio + c));
  }
}

SLX_DEV void norm_stage(const RouterNorm& nm, int H, const uint16_t* ratio,
                        const NormWeights& nw, float* s_x, float* red,
                        bool store) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  uint4 v[kNormJ];
  float ss = 0.f;
  if (t < kNormT) {
#pragma unroll
    for (int j = 0; j < kNormJ; ++j) {
      const int c = (j * kNormT + t) * 8;
      if (c >= H) break;
      uint4 a = *reinterpret_cast<const uint4*>(nm.h_in + c);
      if (nm.delta) {
        const uint4 b = *reinterpret_cast<const uint4*>(nm.delta + c);
        uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
        const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = round_bf16(bf16_lo(pa[q]) + bf16_lo(pb[q]));
          const float hi = round_bf16(bf16_hi(pa[q]) + bf16_hi(pb[q]));
          pa[q] = (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
        }
      }
      if (store) *reinterpret_cast<uint4*>(nm.h_out + c) = a;
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float lo = bf16_lo(pa[q]), hi = bf16_hi(pa[q]);
        ss += lo * lo + hi * hi;
      }
      v[j] = a;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __syncthreads();
  if (lane == 0 && warp < kNormT / 32) red[warp] = ss;
  __syncthreads();
  float tot = red[0];
  for (int w = 1; w < kNormT / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)H + nm.eps);
  if (t < kNormT) {
#pragma unroll
    for (int j = 0; j < kNormJ; ++j) {
      const int c = (j * kNormT + t) * 8;
      if (c >= H) break;
      const uint4 wv = nw.w[j];
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
      if (store) *reinterpret_cast<uint4*>(nm.y + c) = o;
      uint32_t rw[4] = {0, 0, 0, 0};
      if (ratio) {
        const uint4 rv = nw.r[j];
        rw[0] = rv.x; rw[1] = rv.y; rw[2] = rv.z; rw[3] = rv.w;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x0 = bf16_lo(po[q]), x1 = bf16_hi(po[q]);
        if (ratio) {
          x0 = round_bf16(x0 * bf16_lo(rw[q]));
          x1 = round_bf16(x1 * bf16_hi(rw[q]));
        }
        s_x[c + 2 * q] = x0;
        s_x[c + 2 * q + 1] = x1;
      }
    }
  }
}

__global__ void __launch_bounds__(kRouterThreads, 1)
    k_router_wide(const __grid_constant__ WideLaunch L) {
  extern __shared__ __align__(128) uint8_t wsm[];  // the CTA's gate rows (bf16)
  __shared__ __align__(16) float s_x[kRouterMaxH];
  __shared__ float s_logit[kMaxExperts];
  __shared__ float s_bound[kMaxExperts];
  __shared__ uint8_t s_gone[kMaxExperts];
  __shared__ int s_cand[kMaxExperts];
  __shared__ int s_ncand, s_cert, s_last;
  __shared__ float s_part[kWideRows][kWideSplit][2];
  __shared__ __align__(8) uint64_t s_bar;
  const int head = blockIdx.x / L.ctas_per_head, cb = blockIdx.x % L.ctas_per_head;
  const RouterArgs& a = head ? L.h[1] : L.h[0];
  float* gbound = L.bound[head];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, H = a.H;
  const int e0 = cb * kWideRows;
  const int nr = E - e0 < kWideRows ? E - e0 : kWideRows;
  const uint16_t* rows = reinterpret_cast<const uint16_t*>(wsm);
  if (threadIdx.x == 0) {
    mbar_init(&s_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&s_bar, (uint32_t)nr * H * 2);
    bulk_g2s_plain(wsm, a.w + (size_t)e0 * H, (uint32_t)nr * H * 2, &s_bar);
  }
  // fixed weights in flight before the wait: the norm weight and ratio
  // chunks of this thread, the bias of its row
  NormWeights nw;
  if (L.norm.w) norm_weights(L.norm, H, a.ratio, nw);
  const float row_bias =
      (a.bias && threadIdx.x < nr) ? __ldg(a.bias + e0 + threadIdx.x) : 0.f;
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ float s_red[32];
  const uint16_t* xr = a.x;  // one token
  if (L.norm.w) {
    norm_stage(L.norm, H, a.ratio, nw, s_x, s_red, blockIdx.x == 0);
  } else {
  for (int c = threadIdx.x * 8; c < H; c += kRouterThreads * 8) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t rw[4] = {0, 0, 0, 0};
    if (a.ratio) {
      const uint4 rv = *reinterpret_cast<const uint4*>(a.ratio + c);
      rw[0] = rv.x; rw[1] = rv.y; rw[2] = rv.z; rw[3] = rv.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float x0 = bf16_lo(xw[q]), x1 = bf16_hi(xw[q]);
      if (a.ratio) {
        x0 = round_bf16(x0 * bf16_lo(rw[q]));
        x1 = round_bf16(x1 * bf16_hi(rw[q]));
      }
      s_x[c + 2 * q] = x0;
      s_x[c + 2 * q + 1] = x1;
    }
  }
  }
  __syncthreads();
  const bool ok = mbar_wait(&s_bar, 0, a.status);
  // row r, column quarter q: eight fp32 chains per lane, then the tree
  const int r = warp / kWideSplit, q = warp % kWideSplit;
  const int Hq = H / kWideSplit;
  float sv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, av[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (ok && r < nr)
    for (int c = q * Hq + lane * 8; c < (q + 1) * Hq; c += 256)
      dot8(s_x + c, *reinterpret_cast<const uint4*>(rows + (size_t)r * H + c), sv, av);
  const float ss = warp_sum_f32(sum8(sv)), as = warp_sum_f32(sum8(av));
  if (lane == 0) {
    s_part[r][q][0] = ss;
    s_part[r][q][1] = as;
  }
  __syncthreads();
  // adds along one logit: the lane's chain, the 8-way tree, the butterfly,
  // the quarters
  const int depth = (Hq + 255) / 256 + 3 + 5 + 2;
  if (threadIdx.x < nr) {
    const int rr = threadIdx.x, e = e0 + rr;
    const float S = (s_part[rr][0][0] + s_part[rr][1][0]) + (s_part[rr][2][0] + s_part[rr][3][0]);
    const float A = (s_part[rr][0][1] + s_part[rr][1][1]) + (s_part[rr][2][1] + s_part[rr][3][1]);
    const float l = a.bias ? S + row_bias : S;
    a.logits[e] = l;
    gbound[e] = logit_bound(S, A, l, depth);
  }
  // the CTA's stores are ordered before the ticket by the barrier and the
  // ticket's release (cumulative); its acquire orders the last CTA's reads
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = ticket_acq_rel(a.tickets);
    s_last = old == L.ctas_per_head - 1;
    if (s_last) *reinterpret_cast<volatile int32_t*>(a.tickets) = 0;
  }
  __syncthreads();
  if (!s_last) return;
  for (int e = threadIdx.x; e < E; e += kRouterThreads) {
    s_logit[e] = __ldcg(a.logits + e);
    s_bound[e] = __ldcg(gbound + e);
  }
  __syncthreads();
  rank_and_write(a, 0, s_x, s_logit, s_bound, s_gone, s_cand, s_ncand, s_cert);
}

int launch_router_heads(const RouterArgs* heads, int n_heads,
                        cudaStream_t stream, const RouterNorm* norm) {
  if (n_heads < 1 || n_heads > 2) return SLX_ERR_INVALID;
  const RouterArgs& a = heads[0];
  for (int i = 0; i < n_heads; ++i) {
    const RouterArgs& b = heads[i];
    if (b.E > kMaxExperts || b.k > kRouterMaxK || b.k < 1 || b.k > b.E ||
        b.H % 8 || b.H > kRouterMaxH)
      return SLX_ERR_UNSUPPORTED;
    if (b.E != a.E || b.T != a.T || b.H != a.H || b.k != a.k)
      return SLX_ERR_INVALID;
  }
  if (a.T <= 0) return SLX_OK;
  if (a.T > 65535) return SLX_ERR_INVALID;
  const bool wide = a.T == 1 && a.H % (8 * kWideSplit) == 0 && heads[0].bound &&
                    (n_heads < 2 || heads[1].bound);
  if (norm && (!wide || a.H > 8 * kNormT * kNormJ)) return SLX_ERR_UNSUPPORTED;
  if (wide) {
    WideLaunch W = {};
    if (norm) W.norm = *norm;
    W.h[0] = heads[0];
    W.h[1] = n_heads > 1 ? heads[1] : heads[0];
    W.bound[0] = heads[0].bound;
    W.bound[1] = W.h[1].bound;
    W.n_heads = n_heads;
    W.ctas_per_head = (a.E + kWideRows - 1) / kWideRows;
    const int smem = kWideRows * a.H * 2;
    static PerDevice attr;
    std::atomic<int>& slot = attr.here();
    if (!slot.load(std::memory_order_relaxed)) {
      if (cudaFuncSetAttribute(k_router_wide,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kWideRows * kRouterMaxH * 2) != cudaSuccess)
        return SLX_ERR_CUDA;
      slot.store(1, std::memory_order_relaxed);
    }
    return launch_k(k_router_wide, dim3(W.ctas_per_head * n_heads),
                    dim3(kRouterThreads), smem, stream, W) == cudaSuccess
               ? SLX_OK : SLX_ERR_CUDA;
  }
  RouterLaunch L = {};
  L.h[0] = heads[0];
  L.h[1] = n_heads > 1 ? heads[1] : heads[0];
  L.n_heads = n_heads;
  dim3 grid(kRouterCluster * n_heads, a.T);
  return launch_k(k_router, grid, dim3(kRouterThreads), 0, stream, L) ==
                 cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_router(const RouterArgs& a, cudaStream_t stream) {
  return launch_router_heads(&a, 1, stream, nullptr);
}

}  // namespace slx
