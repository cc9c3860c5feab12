// Quantized (MLX affine 2/4/8-bit, group 64) GEMV engine for sm_100a.
//
// Replaces, for batch-1 decode, the three `mx.gather_qmm` calls plus
// `swiglu` of the reference's `switch_forward` (streamlx/pool.py:30-50), the
// id->slot remap (streamlx/integrate.py:90-95) and the score-weighted combine
// of the mlx-lm MoE block around it (streamlx/integrate.py:5-7).  Two
// kernels, chained with programmatic dependent launch so the second one's
// weight stream starts while the first is still running:
//
//   k_qgemv<BITS>  (phase A)  gate+up pair tiles of every routed expert (and
//                  the optional shared expert) -> h = bf16(silu(bf16 g) *
//                  bf16 u) into a small scratch buffer.  The same kernel in
//                  LINEAR mode is the trunk's dense quantized linear.
//   k_down<BITS>   (phase B)  down single tiles of every routed expert,
//                  per-expert bf16 rounding (MLX returns bf16 from
//                  gather_qmm), then the router-score-weighted sum (+ shared
//                  expert) with one bf16 rounding.  Each output row is owned
//                  by one CTA: the combine is deterministic, no atomics.
//
// Weights are read in the tile format of slx_tiles.cuh, so one 16-row tile
// arrives in a single bulk copy; requests are issued many per instruction
// (the copy engine's cost is per request and per issuing instruction).
//
// Warp specialisation: warp 0 issues the bulk copies (TMA engine, L2
// evict-first, mbarrier completion); warps 1..8 split a tile's 64-column
// groups.  Codes are unpacked in registers by one AND per fp16 pair (the
// code becomes an exact fp16 subnormal, slx_common.cuh) and multiplied on
// the tensor cores (mma.sync m16n8k16, fp32 accumulate) against the
// activation, which sits in shared memory as ready-made B fragments with the
// unpack's power-of-two factors folded in.  Per group the fp32 result is
// folded with the MLX affine identity
//     sum_c x_c (s q_c + b) = s * sum_c q_c x_c + b * sum_c x_c,
// so no dequantised weight is ever materialised.
// Every mbarrier wait is bounded (slx_common.cuh: mbar_wait).
#include "slx_kernels.cuh"
#include "slx_pack.cuh"
#include "slx_tiles.cuh"

#ifdef SLX_TRACE
static __device__ unsigned long long g_slx_trace[3][160][16];
extern "C" int slx_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, g_slx_trace, sizeof(g_slx_trace)) ==
                 cudaSuccess ? 0 : -1;
}
#endif

namespace slx {

constexpr int kNW = 8;                    // consumer warps
constexpr int kXTasks = 1;  // activation tasks a consumer thread holds in registers
constexpr int kThreads = 32 * (kNW + 1);  // + producer warp
constexpr int kMaxStages = 32;
constexpr int kRows = 16;

struct TileInfo {
  int token;
  int unit;               // routed unit u = token*k + pick; -1-token: shared
  int ti;                 // 16-row tile index inside the unit
  int valid;
  int valid1;             // LINEAR: second 16-row half inside the matrix
  const uint8_t* src;     // tile in global memory
  uint16_t* out;          // GLU: h + row0; LINEAR: y + row0
};

SLX_DEV int lookup_slot(const int32_t* ids, int u, const int32_t* table,
                        int n_table, int n_slots) {
  const int e = ids[u];
  int s = e;
  // L2 read: a decode launch may rewrite the table while it runs (the
  // in-kernel slot fill), so no L1 line of it may be reused across that
  if (table) s = (e >= 0 && e < n_table) ? __ldcg(table + e) : -1;
  return (s >= 0 && s < n_slots) ? s : -1;
}

// Remembers the last unit's slot so consecutive tiles of one expert cost no
// global loads.
struct SlotCache {
  int unit = -1;
  int slot = -1;
};

SLX_DEV TileInfo gemv_tile(const GemvArgs& a, int q, SlotCache& sc) {
  TileInfo t{};
  if (a.mode == SLX_GEMV_LINEAR) {
    const int tpu = (a.out_features + 31) / 32;
    t.token = q / tpu;
    const int ti = q % tpu;
    t.valid = 1;
    t.valid1 = (32 * ti + 16) < a.out_features;
    t.src = a.lin + (size_t)ti * a.tile_bytes;
    t.out = a.y + (size_t)t.token * a.out_features + 32 * ti;
    return t;
  }
  const int tpu = a.I / kRows;
  const int routed = a.T * a.k * tpu;
  if (q < routed) {
    const int u = q / tpu, ti = q % tpu;
    t.token = u / a.k;
    if (u != sc.unit) {
      sc.unit = u;
      sc.slot = lookup_slot(a.ids, u, a.slot_table, a.n_table, a.n_slots);
    }
    const int slot = sc.slot;
    t.valid = t.valid1 = slot >= 0;
    t.unit = u;
    t.ti = ti;
    t.src = a.bank + (size_t)(slot < 0 ? 0 : slot) * a.slot_stride +
            (size_t)ti * a.tile_bytes;
    t.out = nullptr;
    return t;
  }
  const int qs = q - routed, tps = a.Is / kRows;
  t.token = qs / tps;
  const int ti = qs % tps;
  t.valid = t.valid1 = 1;
  t.unit = -1 - t.token;  // shared expert of token t
  t.ti = ti;
  t.src = a.shared + (size_t)ti * a.tile_bytes;
  t.out = nullptr;
  return t;
}

// ------------------------------------------------- activation fragments ---
//
// frag[G][tig][8]: fp16 pairs matching unpack register j of a thread with
// this tig (columns 64G + 16 tig + col_lo/hi(j)), each multiplied by
// act_scale (a power of two: exact); xsum[G] = sum of the group's 64
// activations (the bias term of the affine identity).  One (group, tig)
// task per thread, all units at once: a single round of global loads.
// An activation the fp16 fragments cannot hold (|x * factor| >= 65504
// would become inf; non-finite inputs) is reported as SLX_ERR_RANGE.
constexpr float kF16Max = 65504.f;

// The tensor cores lose low-order bits of a k16 sum when its products are
// tiny (fp16-subnormal code operands times small activations: measured
// 0.1-24% of bf16 outputs off by an ulp, falling to ~0.05% once the
// activations are raised by 2^6..2^12).  So each activation vector enters
// the fp16 fragments multiplied by a power of two 2^e chosen per vector
// (its largest magnitude lands in [2^12, 2^13)), and the SwiGLU outputs by
// the fixed kHScale; the fold divides by the same power of two, so the
// arithmetic is exact up to that scaling.
constexpr float kHScale = 64.f;       // 2^6 on the down projection's input
constexpr float kHUnit = 262144.f;    // 2^24 / kHScale

SLX_DEV float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// Exponent e for a vector whose largest |value| is m (0: e = 0).
SLX_DEV int vec_exp(float m) {
  if (!(m > 0.f) || !(m < 3.0e38f)) return 0;
  int ex;
  frexpf(m, &ex);                     // m = f * 2^ex, f in [0.5, 1)
  int e = 13 - ex;                    // m * 2^e in [2^12, 2^13)
  return e < -60 ? -60 : (e > 60 ? 60 : e);
}

// Largest |x| of n bf16 values (8 per 16-byte load), this thread's share.
SLX_DEV float absmax_part(const uint16_t* x, int n, int t, int nt) {
  float m = 0.f;
  for (int c = 8 * t; c < n; c += 8 * nt) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      m = fmaxf(m, fmaxf(fabsf(bf16_lo(w[q])), fabsf(bf16_hi(w[q]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

// Largest |x| of the 16 bf16 values of one (group, tig) task.
SLX_DEV float absmax16(const uint4& q0, const uint4& q1) {
  const uint32_t w8[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  float m = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    m = fmaxf(m, fmaxf(fabsf(bf16_lo(w8[q])), fabsf(bf16_hi(w8[q]))));
  return m;
}

// Fragment words and partial sum of task (G, tig) from its 16 values
// (columns 64G + 16 tig .. + 15, eight per uint4).
template <int BITS>
SLX_DEV void frag_from(const uint4& q0, const uint4& q1, int G, int tig,
                       uint32_t* frag, float* part, int32_t* status,
                       float vscale) {
  const uint32_t w8[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int cl = col_lo(BITS, j), ch = col_hi(BITS, j);
    const float xl = (cl & 1) ? bf16_hi(w8[cl >> 1]) : bf16_lo(w8[cl >> 1]);
    const float xh = (ch & 1) ? bf16_hi(w8[ch >> 1]) : bf16_lo(w8[ch >> 1]);
    const float sl = xl * vscale * act_scale(BITS, cl);
    const float sh = xh * vscale * act_scale(BITS, ch);
    if (status && !(fabsf(sl) < kF16Max && fabsf(sh) < kF16Max))
      set_status(status, SLX_ERR_RANGE);
    frag[(G * 4 + tig) * 8 + j] = pack_f16x2(sl, sh);
    s += xl + xh;
  }
  part[G * 4 + tig] = s;
}

template <int BITS>
SLX_DEV void frag_task(const uint16_t* __restrict__ x, int G, int tig,
                       uint32_t* frag, float* part, int32_t* status,
                       float vscale) {
  const uint4* src = reinterpret_cast<const uint4*>(x + 64 * G + 16 * tig);
  frag_from<BITS>(src[0], src[1], G, tig, frag, part, status, vscale);
}

// Sum the four per-tig partials of every group (fixed order).
SLX_DEV void frag_sums(const float* part, float* xsum, int n, int tid,
                       int nthr) {
  for (int i = tid; i < n; i += nthr)
    xsum[i] = (part[4 * i] + part[4 * i + 1]) + (part[4 * i + 2] + part[4 * i + 3]);
}

// The activation fragments of a token too wide for one task per consumer
// thread (two rounds of loads); returns the fold's unit.  All consumer
// threads call this.
SLX_DEV void named_bar_consumers();
template <int BITS>
__device__ __noinline__ float frag_wide(const uint16_t* xr, int in, int nG,
                                        int ct, uint32_t* frag, float* part,
                                        float* s_vmax, int32_t* status) {
  named_bar_consumers();  // every consumer is past the previous token's MMAs
  const float m = absmax_part(xr, in, ct, kNW * 32);
  if ((ct & 31) == 0) s_vmax[ct >> 5] = m;
  named_bar_consumers();
  float mm = 0.f;
  for (int w = 0; w < kNW; ++w) mm = fmaxf(mm, s_vmax[w]);
  const int ve = vec_exp(mm);
  for (int p = ct; p < 4 * nG; p += kNW * 32)
    frag_task<BITS>(xr, p >> 2, p & 3, frag, part, status, pow2f(ve));
  return pow2f(24 - ve);
}

SLX_DEV void load_frag(const uint32_t* frag, int G, int tig, uint32_t (&b)[8]) {
  const uint4* fp = reinterpret_cast<const uint4*>(frag + (G * 4 + tig) * 8);
  const uint4 f0 = fp[0], f1 = fp[1];
  b[0] = f0.x; b[1] = f0.y; b[2] = f0.z; b[3] = f0.w;
  b[4] = f1.x; b[5] = f1.y; b[6] = f1.z; b[7] = f1.w;
}

// The thread's packed codes of row `row` (tile row block `blk`), group G.
template <int BITS>
SLX_DEV void load_unpack(const uint8_t* blk, int row, int G, int tig, int RB,
                         bool swz, uint32_t (&r)[8]) {
  const int off = swz_offset(row, 8 * BITS * G + 2 * BITS * tig, RB, swz);
  const uint8_t* p = blk + off;
  if constexpr (BITS == 2) {
    unpack2(*reinterpret_cast<const uint32_t*>(p), r);
  } else if constexpr (BITS == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    unpack4(w.x, w.y, r);
  } else {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    unpack8(ws, r);
  }
}

// 16 rows x 64 columns of one row block against the activation fragment:
// d = 2^-24 * sum_c q[row, c] * x[c]  (rows g and g+8 in d[0..1] / d[2..3]).
template <int BITS>
SLX_DEV void group_mma(const uint8_t* blk, int RB, bool swz, int G, int g,
                       int tig, const uint32_t (&b)[8], float (&d)[4]) {
  uint32_t ra[8], rb[8];
  load_unpack<BITS>(blk, g, G, tig, RB, swz, ra);
  load_unpack<BITS>(blk, g + 8, G, tig, RB, swz, rb);
  // four independent k16 products (no accumulator chain), summed in fp32
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  float p[4][4];
#pragma unroll
  for (int m = 0; m < 4; ++m)
    mma_f16_16816(p[m], ra[2 * m], rb[2 * m], ra[2 * m + 1], rb[2 * m + 1],
                  b[2 * m], b[2 * m + 1], z);
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = (p[0][i] + p[1][i]) + (p[2][i] + p[3][i]);
}

SLX_DEV void named_bar_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(kNW * 32) : "memory");
}

// fold one group: acc += scale * sum(q*x) + bias * sum(x); sb = scale|bias
SLX_DEV float fold(float acc, float d, uint32_t sb, float xs, float unit) {
  acc = fmaf(bf16_lo(sb) * unit, d, acc);
  return fmaf(bf16_hi(sb), xs, acc);
}

// ------------------------------------------------------- phase A kernel ---
//
// Pipeline without CTA-wide barriers in the steady state:
//   consumer warps: wait full[s] -> MMA over their groups -> partial dot to
//     red[s][warp] -> arrive redfull[s];
//   warp 0: issues tile copies; per tile, waits redfull[s] (which also means
//     stage s is free), refills stage s, reduces the 8 partials, runs the
//     epilogue (SwiGLU -> down-projection fragments, or the LINEAR output)
//     and arrives redempty[s] so consumers may reuse red[s].

template <int BITS>
SLX_DEV void gemv_issue(const GemvArgs& a, const TileInfo& t, uint8_t* dst,
                        uint64_t* bar, uint64_t pol) {
  if (t.valid) {
    mbar_arrive_expect_tx(bar, a.tile_bytes);
    bulk_g2s(dst, t.src, a.tile_bytes, bar, pol);
  } else {
    mbar_arrive(bar);
  }
}

// Reduce the tile's partials (red[w][lane], w < kNW) and write its output.
// Lane (g, tig): tig>>1 selects the matrix (gate/up or rows 0-15/16-31),
// tig&1 the row half.  All 32 lanes must call this.
template <int BITS, int NWR = kNW>
SLX_DEV void gemv_epilogue(const GemvArgs& a, const TileInfo& t,
                           const float* red, int lane) {
  const int g = lane >> 2, tig = lane & 3;
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < NWR; ++w) v += red[w * 32 + lane];
  if (a.mode != SLX_GEMV_GLU) {
    const int mat = tig >> 1;
    const int r = 16 * mat + g + 8 * (tig & 1);
    if (mat == 0 || t.valid1) t.out[r] = f32_to_bf16(v);
    return;
  }
  // h for the tile's 16 rows = 16 activation columns of the down
  // projection, i.e. exactly fragment block (G = ti/4, tig = ti%4) of phase
  // B.  Lane (g, t<2) holds h[row g + 8t].
  const float up = __shfl_down_sync(0xffffffffu, v, 2);
  float hv = 0.f;
  if (tig < 2) {
    const float gb = round_bf16(v), ubf = round_bf16(up);
    hv = t.valid ? round_bf16(gb / (1.f + expf(-gb)) * ubf) : 0.f;
  }
  const int j = lane & 7;
  const int cl = col_lo(BITS, j), ch = col_hi(BITS, j);
  const float lo = __shfl_sync(0xffffffffu, hv, (cl & 7) * 4 + (cl >> 3));
  const float hi = __shfl_sync(0xffffffffu, hv, (ch & 7) * 4 + (ch >> 3));
  const float slo = lo * (kHScale * act_scale(BITS, cl));
  const float shi = hi * (kHScale * act_scale(BITS, ch));
  if (!(fabsf(slo) < kF16Max && fabsf(shi) < kF16Max))
    set_status(a.status, SLX_ERR_RANGE);
  const uint32_t word = pack_f16x2(slo, shi);
  float hsum = hv;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) hsum += __shfl_xor_sync(0xffffffffu, hsum, o);
  uint32_t* fr;
  float* pt;
  if (t.unit >= 0) {
    fr = a.hfrag + (size_t)t.unit * a.unit_frag_words;
    pt = a.hpart + (size_t)t.unit * a.unit_part_floats;
  } else {
    const int tok = -1 - t.unit;
    fr = a.hfrag_sh + (size_t)tok * a.shared_frag_words;
    pt = a.hpart_sh + (size_t)tok * a.shared_part_floats;
  }
  if (lane < 8) fr[t.ti * 8 + lane] = word;  // block (G*4 + tig) = ti
  if (lane == 0) pt[t.ti] = hsum;
}

template <int BITS>
__global__ void __launch_bounds__(kThreads, 2)
    k_qgemv(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nG = tile_ng(a.in), RB = tile_rb(a.in, BITS);
  const bool swz = tile_swizzled(a.in, BITS);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* redfull = full + kMaxStages;
  uint64_t* redempty = redfull + kMaxStages;
  uint32_t* frag = reinterpret_cast<uint32_t*>(smem + 3 * kMaxStages * 8);
  float* xsum = reinterpret_cast<float*>(frag + nG * 32);
  float* part = xsum + nG;     // [nG][4]
  float* red = part + 4 * nG;  // [NS][kNW][32]
  const int NS = a.n_stages;
  float* s_vmax = red + NS * kNW * 32;  // [kNW] consumer warps' max |x|
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(s_vmax + kNW) + 127) & ~uintptr_t(127));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_begin = (int)((long long)a.n_tiles * blockIdx.x / gridDim.x);
  const int q_end = (int)((long long)a.n_tiles * (blockIdx.x + 1) / gridDim.x);
  const int n = q_end - q_begin;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&redfull[i], kNW);
      mbar_init(&redempty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  SLX_TRACE_POINT(0, 0);
  SLX_TRACE_SMID(0);
  // A dense matrix's tiles are fixed weights: they may be in flight before
  // the wait; an expert tile's address depends on the routed ids.  The
  // dependent grid may launch now (dense: it waits for us before reading
  // anything we write) or, for the expert phase, once the ids are final
  // (the down projection reads ids and the slot table before its wait).
  const bool early = a.mode == SLX_GEMV_LINEAR;
  if (!early) pdl_wait_primary();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------- producer + epilogue ---
    // The first NS tiles go out in one instruction (lane i -> tile i): the
    // copy engine serves the requests of one instruction together.
    const uint64_t pol = l2_evict_first_policy();
    const int first = n < NS ? n : NS;
    SlotCache issue_cache, epi_cache;
    if (lane < first)
      gemv_issue<BITS>(a, gemv_tile(a, q_begin + lane, issue_cache),
                       stages + (size_t)lane * a.stage_bytes, &full[lane], pol);
    if (early) pdl_wait_primary();  // before the epilogue writes y
    for (int i = 0; i < n; ++i) {
      const int st = i % NS;
      if (!mbar_wait(&redfull[st], (i / NS) & 1, a.status)) break;
      // every consumer is done with stage st: refill it
      if (lane == 0 && i + NS < n)
        gemv_issue<BITS>(a, gemv_tile(a, q_begin + i + NS, issue_cache),
                         stages + (size_t)st * a.stage_bytes, &full[st], pol);
      gemv_epilogue<BITS>(a, gemv_tile(a, q_begin + i, epi_cache),
                          red + st * kNW * 32, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&redempty[st]);
      if (i < 6) SLX_TRACE_AT(2, 8 + i, globaltimer_ns());
    }
    return;
  }

  // ------------------------------------------------------- consumers ---
  if (early) pdl_wait_primary();  // x comes from the preceding kernel
  const int cw = warp - 1;  // consumer warp 0..kNW-1
  const int ct = threadIdx.x - 32;
  const int g = lane >> 2, tig = lane & 3;
  const int mat = tig >> 1;
  const int sbl = mat * 16 + g + 8 * (tig & 1);  // this lane's SB word slot
  int cached_token = -1;
  float vunit = kSubnormalUnit;
  SlotCache scache;
  for (int q = q_begin, i = 0; q < q_end; ++q, ++i) {
    const int st = i % NS;
    const TileInfo t = gemv_tile(a, q, scache);
    if (t.token != cached_token) {
      const uint16_t* xr = a.x + (size_t)t.token * a.in;
      if (4 * nG <= kXTasks * kNW * 32) {
        // one round of global loads: the thread's (group, tig) tasks keep
        // their 16 values in registers for the scale and the fragments
        uint4 xv[kXTasks][2];
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < kXTasks; ++j) {
          const int p = ct + j * kNW * 32;
          if (p < 4 * nG) {
            const uint4* src = reinterpret_cast<const uint4*>(
                xr + 64 * (p >> 2) + 16 * (p & 3));
            xv[j][0] = src[0];
            xv[j][1] = src[1];
            m = fmaxf(m, absmax16(xv[j][0], xv[j][1]));
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) s_vmax[cw] = m;
        // also: every consumer is past the previous token's MMAs, so its
        // fragments may be overwritten
        named_bar_consumers();
        float mm = 0.f;
        for (int w = 0; w < kNW; ++w) mm = fmaxf(mm, s_vmax[w]);
        const int ve = vec_exp(mm);
        vunit = pow2f(24 - ve);
#pragma unroll
        for (int j = 0; j < kXTasks; ++j) {
          const int p = ct + j * kNW * 32;
          if (p < 4 * nG)
            frag_from<BITS>(xv[j][0], xv[j][1], p >> 2, p & 3, frag, part,
                            a.status, pow2f(ve));
        }
      } else {
        vunit = frag_wide<BITS>(xr, a.in, nG, ct, frag, part, s_vmax, a.status);
      }
      named_bar_consumers();
      frag_sums(part, xsum, nG, ct, kNW * 32);
      named_bar_consumers();
      cached_token = t.token;
      SLX_TRACE_POINT(0, 1);
    }
    if (!t.valid && ct == 0) set_status(a.status, SLX_ERR_UNMAPPED_EXPERT);
    const bool ok = mbar_wait(&full[st], (i / NS) & 1, a.status);
    if (i < 6) SLX_TRACE_POINT(0, 2 + 2 * i);
    const uint8_t* S = stages + (size_t)st * a.stage_bytes;
    float acc = 0.f;
    if (ok && t.valid) {
      const uint8_t* P = S;
      const uint8_t* Q = S + 16 * RB;
      const uint32_t* SB = reinterpret_cast<const uint32_t*>(S + 32 * RB);
      // two groups in flight per warp (independent MMA chains)
      for (int G = cw; G < nG; G += 2 * kNW) {
        const int G2 = G + kNW;
        const bool two = G2 < nG;
        uint32_t b[8], b2[8];
        load_frag(frag, G, tig, b);
        if (two) load_frag(frag, G2, tig, b2);
        float d0[4], d1[4];
        float e0[4] = {0.f, 0.f, 0.f, 0.f}, e1[4] = {0.f, 0.f, 0.f, 0.f};
        group_mma<BITS>(P, RB, swz, G, g, tig, b, d0);
        group_mma<BITS>(Q, RB, swz, G, g, tig, b, d1);
        if (two) {
          group_mma<BITS>(P, RB, swz, G2, g, tig, b2, e0);
          group_mma<BITS>(Q, RB, swz, G2, g, tig, b2, e1);
        }
        const float v = mat == 0 ? ((tig & 1) ? d0[2] : d0[0])
                                 : ((tig & 1) ? d1[2] : d1[0]);
        acc = fold(acc, v, SB[G * 32 + sbl], xsum[G], vunit);
        if (two) {
          const float v2 = mat == 0 ? ((tig & 1) ? e0[2] : e0[0])
                                    : ((tig & 1) ? e1[2] : e1[0]);
          acc = fold(acc, v2, SB[G2 * 32 + sbl], xsum[G2], vunit);
        }
      }
    }
    // hand the partial to the epilogue warp (red[st] free once it has
    // consumed the previous tile that used this buffer)
    if (i >= NS) mbar_wait(&redempty[st], ((i / NS) - 1) & 1, a.status);
    red[(st * kNW + cw) * 32 + lane] = acc;
    __syncwarp();
    if (lane == 0) mbar_arrive(&redfull[st]);
    if (i < 6) SLX_TRACE_POINT(0, 3 + 2 * i);
  }
}

// ------------------------------------------------------- phase B kernel ---
//
// Work item = (token, 16 output rows).  Each consumer warp takes two units
// (routed picks j, j+1, or the shared expert) at a time and the 64-column
// groups G = cw, cw+8, ... of both -- independent MMA chains in flight --
// leaving per-warp partial dots in red[item parity].  Warp 0 (which also
// issued the weight copies) then rounds each unit's dot to bf16, weights it
// by its router score and sums over units in unit order: deterministic, and
// off the consumers' critical path.

template <int BITS>
SLX_DEV float down_unit_groups(const uint8_t* S, int in, int cw, int g,
                               int tig, int rrow, const uint32_t* fr,
                               const float* xs) {
  const int nG = tile_ng(in), RB = tile_rb(in, BITS);
  const bool swz = tile_swizzled(in, BITS);
  const uint32_t* SB = reinterpret_cast<const uint32_t*>(S + 16 * RB);
  float acc = 0.f;
  for (int G = cw; G < nG; G += 2 * kNW) {
    const int G2 = G + kNW;
    const bool two = G2 < nG;
    uint32_t b[8], b2[8];
    load_frag(fr, G, tig, b);
    if (two) load_frag(fr, G2, tig, b2);
    float d[4], e[4] = {0.f, 0.f, 0.f, 0.f};
    group_mma<BITS>(S, RB, swz, G, g, tig, b, d);
    if (two) group_mma<BITS>(S, RB, swz, G2, g, tig, b2, e);
    acc = fold(acc, (tig & 1) ? d[2] : d[0], SB[G * 16 + rrow], xs[G],
               kHUnit);
    if (two)
      acc = fold(acc, (tig & 1) ? e[2] : e[0], SB[G2 * 16 + rrow], xs[G2],
                 kHUnit);
  }
  return acc;
}

template <int BITS>
__global__ void __launch_bounds__(kThreads, 2)
    k_down(const __grid_constant__ DownArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int U = a.n_units;
  const int nGr = tile_ng(a.I), nGs = a.Is ? tile_ng(a.Is) : 0;
  const int nGmax = nGr > nGs ? nGr : nGs;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* itemfull = full + kMaxStages;  // [2], count kNW
  uint64_t* itemempty = itemfull + 2;      // [2], count 1
  uint32_t* frag = reinterpret_cast<uint32_t*>(smem + (kMaxStages + 4) * 8);
  float* part = reinterpret_cast<float*>(frag + (size_t)U * nGmax * 32);
  //            ^ [U][nGmax][4], 16-byte aligned (float4 copies)
  float* xsum = part + (size_t)4 * U * nGmax;      // [U][nGmax]
  float* red = xsum + (size_t)U * nGmax;           // [2][kNW][U][16]
  float* ysm = red + (size_t)2 * kNW * U * kRows;  // [U][16]
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(ysm + (size_t)U * kRows) + 127) &
      ~uintptr_t(127));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = a.n_stages;
  const int tph = a.H / kRows;
  const int q_begin = (int)((long long)a.n_items * blockIdx.x / gridDim.x);
  const int q_end = (int)((long long)a.n_items * (blockIdx.x + 1) / gridDim.x);
  const int n_it = q_end - q_begin;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&itemfull[i], kNW);
      mbar_init(&itemempty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();  // the next op waits for this grid to finish

  if (warp == 0) {
    // ------------------------------------------- producer + reduction ---
    // Weights do not depend on phase A, so stream them before it finishes.
    // Request seq = item * U + unit goes to stage seq % NS (NS >= U); lane l
    // of a round issues seq base + l, so one instruction carries up to 32.
    const uint64_t pol = l2_evict_first_policy();
    const int total = n_it * U;
    auto issue = [&](int seq) {
      const int st = seq % NS;
      const int q = q_begin + seq / U, j = seq % U;
      const int token = q / tph, rb = q % tph;
      const bool shared = j >= a.k;
      const int bytes = shared ? a.tile_bytes_sh : a.tile_bytes;
      const uint8_t* src;
      bool valid = true;
      if (!shared) {
        const int slot = lookup_slot(a.ids, token * a.k + j, a.slot_table,
                                     a.n_table, a.n_slots);
        valid = slot >= 0;
        src = a.bank + (size_t)(valid ? slot : 0) * a.slot_stride +
              a.a_bytes + (size_t)rb * a.tile_bytes;
      } else {
        src = a.shared + a.a_bytes_sh + (size_t)rb * a.tile_bytes_sh;
      }
      if (valid) {
        mbar_arrive_expect_tx(&full[st], bytes);
        bulk_g2s(stages + (size_t)st * a.stage_bytes, src, bytes, &full[st], pol);
      } else {
        mbar_arrive(&full[st]);
      }
    };
    const int first = total < NS ? total : NS;
    if (lane == 0) SLX_TRACE_AT(1, 12, globaltimer_ns());
    for (int base = 0; base < first; base += 32)
      if (base + lane < first) issue(base + lane);
    __syncwarp();
    if (lane == 0) SLX_TRACE_AT(1, 13, globaltimer_ns());  // issued
    for (int it = 0; it < n_it; ++it) {
      const int b = it & 1;
      if (!mbar_wait(&itemfull[b], (it >> 1) & 1, a.status)) break;
      // the item's stages are free: issue the requests that reuse them
      const int lo = it * U + NS, hi = (it + 1) * U + NS;
      for (int s0 = lo; s0 < hi && s0 < total; s0 += 32)
        if (s0 + lane < hi && s0 + lane < total) issue(s0 + lane);
      // rounding, score weighting and the combine of item it
      const int q = q_begin + it;
      const int token = q / tph, row0 = (q % tph) * kRows;
      const float* rd = red + (size_t)b * kNW * U * kRows;
      for (int p = lane; p < U * kRows; p += 32) {
        const int j = p / kRows, r = p % kRows;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += rd[((size_t)w * U + j) * kRows + r];
        const bool valid = j >= a.k || lookup_slot(a.ids, token * a.k + j,
                                                   a.slot_table, a.n_table,
                                                   a.n_slots) >= 0;
        const float y = valid ? round_bf16(v) : 0.f;  // gather_qmm: bf16
        if (!a.scores)
          a.out[((size_t)token * a.k + j) * a.H + row0 + r] = f32_to_bf16(y);
        else
          ysm[j * kRows + r] = (j < a.k) ? a.scores[token * a.k + j] * y : y;
      }
      __syncwarp();
      if (a.scores && lane < kRows) {
        float v = 0.f;
        for (int j = 0; j < U; ++j) v += ysm[j * kRows + lane];
        a.out[(size_t)token * a.H + row0 + lane] = f32_to_bf16(v);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&itemempty[b]);
    }
    SLX_TRACE_POINT(1, 14);
    return;
  }

  const int cw = warp - 1, ct = threadIdx.x - 32;
  const int g = lane >> 2, tig = lane & 3;
  const int rrow = g + 8 * (tig & 1);
  SLX_TRACE_POINT(1, 0);
  SLX_TRACE_SMID(1);
  if (a.pdl) pdl_wait_primary();  // the activation fragments come from phase A
  SLX_TRACE_POINT(1, 1);
  int cached_token = -1;
  for (int q = q_begin, it = 0; q < q_end; ++q, ++it) {
    const int token = q / tph;
    if (token != cached_token) {
      // Fragments of every unit's activation were written by phase A; copy
      // them (all loads in flight before any store) and sum the partials.
      named_bar_consumers();
      const int pu = nGmax * 8;  // uint4 per unit in shared memory
      for (int base = ct; base < U * pu; base += 4 * kNW * 32) {
        uint4 v[4];
        int dst[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int p = base + r * kNW * 32;
          const int j = p / pu, o = p % pu;
          dst[r] = -1;
          if (j < U) {
            const bool shared = j >= a.k;
            if (o < (shared ? nGs : nGr) * 8) {
              const uint32_t* src =
                  shared ? a.hfrag_sh + (size_t)token * a.shared_frag_words
                         : a.hfrag + (size_t)(token * a.k + j) * a.unit_frag_words;
              v[r] = reinterpret_cast<const uint4*>(src)[o];
              dst[r] = p;
            }
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (dst[r] >= 0) reinterpret_cast<uint4*>(frag)[dst[r]] = v[r];
      }
      for (int p = ct; p < U * nGmax; p += kNW * 32) {
        const int j = p / nGmax, G = p % nGmax;
        const bool shared = j >= a.k;
        if (G < (shared ? nGs : nGr)) {
          const float* src = shared
              ? a.hpart_sh + (size_t)token * a.shared_part_floats
              : a.hpart + (size_t)(token * a.k + j) * a.unit_part_floats;
          reinterpret_cast<float4*>(part)[p] =
              reinterpret_cast<const float4*>(src)[G];
        }
      }
      named_bar_consumers();
      frag_sums(part, xsum, U * nGmax, ct, kNW * 32);
      named_bar_consumers();
      cached_token = token;
      SLX_TRACE_POINT(1, 2);
    }
    const int b = it & 1;
    if (it >= 2) mbar_wait(&itemempty[b], ((it >> 1) - 1) & 1, a.status);
    float* rd = red + (size_t)b * kNW * U * kRows;
    // every tile of the item was requested long before phase A finished:
    // wait for all of them, then compute the units back to back (no
    // barrier between units, so their loads and MMAs overlap)
    bool ok_all = true;
    for (int j = 0; j < U; ++j)
      ok_all &= mbar_wait(&full[(it * U + j) % NS], ((it * U + j) / NS) & 1,
                          a.status);
    if (it == 0) SLX_TRACE_POINT(1, 8);
    for (int j0 = 0; j0 < U; j0 += 3) {
      float acc[3] = {0.f, 0.f, 0.f};
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int j = j0 + u;
        if (j < U && ok_all)
          acc[u] = down_unit_groups<BITS>(
              stages + (size_t)((it * U + j) % NS) * a.stage_bytes,
              j >= a.k ? a.Is : a.I, cw, g, tig, rrow,
              frag + (size_t)j * nGmax * 32, xsum + (size_t)j * nGmax);
      }
      if (tig < 2) {
#pragma unroll
        for (int u = 0; u < 3; ++u)
          if (j0 + u < U) rd[((size_t)cw * U + j0 + u) * kRows + rrow] = acc[u];
      }
    }
    if (it == 0) SLX_TRACE_POINT(1, 9);
    __syncwarp();
    if (lane == 0) mbar_arrive(&itemfull[b]);
  }
}

// ------------------------------------------------------------ launchers ---

static PerDevice g_num_sms;
static int num_sms() {
  std::atomic<int>& slot = g_num_sms.here();
  int n = slot.load(std::memory_order_relaxed);
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess || n <= 0)
      n = 148;
    slot.store(n, std::memory_order_relaxed);
  }
  return n;
}

// ------------------------------------------------ fused decode SwitchGLU ---
//
// One cooperative launch does both phases for a single token (decode):
//   start   warp 0 requests every gate/up tile and every down tile this CTA
//           will need (one bulk copy each, all in flight at once); the 16
//           compute warps build the activation fragments meanwhile;
//   phase A the compute warps take 64-column groups G = w, w+16, ... of each
//           of the CTA's gate/up tiles; one warp per tile reduces the
//           partials and writes SwiGLU(h) as down-projection fragments;
//   barrier every CTA has written its fragments (grid-wide arrive/wait on a
//           counter in scratch, bounded);
//   phase B the fragments of all units are loaded once, the compute warps
//           take (unit, group) tasks of the CTA's 16-row output items, and
//           one warp per item rounds each unit's rows to bf16, weights them
//           by the router scores and sums the units in order (+ shared).
// Every reduction runs in a fixed order, so results do not depend on timing.

constexpr int kFusedSmemMax = 220 * 1024;
constexpr int kFW = 16;                   // compute warps
constexpr int kFThreads = 32 * (kFW + 1);

// barrier of the fused kernel's compute warps only
SLX_DEV void named_bar_fused() {
  asm volatile("bar.sync 2, %0;" ::"n"(kFW * 32) : "memory");
}
constexpr int kFMaxA = 8;                 // gate/up tiles per CTA
constexpr int kFMaxB = 64;                // down tiles per CTA
constexpr int kFMaxUnits = 64;
constexpr int kFTable = 1024;             // slot tables staged in shared memory

struct FusedArgs {
  GemvArgs a;
  DownArgs d;
  unsigned long long* bar;  // arrival counter (only grows)
  int off_frag, off_part, off_xsum, off_reda, off_stage_a, off_x;
  int off_bfrag, off_bpart, off_bxsum, off_redb, off_stage_b, off_meta;
  int stage_a, stage_b;  // bytes per A / B tile slot
  int bfrag_bulk;        // phase-B fragments by bulk copy
  int b_late;            // down tiles share the gate/up slots: request them
                         // once phase A is done (they load during the barrier)
  // in-kernel slot fill of graph-launched decode (slx_fill_service); off
  // (svc_on = 0) for plain calls
  int svc_on, svc_layer, svc_max_items;
  const int32_t* svc_stamp;
  int32_t* svc_log;
  const int32_t* svc_pred_ids;
  const float* svc_pred_scores;
  int32_t* svc_park;
  const int32_t* svc_release;
  const uint8_t* svc_desc;
  int32_t* svc_go;
  int32_t* svc_table;
  long long svc_wait_ns;
  // expert parallelism (slx_ep_exchange): the per-unit bf16 rows of the
  // units this rank owns go to every rank's receive block, then every CTA
  // counts itself on every rank's counter of this layer; ids without a slot
  // here belong to another rank (not an error)
  int ep_on, ep_rank, ep_nranks, ep_layer, ep_layers;
  const int32_t* ep_stamp;
  uint16_t* ep_recv[SLX_EP_MAX_RANKS];
  unsigned int* ep_count[SLX_EP_MAX_RANKS];
};

SLX_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
SLX_DEV void red_release_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// All CTAs of a cooperative grid; call from one thread after a CTA barrier.
// The counter only grows: a launch's CTAs all read a value inside
// [n * nblocks, (n + 1) * nblocks) on entry (the earlier launches are
// complete), add one each with a release reduction (no reply to wait for,
// unlike a returning atomic), and wait until it reaches (n + 1) * nblocks.
SLX_DEV bool grid_barrier(unsigned long long* cnt, int nblocks,
                          int32_t* status,
                          unsigned long long limit_ns = kWaitLimitNs) {
  const unsigned long long nb = (unsigned long long)nblocks;
  const unsigned long long v = ld_acquire_u64(cnt);
  const unsigned long long target = v - v % nb + nb;
  red_release_add_u64(cnt, 1ull);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; ld_acquire_u64(cnt) < target; ++i) {
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      set_status(status, SLX_ERR_DEVICE_TIMEOUT);
      return false;
    }
    if (i > 4096) __nanosleep(128);   // a long wait (a parked layer) polls gently
  }
  return true;
}

// ------------------------------------------------ in-kernel slot fill ---
//
// slx_fill_service protocol (include/streamlx_cuda.h): the layer record
// goes to the host on entry; a layer with an unmapped routed expert parks
// until the host's copy stream has landed the descriptor, the raw expert
// bytes and the release ticket, then every CTA repacks a share of the
// items into their slots and the new expert -> slot table is installed
// before any weight tile is requested.

SLX_DEV int ld_volatile_s32(const int32_t* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Off the hot path (out of line keeps the decode kernel's code compact: a
// one-CTA-per-SM kernel runs each code line once, so every instruction-cache
// line it touches costs a miss).
__device__ __noinline__ void svc_write_log(const FusedArgs& f, const GemvArgs& a,
                                           int need) {
  volatile int32_t* L = f.svc_log;
  if (!L) return;
  const int stamp = ld_volatile_s32(f.svc_stamp);
  L[1] = need;
  L[2] = a.k;
  for (int j = 0; j < a.k; ++j) {
    L[4 + j] = a.ids[j];
    L[20 + j] = f.svc_pred_ids ? f.svc_pred_ids[j] : -1;
    L[36 + j] = f.svc_pred_scores ? __float_as_int(f.svc_pred_scores[j]) : 0;
  }
  // the stamp last, with release semantics at system scope: a host that
  // sees it sees the words above (one writer; the host reads in order)
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(f.svc_log), "r"(stamp)
               : "memory");
}

// Every thread of every CTA calls this after the CTA agreed that some routed
// id of this launch has no slot.
template <int BITS>
__device__ __noinline__ void svc_fill(const FusedArgs& f, const GemvArgs& a) {
  __shared__ int s_ok;
  __shared__ __align__(16) slx_fill_item s_item;
  __shared__ int s_nitems;
  const int stamp = ld_volatile_s32(f.svc_stamp);
  const int ticket = (int)(((unsigned)stamp << 8) | (unsigned)f.svc_layer);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    volatile int32_t* P = f.svc_park;
    P[1] = f.svc_layer;
    P[2] = stamp;
    __threadfence_system();
    P[0] = ticket;
    __threadfence_system();
    const uint64_t t0 = globaltimer_ns();
    int v = 0;
    for (uint32_t i = 0;; ++i) {
      v = ld_volatile_s32(f.svc_release);
      if (v == ticket || v == -ticket) break;
      if ((i & 15u) == 0 && globaltimer_ns() - t0 > (uint64_t)f.svc_wait_ns) {
        v = 0;
        break;
      }
      __nanosleep(256);
    }
    *reinterpret_cast<volatile int32_t*>(f.svc_go) = v == ticket ? ticket : -ticket;
    if (v != ticket)
      set_status(a.status, v == 0 ? SLX_ERR_DEVICE_TIMEOUT : SLX_ERR_UNMAPPED_EXPERT);
  }
  __syncthreads();
  // every CTA arrives at once; CTA 0 only after the release (or timeout)
  if (threadIdx.x == 0) {
    grid_barrier(f.bar, gridDim.x, a.status,
                 (unsigned long long)f.svc_wait_ns + kWaitLimitNs);
    s_ok = ld_volatile_s32(f.svc_go) == ticket;
    s_nitems = 0;
    if (s_ok) {
      const slx_fill_header* h =
          reinterpret_cast<const slx_fill_header*>(f.svc_desc);
      const int n = __ldcg(&h->n_items);
      if (__ldcg(&h->ticket) != ticket || __ldcg(&h->layer) != f.svc_layer ||
          n < 0 || n > f.svc_max_items || __ldcg(&h->n_table) != a.n_table) {
        set_status(a.status, SLX_ERR_INVALID);
        s_ok = 0;
      } else {
        s_nitems = n;
      }
    }
  }
  __syncthreads();
  if (s_ok) {
    const int H = a.in, I = a.I;
    const int na = I / 16, tpe = na + H / 16;
    const slx_fill_item* items = reinterpret_cast<const slx_fill_item*>(
        f.svc_desc + sizeof(slx_fill_header));
    const int32_t* tab = reinterpret_cast<const int32_t*>(
        f.svc_desc + sizeof(slx_fill_header) +
        (size_t)f.svc_max_items * sizeof(slx_fill_item));
    const int jobs = s_nitems * tpe;
    for (int job = blockIdx.x; job < jobs; job += gridDim.x) {
      const int it = job / tpe, t = job % tpe;
      if (threadIdx.x < (int)(sizeof(slx_fill_item) / 16))
        reinterpret_cast<uint4*>(&s_item)[threadIdx.x] =
            __ldcg(reinterpret_cast<const uint4*>(items + it) + threadIdx.x);
      __syncthreads();
      bool good = s_item.slot >= 0 && s_item.slot < a.n_slots;
      for (int p = 0; p < 9; ++p)
        good &= s_item.part[p] != nullptr &&
                (reinterpret_cast<uintptr_t>(s_item.part[p]) & 15u) == 0;
      if (good) {
        uint8_t* dst = const_cast<uint8_t*>(a.bank) +
                       (size_t)s_item.slot * a.slot_stride;
        const QSrc G = {(const uint8_t*)s_item.part[0],
                        (const uint16_t*)s_item.part[1],
                        (const uint16_t*)s_item.part[2]};
        const QSrc U = {(const uint8_t*)s_item.part[3],
                        (const uint16_t*)s_item.part[4],
                        (const uint16_t*)s_item.part[5]};
        const QSrc D = {(const uint8_t*)s_item.part[6],
                        (const uint16_t*)s_item.part[7],
                        (const uint16_t*)s_item.part[8]};
        if (t < na)
          pack_pair(dst + (size_t)t * pair_tile_bytes(H, BITS), G, 16 * t, U,
                    16 * t, I, H, BITS);
        else
          pack_single(dst + expert_a_bytes(H, I, BITS) +
                          (size_t)(t - na) * single_tile_bytes(I, BITS),
                      D, 16 * (t - na), I, BITS);
      } else if (threadIdx.x == 0 && t == 0) {
        set_status(a.status, SLX_ERR_INVALID);
      }
      __syncthreads();  // s_item is reused by the next job
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n_table;
         i += gridDim.x * blockDim.x)
      f.svc_table[i] = __ldcg(tab + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) grid_barrier(f.bar, gridDim.x, a.status);
  __syncthreads();
  // the slots were written through the generic proxy; the weight tiles are
  // read by bulk copies (async proxy)
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Up to four 64-column groups G0..G0+n-1 of a 16-row down tile, folded in
// group order: per-row partial (lanes with tig < 2 hold rows g and g + 8).
// The groups' fragment loads and MMAs are independent, so they overlap.
template <int BITS>
SLX_DEV float down_quad(const uint8_t* S, int in, int G0, int n, int g,
                        int tig, int rrow, const uint32_t* fr, const float* xs) {
  const int RB = tile_rb(in, BITS);
  const bool swz = tile_swizzled(in, BITS);
  const uint32_t* SB = reinterpret_cast<const uint32_t*>(S + 16 * RB);
  // groups past the unit's last one (n < 4) repeat its last group, weight 0
  int G[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) G[q] = G0 + (q < n ? q : n - 1);
  uint32_t b[4][8];
  float dd[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) load_frag(fr, G[q], tig, b[q]);
#pragma unroll
  for (int q = 0; q < 4; ++q) group_mma<BITS>(S, RB, swz, G[q], g, tig, b[q], dd[q]);
  float acc = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float a = fold(acc, (tig & 1) ? dd[q][2] : dd[q][0], SB[G[q] * 16 + rrow],
                         xs[G[q]], kHUnit);
    acc = q < n ? a : acc;
  }
  return acc;
}

// gemv_issue in pieces of about kBulkPiece bytes: the copy engine keeps
// several bulk copies in flight per SM, so a few medium copies stream from
// DRAM faster than one large one (measured: 24 MB over 148 SMs in 25.6 KB
// copies ~3.6 TB/s, in 12.8 KB copies ~4.7 TB/s).
constexpr int kBulkPiece = 12800;
SLX_DEV void issue_pieces(const uint8_t* src, uint8_t* dst, int bytes,
                          uint64_t* bar, uint64_t pol) {
  mbar_arrive_expect_tx(bar, bytes);
  const int n = (bytes + kBulkPiece - 1) / kBulkPiece;
  const int piece = ((bytes + n - 1) / n + 15) & ~15;
  for (int o = 0; o < bytes; o += piece)
    bulk_g2s(dst + o, src + o, bytes - o < piece ? bytes - o : piece, bar, pol);
}

// Tile q of a one-token launch, with the routed units' slots already looked
// up (slot[u] < 0: no slot).
SLX_DEV TileInfo fused_tile(const GemvArgs& a, int q, const int* slot) {
  TileInfo t{};
  const int tpu = a.I / kRows;
  const int routed = a.k * tpu;
  if (q < routed) {
    const int u = q / tpu, s = slot[u];
    t.valid = t.valid1 = s >= 0;
    t.unit = u;
    t.ti = q % tpu;
    t.src = a.bank + (size_t)(s < 0 ? 0 : s) * a.slot_stride +
            (size_t)t.ti * a.tile_bytes;
    return t;
  }
  t.valid = t.valid1 = 1;
  t.unit = -1;  // the token's shared expert
  t.ti = q - routed;
  t.src = a.shared + (size_t)t.ti * a.tile_bytes;
  return t;
}

// Rows row0..row0+15 of unit j (lanes 0..15 hold them) into the receive
// block of this step and layer: a routed unit to every rank, the shared
// expert (unit k, computed by every rank) to this rank only.
__device__ __noinline__ void ep_write_rows(const FusedArgs& f, const DownArgs& d, int j,
                           int row0, float y, int lane) {
  const uint32_t b = lane < kRows ? (uint32_t)f32_to_bf16(y) : 0u;
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int src = (lane & 1) * 8 + 2 * q;
    const uint32_t lo = __shfl_sync(0xffffffffu, b, src);
    const uint32_t hi = __shfl_sync(0xffffffffu, b, src + 1);
    w[q] = lo | (hi << 16);
  }
  if (lane >= 2) return;
  const int stamp = *f.ep_stamp;
  const size_t block = ((size_t)(stamp & 1) * f.ep_layers + f.ep_layer) *
                       (size_t)(d.k + 1) * d.H;
  const size_t off = block + (size_t)j * d.H + row0 + 8 * lane;
  const uint4 v = make_uint4(w[0], w[1], w[2], w[3]);
  if (j >= d.k) {
    *reinterpret_cast<uint4*>(f.ep_recv[f.ep_rank] + off) = v;
    return;
  }
  for (int r = 0; r < f.ep_nranks; ++r)
    *reinterpret_cast<uint4*>(f.ep_recv[r] + off) = v;
}

// This CTA's rows are written (every thread's stores are ordered before
// thread 0's by the preceding barrier, and a release is cumulative over
// them): count the CTA on every rank.
SLX_DEV void ep_signal(const FusedArgs& f) {
  if (threadIdx.x != 0) return;
  const int stamp = *f.ep_stamp;
  const int slot = (stamp & 1) * f.ep_layers + f.ep_layer;
  for (int r = 0; r < f.ep_nranks; ++r)
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(
                     f.ep_count[r] + slot)
                 : "memory");
}

// Phase-B fragments of the units a CTA touches, by plain loads (when the
// units' rows do not line up for one bulk copy).  Every thread calls this.
__device__ __noinline__ void load_bfrag_lsu(const DownArgs& d, uint32_t* bfrag,
                                            float* bpart, int U, int nGmax,
                                            int nGr, int nGs, int qb0, int nbt) {
  const int w0 = qb0 % U;
  auto touched = [&](int j) { return nbt >= U || (j - w0 + U) % U < nbt; };
  const int pu = nGmax * 8;  // uint4 per unit
  const int total = U * pu;
  const int totp = U * nGmax;  // float4 partial sums
  uint4* bf4 = reinterpret_cast<uint4*>(bfrag);
  auto part_of = [&](int q) {
    const int j = q / nGmax, G = q % nGmax;
    const bool sh = j >= d.k;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (touched(j) && G < (sh ? nGs : nGr))
      v = __ldcg(reinterpret_cast<const float4*>(
                     sh ? d.hpart_sh : d.hpart + (size_t)j * d.unit_part_floats) +
                 G);
    return v;
  };
  // the fragments and (in the first round) the partial sums in one round
  // of loads per thread
  for (int base = threadIdx.x, it = 0; base < total || it == 0;
       base += 4 * kFThreads, ++it) {
    uint4 v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int p = base + r * kFThreads;
      v[r] = make_uint4(0u, 0u, 0u, 0u);
      if (p < total) {
        const int j = p / pu, o = p % pu;
        const bool sh = j >= d.k;
        if (touched(j) && o < (sh ? nGs : nGr) * 8)
          v[r] = __ldcg(reinterpret_cast<const uint4*>(
                            sh ? d.hfrag_sh : d.hfrag + (size_t)j * d.unit_frag_words) +
                        o);
      }
    }
    float4 pv = make_float4(0.f, 0.f, 0.f, 0.f);
    const bool has_p = it == 0 && (int)threadIdx.x < totp;
    if (has_p) pv = part_of(threadIdx.x);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int p = base + r * kFThreads;
      if (p < total) bf4[p] = v[r];
    }
    if (has_p) reinterpret_cast<float4*>(bpart)[threadIdx.x] = pv;
  }
  for (int q = threadIdx.x + kFThreads; q < totp; q += kFThreads)
    reinterpret_cast<float4*>(bpart)[q] = part_of(q);
}

template <int BITS>
__global__ void __launch_bounds__(kFThreads, 1)
    k_switchglu_fused(const __grid_constant__ FusedArgs f) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvArgs& a = f.a;
  const DownArgs& d = f.d;
  uint64_t* fullA = reinterpret_cast<uint64_t*>(smem);
  uint64_t* fullB = fullA + kFMaxA;
  uint64_t* fullX = fullB + kFMaxB;  // the token's activations
  uint64_t* fullF = fullX + 1;       // phase-B fragments
  uint32_t* frag = reinterpret_cast<uint32_t*>(smem + f.off_frag);
  float* part = reinterpret_cast<float*>(smem + f.off_part);
  float* xsum = reinterpret_cast<float*>(smem + f.off_xsum);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + f.off_x);
  float* redA = reinterpret_cast<float*>(smem + f.off_reda);  // [na][kFW][32]
  uint8_t* stA = smem + f.off_stage_a;
  uint32_t* bfrag = reinterpret_cast<uint32_t*>(smem + f.off_bfrag);
  float* bpart = reinterpret_cast<float*>(smem + f.off_bpart);
  float* bxsum = reinterpret_cast<float*>(smem + f.off_bxsum);
  float* redB = reinterpret_cast<float*>(smem + f.off_redb);  // [tiles][nq][16]
  uint8_t* stB = smem + f.off_stage_b;
  int* meta = reinterpret_cast<int*>(smem + f.off_meta);      // A tile valid + unit valid
  __shared__ float s_vmax[kFW];
  __shared__ float s_vunit;
  __shared__ int s_slot[kFMaxUnits];
  __shared__ int s_table[kFTable];
  __shared__ float s_score[kFMaxUnits];  // combine weight per unit (shared: 1)
  __shared__ int s_need;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G_ = gridDim.x, bid = blockIdx.x;
  const int nG = tile_ng(a.in);
  const int RB = tile_rb(a.in, BITS);
  const bool swz = tile_swizzled(a.in, BITS);
  const int qa0 = (int)((long long)a.n_tiles * bid / G_);
  const int na = (int)((long long)a.n_tiles * (bid + 1) / G_) - qa0;
  const int U = d.n_units;
  // phase B: whole 16-row items per CTA (an item's units combine in the
  // CTA that computed them), item-major tiles [qb0, qb0 + nbt)
  const int it0 = (int)((long long)d.n_items * bid / G_);
  const int qb0 = it0 * U;
  const int nbt = ((int)((long long)d.n_items * (bid + 1) / G_) - it0) * U;
  const int nGr = tile_ng(d.I), nGs = d.Is ? tile_ng(d.Is) : 0;
  const int nGmax = nGr > nGs ? nGr : nGs;
  const int nq = (nGmax + 3) >> 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kFMaxA; ++i) mbar_init(&fullA[i], 1);
    for (int i = 0; i < kFMaxB; ++i) mbar_init(&fullB[i], 1);
    mbar_init(fullX, 1);
    mbar_init(fullF, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait_primary();
  SLX_TRACE_POINT(0, 0);
  SLX_TRACE_SMID(0);
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(fullX, a.in * 2);
    bulk_g2s_plain(xs, a.x, a.in * 2, fullX);
  }

  // slots of the routed experts, one lane each; s_need: one has none
  // the expert -> slot table comes in whole, beside the ids (one L2 round
  // trip for both instead of ids, then table entries)
  const bool tab_smem = a.slot_table && a.n_table <= kFTable;
  auto lookup_slots = [&]() {
    if (tab_smem && warp > 0)
      for (int e = threadIdx.x - 32; e < a.n_table; e += kFW * 32)
        s_table[e] = __ldcg(a.slot_table + e);
    int e_id = -1;
    if (warp == 0 && lane < a.k) e_id = a.ids[lane];
    __syncthreads();
    if (warp == 0) {
      unsigned miss = 0u;
      for (int j0 = 0; j0 < a.k; j0 += 32) {
        const int j = j0 + lane;
        int sl = -1;
        if (j < a.k) {
          if (tab_smem) {
            const int e = j0 == 0 ? e_id : a.ids[j];
            sl = (e >= 0 && e < a.n_table) ? s_table[e] : -1;
            if (sl >= a.n_slots) sl = -1;
          } else {
            sl = lookup_slot(a.ids, j, a.slot_table, a.n_table, a.n_slots);
          }
          s_slot[j] = sl;
        }
        miss |= __ballot_sync(0xffffffffu, j < a.k && sl < 0);
      }
      if (lane == 0) s_need = miss != 0u;
    }
    __syncthreads();
  };
  lookup_slots();
  if (threadIdx.x == 0) SLX_TRACE_AT(1, 12, globaltimer_ns());
  // the layer record for the host: before a park (the host serves from it),
  // else after this CTA's copies are requested (a system-scope store costs
  // a host round trip)
  const bool log_late = f.svc_on && !s_need;
  if (f.svc_on && s_need) {  // the same verdict in every CTA (same ids, same table)
    if (bid == 0 && threadIdx.x == 0) svc_write_log(f, a, 1);
    svc_fill<BITS>(f, a);
    lookup_slots();
  }

  // source of this CTA's down tile s (null: the unit has no slot)
  auto b_src = [&](int s, int& bytes) -> const uint8_t* {
    const int sg = qb0 + s, item = sg / U, j = sg % U;
    if (j >= d.k) {
      bytes = d.tile_bytes_sh;
      return d.shared + d.a_bytes_sh + (size_t)item * d.tile_bytes_sh;
    }
    bytes = d.tile_bytes;
    const int slot = s_slot[j];
    if (slot < 0) return nullptr;
    return d.bank + (size_t)slot * d.slot_stride + d.a_bytes +
           (size_t)item * d.tile_bytes;
  };
  auto issue_b = [&]() {
    const uint64_t pol = l2_evict_first_policy();
    for (int s = lane; s < nbt; s += 32) {
      int bytes = 0;
      const uint8_t* src = b_src(s, bytes);
      if (src) {
        mbar_arrive_expect_tx(&fullB[s], bytes);
        bulk_g2s(stB + (size_t)s * f.stage_b, src, bytes, &fullB[s], pol);
      } else {
        mbar_arrive(&fullB[s]);
      }
    }
  };
  if (warp == 0) {
    // ---- every weight request of this CTA, up front ----
    const uint64_t pol = l2_evict_first_policy();
    if (lane < na) {
      const TileInfo t = fused_tile(a, qa0 + lane, s_slot);
      meta[lane] = t.valid;
      if (!t.valid && !f.ep_on) set_status(a.status, SLX_ERR_UNMAPPED_EXPERT);
      if (t.valid)
        issue_pieces(t.src, stA + (size_t)lane * f.stage_a, a.tile_bytes, &fullA[lane], pol);
      else
        mbar_arrive(&fullA[lane]);
    }
    if (!f.b_late) {
      issue_b();
    }
    if (lane == 0) SLX_TRACE_AT(1, 13, globaltimer_ns());
    // after every request (each copy instruction orders after the memory
    // operations before it): the units' validity and combine weights, read
    // in phase B, and the host record
    for (int j = lane; j < U; j += 32) {
      meta[kFMaxA + j] = j >= d.k || s_slot[j] >= 0;
      s_score[j] = (d.scores && j < d.k) ? d.scores[j] : 1.f;
    }
    if (log_late && bid == 0 && lane == 0) svc_write_log(f, a, 0);
    if (f.b_late) {
      // the down tiles share the gate/up stages: once this CTA's gate/up
      // bytes are in, start the down tiles' DRAM reads into L2 (they land
      // during the epilogue and the grid barrier); the copies into shared
      // memory follow once phase A is done
      if (na > 0) mbar_wait(&fullA[na - 1], 0, a.status);
      for (int s = lane; s < nbt; s += 32) {
        int bytes = 0;
        const uint8_t* src = b_src(s, bytes);
        if (src) bulk_prefetch_l2(src, bytes);
      }
    }
  } else {
    // ---- activation fragments of the token (per-token scale first) ----
    const int ct = threadIdx.x - 32;
    mbar_wait(fullX, 0, a.status);
    SLX_TRACE_POINT(1, 14);
    const float m = absmax_part(xs, a.in, ct, kFW * 32);
    if (lane == 0) s_vmax[warp - 1] = m;
    named_bar_fused();
    float mm = 0.f;
    for (int w = 0; w < kFW; ++w) mm = fmaxf(mm, s_vmax[w]);
    const int ve = vec_exp(mm);
    if (ct == 0) s_vunit = pow2f(24 - ve);
    for (int p = ct; p < 4 * nG; p += kFW * 32)
      frag_task<BITS>(xs, p >> 2, p & 3, frag, part, a.status, pow2f(ve));
    // the compute warps only: phase A need not wait for warp 0's requests
    named_bar_fused();
    frag_sums(part, xsum, nG, ct, kFW * 32);
    named_bar_fused();
  }
  SLX_TRACE_POINT(0, 1);

  // ---- phase A: gate/up groups ----
  if (warp > 0) {
    const float vunit = s_vunit;
    const int cw = warp - 1;
    const int g = lane >> 2, tig = lane & 3;
    const int mat = tig >> 1;
    const int sbl = mat * 16 + g + 8 * (tig & 1);
#ifdef SLX_TRACE
    int tr_seen = 0;
#endif
    for (int i = 0; i < na; ++i) {
      const bool ok = mbar_wait(&fullA[i], 0, a.status);
      if (i < 3) SLX_TRACE_POINT(0, 2 + i);
#ifdef SLX_TRACE
      if (threadIdx.x == 32 && nbt > 0 && !f.b_late) {
        if (!(tr_seen & 1) && mbar_try_wait(&fullB[0], 0)) { SLX_TRACE_POINT(1, 8); tr_seen |= 1; }
        if (!(tr_seen & 2) && mbar_try_wait(&fullB[nbt - 1], 0)) { SLX_TRACE_POINT(1, 9); tr_seen |= 2; }
      }
#endif
      const uint8_t* S = stA + (size_t)i * f.stage_a;
      float acc = 0.f;
      if (ok && meta[i]) {
        const uint8_t* P = S;
        const uint8_t* Q = S + 16 * RB;
        const uint32_t* SB = reinterpret_cast<const uint32_t*>(S + 32 * RB);
        for (int G = cw; G < nG; G += 2 * kFW) {
          const int G2 = G + kFW;
          const bool two = G2 < nG;
          uint32_t b[8], b2[8];
          load_frag(frag, G, tig, b);
          if (two) load_frag(frag, G2, tig, b2);
          float d0[4], d1[4];
          float e0[4] = {0.f, 0.f, 0.f, 0.f}, e1[4] = {0.f, 0.f, 0.f, 0.f};
          group_mma<BITS>(P, RB, swz, G, g, tig, b, d0);
          group_mma<BITS>(Q, RB, swz, G, g, tig, b, d1);
          if (two) {
            group_mma<BITS>(P, RB, swz, G2, g, tig, b2, e0);
            group_mma<BITS>(Q, RB, swz, G2, g, tig, b2, e1);
          }
          const float v = mat == 0 ? ((tig & 1) ? d0[2] : d0[0])
                                   : ((tig & 1) ? d1[2] : d1[0]);
          acc = fold(acc, v, SB[G * 32 + sbl], xsum[G], vunit);
          if (two) {
            const float v2 = mat == 0 ? ((tig & 1) ? e0[2] : e0[0])
                                      : ((tig & 1) ? e1[2] : e1[0]);
            acc = fold(acc, v2, SB[G2 * 32 + sbl], xsum[G2], vunit);
          }
        }
      }
      redA[((size_t)i * kFW + cw) * 32 + lane] = acc;
    }
  }
  __syncthreads();
  SLX_TRACE_POINT(0, 5);
  // one warp per tile: reduce the 16 partials, SwiGLU, write fragments
  if (warp > 0 && warp - 1 < na) {
    const int i = warp - 1;
    TileInfo t = fused_tile(a, qa0 + i, s_slot);
    t.valid = t.valid1 = meta[i];
    gemv_epilogue<BITS, kFW>(a, t, redA + (size_t)i * kFW * 32, lane);
  }
  if (warp == 0 && f.b_late) issue_b();  // the A stages are free now
  // the SwiGLU fragments are read by other CTAs' bulk copies
  fence_proxy_async_global();
  __syncthreads();
  SLX_TRACE_POINT(0, 6);
#ifdef SLX_TRACE
  if (threadIdx.x == 32 && nbt > 0 && !f.b_late) {
    if (mbar_try_wait(&fullB[nbt - 1], 0)) SLX_TRACE_POINT(1, 10);
    else SLX_TRACE_POINT(1, 11);
  }
#endif
  if (threadIdx.x == 0) grid_barrier(f.bar, G_, a.status);
  __syncthreads();
  SLX_TRACE_POINT(0, 7);
  pdl_launch_dependents();
  if (nbt == 0) {
    if (f.ep_on) ep_signal(f);
    return;
  }

  // ---- phase B: fragments of the units (bulk copies from L2) ----
  if (f.bfrag_bulk) {
    if (threadIdx.x == 0) {
      fence_proxy_async_global();
      const uint32_t fr = (uint32_t)d.k * nGr * 128, pr = (uint32_t)d.k * nGr * 16;
      const uint32_t fs = (uint32_t)nGs * 128, ps = (uint32_t)nGs * 16;
      mbar_arrive_expect_tx(fullF, fr + pr + fs + ps);
      bulk_g2s_plain(bfrag, d.hfrag, fr, fullF);
      bulk_g2s_plain(bpart, d.hpart, pr, fullF);
      if (fs) {
        bulk_g2s_plain(bfrag + (size_t)d.k * nGmax * 32, d.hfrag_sh, fs, fullF);
        bulk_g2s_plain(bpart + (size_t)d.k * nGmax * 4, d.hpart_sh, ps, fullF);
      }
    }
    mbar_wait(fullF, 0, d.status);
    SLX_TRACE_POINT(1, 0);
  } else {
    load_bfrag_lsu(d, bfrag, bpart, U, nGmax, nGr, nGs, qb0, nbt);
    SLX_TRACE_POINT(1, 1);
  }
  __syncthreads();
  SLX_TRACE_POINT(1, 2);
  frag_sums(bpart, bxsum, U * nGmax, threadIdx.x, kFThreads);
  __syncthreads();
  SLX_TRACE_POINT(0, 8);
  // ---- phase B: (tile, group quad) tasks ----
  if (warp > 0) {
    const int cw = warp - 1;
    const int g = lane >> 2, tig = lane & 3;
    const int rrow = g + 8 * (tig & 1);
    const int ntask = nbt * nq;
    for (int task = cw; task < ntask; task += kFW) {
      const int s = task / nq, gq = task % nq;
      const int j = (qb0 + s) % U;
      const int in = j >= d.k ? d.Is : d.I;
      const int ng = tile_ng(in);
      const int G0 = 4 * gq;
      const bool ok = mbar_wait(&fullB[s], 0, d.status);
      if (task == cw) SLX_TRACE_POINT(0, 11);
      float v = 0.f;
      if (G0 < ng && ok && meta[kFMaxA + j])
        v = down_quad<BITS>(stB + (size_t)s * f.stage_b, in, G0,
                            ng - G0 < 4 ? ng - G0 : 4, g, tig, rrow,
                            bfrag + (size_t)j * nGmax * 32,
                            bxsum + (size_t)j * nGmax);
      if (tig < 2) redB[((size_t)s * nq + gq) * kRows + rrow] = v;
      if (task == cw) SLX_TRACE_POINT(1, 3);
    }
    SLX_TRACE_POINT(1, 4);
  }
  __syncthreads();
  SLX_TRACE_POINT(0, 9);
  // ---- per item: bf16 per unit, score weights, combine in unit order ----
  const int i_first = qb0 / U, i_last = (qb0 + nbt - 1) / U;
  for (int i = i_first + warp; i <= i_last; i += kFW + 1) {
    const int row0 = i * kRows;
    auto unit_y = [&](int j) {  // lane < 16: row lane of unit j
      const int s = i * U + j - qb0;
      float v = 0.f;
      if (lane < kRows)
        for (int gq = 0; gq < nq; ++gq) v += redB[((size_t)s * nq + gq) * kRows + lane];
      return meta[kFMaxA + j] ? round_bf16(v) : 0.f;
    };
    if (f.ep_on) {
      for (int j = 0; j < U; ++j)
        if (meta[kFMaxA + j]) ep_write_rows(f, d, j, row0, unit_y(j), lane);
      continue;
    }
    if (!d.scores) {
      for (int j = 0; j < U; ++j) {
        const float y = unit_y(j);
        if (lane < kRows) d.out[(size_t)j * d.H + row0 + lane] = f32_to_bf16(y);
      }
      continue;
    }
    float y_out = 0.f;  // lane < 16: row lane
    for (int j = 0; j < U; ++j) {
      const float y = unit_y(j);
      y_out = (j < d.k) ? fmaf(s_score[j], y, y_out) : y_out + y;
    }
    if (lane < kRows) d.out[row0 + lane] = f32_to_bf16(y_out);
  }
  if (f.ep_on) {
    __syncthreads();
    ep_signal(f);
  }
  SLX_TRACE_POINT(0, 10);
}

// Shared-memory layout of the fused kernel for one problem, or 0 if it
// does not fit one CTA per SM.  Preferred: gate/up stages and down stages
// side by side (every copy requested at the start), the phase-B fragments
// reusing the gate/up stages; else the down tiles reuse the gate/up stages
// once phase A is done (b_late), their DRAM reads started as L2 prefetches.
template <int BITS>
static int fused_layout(FusedArgs& f, int grid) {
  const GemvArgs& a = f.a;
  const DownArgs& d = f.d;
  const int nG = tile_ng(a.in);
  const int U = d.n_units;
  const int na_max = (a.n_tiles + grid - 1) / grid;
  const int nb_max = (d.n_items + grid - 1) / grid * U;
  if (na_max > kFMaxA || nb_max > kFMaxB || U > kFMaxUnits || a.k > kFMaxUnits)
    return 0;
  const int nGr = tile_ng(d.I), nGs = d.Is ? tile_ng(d.Is) : 0;
  const int nGmax = nGr > nGs ? nGr : nGs;
  const int nq = (nGmax + 3) / 4;
  auto al = [](int v) { return (v + 127) & ~127; };
  int o = (kFMaxA + kFMaxB + 2) * 8;
  o = al(o); f.off_x = o;       o += a.in * 2;
  o = al(o); f.off_frag = o;    o += nG * 32 * 4;
  o = al(o); f.off_part = o;    o += nG * 4 * 4;
  o = al(o); f.off_xsum = o;    o += nG * 4;
  o = al(o); f.off_reda = o;    o += na_max * kFW * 32 * 4;
  o = al(o); f.off_meta = o;    o += (kFMaxA + kFMaxUnits) * 4;
  o = al(o); f.off_redb = o;    o += nb_max * nq * kRows * 4;
  const int bf = al(U * nGmax * 32 * 4), bp = al(U * nGmax * 4 * 4),
            bx = al(U * nGmax * 4);
  f.stage_a = al((int)pair_tile_bytes(a.in, BITS));
  const int tb = d.tile_bytes > d.tile_bytes_sh ? d.tile_bytes : d.tile_bytes_sh;
  f.stage_b = al(tb);
  const int bytes_a = na_max * f.stage_a, bytes_b = nb_max * f.stage_b;
  // the routed units' SwiGLU fragments arrive in one bulk copy when their
  // rows have the fragment buffer's stride
  f.bfrag_bulk = nGr == nGmax && d.unit_frag_words == nGr * 32 &&
                 d.unit_part_floats == nGr * 4;
  o = al(o);
  if (bf + bp + bx <= bytes_a && o + bytes_a + bytes_b <= kFusedSmemMax) {
    f.b_late = 0;
    f.off_stage_a = o;
    f.off_bfrag = o;
    f.off_bpart = o + bf;
    f.off_bxsum = o + bf + bp;
    f.off_stage_b = o + bytes_a;
    return o + bytes_a + bytes_b;
  }
  f.off_bfrag = o;
  f.off_bpart = o + bf;
  f.off_bxsum = o + bf + bp;
  o += bf + bp + bx;
  f.off_stage_a = o;
  if (o + bytes_a + bytes_b <= kFusedSmemMax) {
    f.b_late = 0;
    f.off_stage_b = o + bytes_a;
    return o + bytes_a + bytes_b;
  }
  f.b_late = 1;
  f.off_stage_b = o;
  return o + (bytes_a > bytes_b ? bytes_a : bytes_b);
}

template <int BITS>
static int launch_fused_t(FusedArgs f, cudaStream_t stream) {
  static PerDevice grid_of;  // grid + 1 per device (1: cannot run)
  std::atomic<int>& gslot = grid_of.here();
  int max_grid = gslot.load(std::memory_order_relaxed) - 1;
  if (max_grid < 0) {
    int per_sm = 0;
    if (cudaFuncSetAttribute(k_switchglu_fused<BITS>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kFusedSmemMax) != cudaSuccess)
      return SLX_ERR_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, k_switchglu_fused<BITS>, kFThreads, kFusedSmemMax) !=
        cudaSuccess)
      return SLX_ERR_CUDA;
    max_grid = per_sm >= 1 ? num_sms() : 0;
    gslot.store(max_grid + 1, std::memory_order_relaxed);
  }
  if (max_grid <= 0) return SLX_ERR_UNSUPPORTED;
  const int grid = max_grid;
  const int bytes = fused_layout<BITS>(f, grid);
  if (bytes <= 0 || bytes > kFusedSmemMax) return SLX_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  // as a PDL secondary the launch's set-up overlaps the preceding kernel;
  // the kernel waits (griddepcontrol.wait) before it reads anything
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  static PerDevice pdl_refused;  // set if the driver refuses the combination
  std::atomic<int>& pslot = pdl_refused.here();
  cfg.numAttrs = (!pslot.load(std::memory_order_relaxed) && pdl_enabled()) ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_switchglu_fused<BITS>, f);
  if (e != cudaSuccess && cfg.numAttrs == 2) {
    (void)cudaGetLastError();
    pslot.store(1, std::memory_order_relaxed);
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_switchglu_fused<BITS>, f);
  }
  return e == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_switchglu_fused(const GemvArgs& a, const DownArgs& d, void* bar,
                           int bits, cudaStream_t stream,
                           const slx_fill_service* svc,
                           const slx_ep_exchange* ep) {
  if (a.T != 1 || d.T != 1) return SLX_ERR_UNSUPPORTED;
  FusedArgs f = {};
  f.a = a;
  f.d = d;
  f.bar = reinterpret_cast<unsigned long long*>(bar);
  if (ep) {
    f.ep_on = 1;
    f.ep_rank = ep->rank;
    f.ep_nranks = ep->n_ranks;
    f.ep_layer = ep->layer;
    f.ep_layers = ep->n_layers;
    f.ep_stamp = ep->stamp;
    for (int r = 0; r < ep->n_ranks; ++r) {
      f.ep_recv[r] = reinterpret_cast<uint16_t*>(ep->recv[r]);
      f.ep_count[r] = ep->count[r];
    }
  }
  if (svc) {
    f.svc_on = 1;
    f.svc_layer = svc->layer;
    f.svc_max_items = svc->max_items;
    f.svc_stamp = svc->stamp;
    f.svc_log = svc->log;
    f.svc_pred_ids = svc->pred_ids;
    f.svc_pred_scores = svc->pred_scores;
    f.svc_park = svc->park;
    f.svc_release = svc->release;
    f.svc_desc = reinterpret_cast<const uint8_t*>(svc->desc);
    f.svc_go = svc->go;
    f.svc_table = const_cast<int32_t*>(a.slot_table);
    f.svc_wait_ns = (long long)svc->wait_ns;
  }
  switch (bits) {
    case 2: f.a.tile_bytes = (int)pair_tile_bytes(a.in, 2); break;
    case 4: f.a.tile_bytes = (int)pair_tile_bytes(a.in, 4); break;
    case 8: f.a.tile_bytes = (int)pair_tile_bytes(a.in, 8); break;
    default: return SLX_ERR_UNSUPPORTED;
  }
  switch (bits) {
    case 2: return launch_fused_t<2>(f, stream);
    case 4: return launch_fused_t<4>(f, stream);
    default: return launch_fused_t<8>(f, stream);
  }
}

// Phase A and phase B each request exactly kSmemTarget bytes: one CTA of
// each fits on an SM (2 x 113 KB + 2 x 1 KB reserved = the full 228 KB), and
// -- because two CTAs of either kernel alone also need the full carve-out --
// both kernels run with the same shared-memory configuration.  An SM must
// drain to change configuration, so matching them is what lets the PDL
// secondary start beside a running primary.
constexpr int kSmemTarget = 113 * 1024;
constexpr int kSmemBudget = kSmemTarget;
constexpr int kSmemMax = 227 * 1024;

// Raise the kernel's dynamic shared-memory limit once per instantiation and
// device.
template <typename K, int TAG>
static cudaError_t set_smem(K kern, int bytes) {
  static PerDevice configured;
  std::atomic<int>& slot = configured.here();
  if (bytes <= slot.load(std::memory_order_relaxed)) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess) slot.store(kSmemMax, std::memory_order_relaxed);
  return e;
}

template <int BITS>
static int launch_gemv_t(GemvArgs a, cudaStream_t stream, bool pdl_secondary) {
  const int nG = tile_ng(a.in);
  a.tile_bytes = (int)pair_tile_bytes(a.in, BITS);
  a.stage_bytes = (a.tile_bytes + 127) & ~127;
  // fixed part + per stage (tile + its kNW x 32 partials)
  const int fixed = 3 * kMaxStages * 8 + nG * 32 * 4 + nG * 4 * 5 + kNW * 4 + 128;
  const int per_stage = a.stage_bytes + kNW * 32 * 4;
  int ns = (kSmemBudget - fixed) / per_stage;
  if (ns < 2) ns = (kSmemMax - fixed) / per_stage;
  if (ns > kMaxStages) ns = kMaxStages;
  if (ns < 2) return SLX_ERR_UNSUPPORTED;
  a.n_stages = ns;
  int smem = fixed + ns * per_stage;
  if (smem < kSmemTarget) smem = kSmemTarget;
  if (pdl_enabled()) pdl_secondary = true;
  a.wait_primary = pdl_secondary ? 1 : 0;
  if (a.n_tiles <= 0) return SLX_OK;
  int grid = num_sms();
  // a long dense GEMV (the lm_head) streams from HBM: two CTAs per SM keep
  // twice the tiles in flight (the shared-memory request fits two)
  if (a.mode == SLX_GEMV_LINEAR && a.n_tiles >= 8 * grid) grid *= 2;
  if (grid > a.n_tiles) grid = a.n_tiles;
  cudaError_t e = set_smem<decltype(&k_qgemv<BITS>), BITS>(k_qgemv<BITS>, smem);
  if (e != cudaSuccess) return SLX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_secondary ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, k_qgemv<BITS>, a);
  return e == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_gemv(GemvArgs a, int bits, cudaStream_t stream, bool pdl_secondary) {
  switch (bits) {
    case 2: return launch_gemv_t<2>(a, stream, pdl_secondary);
    case 4: return launch_gemv_t<4>(a, stream, pdl_secondary);
    case 8: return launch_gemv_t<8>(a, stream, pdl_secondary);
    default: return SLX_ERR_UNSUPPORTED;
  }
}

template <int BITS>
static int launch_down_t(DownArgs a, cudaStream_t stream) {
  const int nGr = tile_ng(a.I), nGs = a.Is ? tile_ng(a.Is) : 0;
  const int nGmax = nGr > nGs ? nGr : nGs;
  a.tile_bytes = (int)single_tile_bytes(a.I, BITS);
  a.tile_bytes_sh = a.Is ? (int)single_tile_bytes(a.Is, BITS) : 0;
  a.a_bytes = (long long)expert_a_bytes(a.H, a.I, BITS);
  a.a_bytes_sh = a.Is ? (long long)expert_a_bytes(a.H, a.Is, BITS) : 0;
  const int tb = a.tile_bytes > a.tile_bytes_sh ? a.tile_bytes : a.tile_bytes_sh;
  a.stage_bytes = (tb + 127) & ~127;
  const int fixed = (kMaxStages + 4) * 8 + a.n_units * nGmax * (32 * 4 + 4 * 5) +
                    (2 * kNW + 1) * a.n_units * kRows * 4 + 128;
  // Stages of a work item are released together at its end, so the ring
  // must hold every unit of one item (else the producer could never issue
  // the item's last units).
  int ns = (kSmemBudget - fixed) / a.stage_bytes;
  if (ns < a.n_units) ns = (kSmemMax - fixed) / a.stage_bytes;
  if (ns > kMaxStages) ns = kMaxStages;
  if (ns < a.n_units || ns < 2) return SLX_ERR_UNSUPPORTED;
  a.n_stages = ns;
  int smem = fixed + ns * a.stage_bytes;
  if (smem < kSmemTarget) smem = kSmemTarget;
  if (a.n_items <= 0) return SLX_OK;
  int grid = num_sms();
  if (grid > a.n_items) grid = a.n_items;
  cudaError_t e = set_smem<decltype(&k_down<BITS>), 100 + BITS>(k_down<BITS>, smem);
  if (e != cudaSuccess) return SLX_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (a.pdl || pdl_enabled()) ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, k_down<BITS>, a);
  return e == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

int launch_down(DownArgs a, int bits, cudaStream_t stream) {
  switch (bits) {
    case 2: return launch_down_t<2>(a, stream);
    case 4: return launch_down_t<4>(a, stream);
    case 8: return launch_down_t<8>(a, stream);
    default: return SLX_ERR_UNSUPPORTED;
  }
}

// ---------------------------------------------------- dequant (bit-exact) --

// out[r, c] = scale * q + bias for rows listed in `rows`; fp32 or bf16
// output.  MLX layout input.  One rounding (fmaf of an exact product).
__global__ void k_dequant_rows(const uint32_t* __restrict__ w,
                               const uint16_t* __restrict__ s,
                               const uint16_t* __restrict__ b, int in, int bits,
                               int gs, const int32_t* __restrict__ rows,
                               int nrows, int n_src_rows, void* out,
                               int out_bf16, int32_t* status) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int r = blockIdx.y;
  if (r >= nrows) return;
  const int src = rows ? rows[r] : r;
  if (src < 0 || src >= n_src_rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0)
      set_status(status, SLX_ERR_OUT_OF_RANGE);
    return;
  }
  const int per = 32 / bits;
  const int wpr = in / per;
  const int ng = in / gs;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < in;
       c += gridDim.x * blockDim.x) {
    const uint32_t word = w[(size_t)src * wpr + c / per];
    const uint32_t q = (word >> ((c % per) * bits)) & ((1u << bits) - 1u);
    const float sc = bf16_to_f32(s[(size_t)src * ng + c / gs]);
    const float bi = bf16_to_f32(b[(size_t)src * ng + c / gs]);
    const float v = fmaf(sc, (float)q, bi);
    if (out_bf16)
      reinterpret_cast<uint16_t*>(out)[(size_t)r * in + c] = f32_to_bf16(v);
    else
      reinterpret_cast<float*>(out)[(size_t)r * in + c] = v;
  }
}

int launch_dequant_rows(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                        int in, int bits, int gs, const int32_t* rows,
                        int nrows, int n_src_rows, void* out, int out_bf16,
                        int32_t* status, cudaStream_t stream) {
  if (nrows <= 0) return SLX_OK;
  if (nrows > 65535) return SLX_ERR_INVALID;
  dim3 grid((in + 255) / 256, nrows);
  return launch_k(k_dequant_rows, grid, dim3(256), 0, stream, w, s, b, in, bits,
                  gs, rows, nrows, n_src_rows, out, out_bf16, status) ==
                 cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace slx
