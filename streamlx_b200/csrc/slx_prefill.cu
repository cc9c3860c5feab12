// Expert-major prefill (K3): the grouped quantized SwitchGLU of every
// (token, expert) pair of a prefill chunk, pairs grouped by expert, on the
// 5th-generation tensor cores (tcgen05.mma, fp32 accumulators in TMEM).
//
// Reference: streamlx/integrate.py:141-232 (_expert_sweep) runs
// switch_forward (streamlx/pool.py:30-50: gather_qmm gate/up, swiglu,
// gather_qmm down) over the pairs of each 16-expert batch.  Here one launch
// pair covers every pair of the chunk whose expert has a slot:
//
//   k_pf_pack_x   gathers each pair's token row into the B-operand image of
//                 phase 1 (fp16, 128-byte swizzled K-major rows, one
//                 64-column chunk per quantization group) plus per-group sums;
//   k_prefill<1>  D[128 x N] = [gate rows r..r+63 ; up rows r..r+63] x X^T
//                 over K = hidden, then SwiGLU in the epilogue, written as
//                 phase 2's B image (chunk r/64) + its group sums;
//   k_prefill<2>  D[128 x N] = down rows h..h+127 x Hact^T over K = inter,
//                 rounded to bf16 and stored per pair.
//
// Swap-AB: weight rows fill the M = 128 side of the MMA, the pairs of one
// expert (up to 128, padded to a multiple of 16) are N.
//
// Exact affine arithmetic on fp16 tensor cores.  MLX affine 2-bit weights
// are w = s*q + b per group of 64 (s, b bf16, q in 0..3).  s*q has at most
// 8 + 2 significant bits, so it is EXACT in fp16 (11 bits) whenever
// 2^-17 <= |s| and 3|s| <= 65504; the dequant warps produce it with one fp16
// FMA on the magic-number expansion (1024 + q) * s - 1024 * s.  The bias
// term b * sum(x over the group) rides on extra K columns: per group two
// columns, A = (b, b), B = (hi, lo) with hi + lo = fp32 group sum (hi/lo
// fp16).  The activations enter as fp16 (bf16 values are exact in fp16 for
// 2^-14 <= |x| < 65504; below that the rounding error is < 2^-25).  So each
// output is sum_i s*q_i*x_i + b*sum x accumulated in fp32 -- the same value
// MLX's quantized matrix-vector product forms (scale * dot(q, x) + bias *
// sum(x)) -- and the rounding points are those of switch_forward: gate / up
// outputs to bf16, silu(gate)*up to bf16, down output to bf16.
//
// Inside each 16-code word the K order is permuted so a code pair
// (q[j], q[j+8]) -- one AND of the packed word -- fills one 32-bit A column;
// the B images use the same order (position 16i + 2j + t <- element
// 16i + j + 8t).
//
// Warp roles (448 threads, one CTA per SM, persistent over work items):
//   warp 0      TMEM allocation; lane 0 streams B chunks (cp.async.bulk,
//               the TMA engine) into a 4-stage ring of two-chunk stages;
//   warp 1      lane 0 issues the MMAs (M128 x N x K16, kind::f16) and
//               commits them to the stage / accumulator barriers;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (two TMEM buffers so
//               the next item's MMAs overlap it);
//   warps 6-13  dequantization: each thread owns one A row (TMEM lane),
//               prefetches its packed codes with cp.async eight chunks ahead,
//               and writes fp16 A columns straight into TMEM (tcgen05.st;
//               the MMA reads A from TMEM) or, in the shared-memory
//               variant, into a swizzled A ring.
// Every wait is bounded (2 s); on expiry the kernel records
// SLX_ERR_DEVICE_TIMEOUT, drains its in-flight copies and MMAs, frees TMEM
// and returns.
#include "slx_kernels.cuh"
#include "slx_tiles.cuh"

// Diagnostics build only (-DSLX_PF_TRACE): %globaltimer stamps of each
// warp role at pipeline stages 8..15 of phase 1, per CTA.
#ifdef SLX_PF_TRACE
static __device__ unsigned long long g_pf_trace[148][8][8];
extern "C" int slx_pf_trace_read(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, g_pf_trace, sizeof(g_pf_trace)) ==
                 cudaSuccess ? 0 : -1;
}
#define PF_STAMP(G, E)                                                     \
  do {                                                                     \
    if (PHASE == 1 && blockIdx.x < 148 && (G) >= 8 && (G) < 16)            \
      g_pf_trace[blockIdx.x][(G) - 8][E] = slx::globaltimer_ns();          \
  } while (0)
#else
#define PF_STAMP(G, E) \
  do {                 \
  } while (0)
#endif

namespace slx {
namespace {

constexpr int kNT = 128;            // max pairs per block (MMA N)
// Tuning (compile-time; the defaults are the shipped configuration).
#ifndef SLX_PF_STAGES
#define SLX_PF_STAGES 4       // stages with the operand in TMEM (2 or 4)
#endif
#ifndef SLX_PF_L2_PREFETCH
#define SLX_PF_L2_PREFETCH 1  // prefetch B chunks one ring ahead into L2
#endif
#ifndef SLX_PF_SLEEP_WAIT
#define SLX_PF_SLEEP_WAIT 1   // barrier polls with a suspend-time hint
#endif
#ifndef SLX_PF_DQ_DEPTH
#define SLX_PF_DQ_DEPTH 4     // code prefetch depth in stages (2..4)
#endif

constexpr int kCPS = 2;             // 64-column chunks per pipeline stage
constexpr int kS = 4;               // max pipeline stages
// stages: 4 with the weight operand in TMEM (A ring 4 x 64 columns + two
// 128-column accumulators = 512), 2 with it in shared memory (the A ring
// then takes 2 x 32 KB of shared memory); 8 resp. 4 chunks in flight
constexpr int stages(bool atmem) { return atmem ? SLX_PF_STAGES : 2; }
constexpr int kRowB = 128;          // bytes of one 64-column fp16 chunk row
constexpr int kStageB = kNT * kRowB;     // B chunk (16 KB)
constexpr int kStageA = 128 * kRowB;     // A chunk, shared-memory variant
constexpr int kThreads = 448;
constexpr int kDqThreads = 256;
constexpr int kDqDepth = SLX_PF_DQ_DEPTH;  // cp.async tasks (stages) in flight per thread
constexpr int kAccCol = 32 * kCPS * kS;  // TMEM: A ring at 0..255, accumulators after
constexpr int kTmemCols = 512;
constexpr int kXchStride = kNT + 2; // bf16 per row of the up-value exchange

// --------------------------------------------------------------- tcgen05 --

SLX_DEV void tc_alloc(uint32_t* dst, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst)), "r"(ncols) : "memory");
}
SLX_DEV void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SLX_DEV void tc_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}
SLX_DEV void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
SLX_DEV void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive (once) on `bar` when every MMA this thread issued so far completes.
SLX_DEV void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      ::"r"(smem_u32(bar)) : "memory");
}
SLX_DEV void tc_mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc,
                       uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}
SLX_DEV void tc_mma_ts(uint32_t d, uint32_t a_tmem, uint64_t bdesc,
                       uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}
SLX_DEV void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}
SLX_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SLX_DEV void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]),
        "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]),
        "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
        "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
SLX_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded mbarrier wait whose polls let the thread sleep in the hardware
// (try_wait with a suspend-time hint of 0.2 ms) instead of spinning: the
// waiting warps then leave their issue slots to the working ones.
SLX_DEV bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int32_t* status) {
  if (!SLX_PF_SLEEP_WAIT) return mbar_wait(bar, parity, status);
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(200000u)
        : "memory");
    if (done) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_status(status, SLX_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes stacked along M/N (stride 1024), descriptor version 1.
SLX_DEV uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;              // leading byte offset (unused: swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset
  d |= (uint64_t)1u << 46;              // version
  d |= (uint64_t)2u << 61;              // SWIZZLE_128B
  return d;
}
// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D,
// M = 128, N = n.
SLX_DEV uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ------------------------------------------------------- misc async ops --

SLX_DEV void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
SLX_DEV void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
SLX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SLX_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
SLX_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
SLX_DEV void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
SLX_DEV void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"(dst), "r"(smem_u32(src)), "r"(bytes) : "memory");
}
SLX_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
SLX_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
SLX_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
SLX_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
SLX_DEV void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Named barrier that also ORs a predicate over its n threads: every thread
// gets the same answer, so a decision to stop is taken by all alike.
SLX_DEV bool named_bar_or(int id, int n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r) : "r"((uint32_t)p), "r"(id), "r"(n) : "memory");
  return r != 0;
}

// Position of element r (0..63) of a group inside the permuted K order.
SLX_HOST_DEV int kpos(int r) { return (r & ~15) + 2 * (r & 7) + ((r >> 3) & 1); }
// Byte offset of fp16 position pos of row n inside a 128-byte-swizzled chunk.
SLX_DEV int sw_off(int n, int pos) {
  return n * kRowB + ((((pos >> 3) ^ (n & 7))) << 4) + ((pos & 7) << 1);
}
SLX_DEV uint16_t h_bits(__half h) { return *reinterpret_cast<uint16_t*>(&h); }

}  // namespace

struct PrefillArgs {
  const uint8_t* bank;
  long long slot_stride;
  int n_slots, H, I;
  const int4* blocks;  // {slot, first pair, pairs, 0}
  int n_blocks, n_pairs, n_items, n_mb;
  int nG, nC, nStg;    // this phase: groups along K, chunks incl. bias
                       // chunks, pipeline stages per item
  const uint8_t* bimg; // this phase's B image [n_blocks][nC][kNT][128]
  uint8_t* himg;       // phase 1 output: phase 2's B image
  int nG2, nC2;
  uint16_t* out;       // phase 2: [n_out, H] bf16
  const int32_t* out_row;
  int n_out;
  int32_t* status;
  int off_b, off_a, off_stg, off_btab, off_xch, off_hst, off_orow;  // from the aligned base
};

namespace {

SLX_DEV bool block_ok(const PrefillArgs& a, int4 bl) {
  return bl.x >= 0 && bl.x < a.n_slots && bl.z >= 1 && bl.z <= kNT &&
         bl.y >= 0 && (long long)bl.y + bl.z <= a.n_pairs;
}

// Cursor over this CTA's (item, chunk) tasks; invalid blocks are skipped by
// every role alike.
struct Cur {
  int j, c, item, blk, mb, slot, p0, n;
  bool end;
};
SLX_DEV void cur_seek(const PrefillArgs& a, Cur& t) {
  for (;; ++t.j) {
    t.item = blockIdx.x + t.j * gridDim.x;
    if (t.item >= a.n_items) { t.end = true; return; }
    t.blk = t.item / a.n_mb;
    const int4 bl = a.blocks[t.blk];
    if (block_ok(a, bl)) {
      t.mb = t.item % a.n_mb;
      t.slot = bl.x; t.p0 = bl.y; t.n = bl.z;
      t.end = false;
      return;
    }
  }
}
SLX_DEV void cur_init(const PrefillArgs& a, Cur& t) { t.j = 0; t.c = 0; cur_seek(a, t); }
SLX_DEV void cur_next_item(const PrefillArgs& a, Cur& t) { t.c = 0; ++t.j; cur_seek(a, t); }
// t.c counts the item's pipeline stages (kCPS chunks each)
SLX_DEV void cur_next(const PrefillArgs& a, Cur& t) {
  if (++t.c == a.nStg) cur_next_item(a, t);
}

SLX_DEV int npad16(int n) { return (n + 15) & ~15; }
SLX_DEV int bias_ksteps(int nG, int cb) {  // issued K steps of bias chunk cb
  const int cols = 2 * nG - 64 * cb;
  const int k = (cols + 15) / 16;
  return k > 4 ? 4 : k;
}

// Where A row m (this thread) of an item reads its packed codes: the row's
// first byte, its swizzle key, and its scale|bias word of group 0 with the
// word stride between groups (computed once per item).
struct RowSrc {
  const uint8_t* row;
  const uint32_t* sb;
  int swz, sbs, j;
};
template <int PHASE>
SLX_DEV void row_src(const PrefillArgs& a, int slot, int mb, int m, RowSrc& o) {
  const uint8_t* e = a.bank + (size_t)slot * a.slot_stride;
  if (PHASE == 1) {
    const int RB = tile_rb(a.H, 2);
    const int r = mb * 64 + (m & 63), mat = m >> 6;
    const int t = r >> 4, tr = r & 15;
    const uint8_t* base = e + (size_t)t * pair_tile_bytes(a.H, 2);
    o.row = base + (size_t)(mat * 16 + tr) * RB;
    o.swz = tile_swizzled(a.H, 2) ? (tr & 7) : 0;
    o.sb = reinterpret_cast<const uint32_t*>(base + 32 * RB) + mat * 16 + tr;
    o.sbs = 32;
  } else {
    const int RB = tile_rb(a.I, 2);
    const int r = mb * 128 + m;
    const int t = r >> 4, tr = r & 15;
    const uint8_t* base = e + expert_a_bytes(a.H, a.I, 2) +
                          (size_t)t * single_tile_bytes(a.I, 2);
    o.row = base + (size_t)tr * RB;
    o.swz = tile_swizzled(a.I, 2) ? (tr & 7) : 0;
    o.sb = reinterpret_cast<const uint32_t*>(base + 16 * RB) + tr;
    o.sbs = 16;
  }
}

}  // namespace

template <int PHASE, bool ATMEM>
__global__ void __launch_bounds__(kThreads, 1)
    k_prefill(const __grid_constant__ PrefillArgs a) {
  constexpr int S = stages(ATMEM);
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t* bar_tx = reinterpret_cast<uint64_t*>(smem_raw);  // [S] B bytes landed
  uint64_t* bar_dq = bar_tx + kS;                            // [S] A written
  uint64_t* bar_empty = bar_dq + kS;                         // [S] MMAs done
  uint64_t* bar_full = bar_empty + kS;                       // [2] accumulator ready
  uint64_t* bar_free = bar_full + 2;                          // [2] accumulator drained
  uint64_t* bar_done = bar_free + 2;                          // all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // 1024-aligned region for the swizzled buffers
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - ((raw + 256u) & 1023u)) & 1023u) + 256;
  uint8_t* sB = base + a.off_b;
  uint8_t* sA = base + a.off_a;
  uint8_t* stg = base + a.off_stg;
  __half* btab = reinterpret_cast<__half*>(base + a.off_btab);
  uint16_t* xch = reinterpret_cast<uint16_t*>(base + a.off_xch);  // up values, bf16
  uint8_t* hst = base + a.off_hst;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bar_tx[i], 1);
      mbar_init(&bar_dq[i], kDqThreads / 32);
      mbar_init(&bar_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_free[i], 4);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tc_alloc(tmem_slot, kTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto fail = [&](int code) {
    set_status(a.status, code);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ---------------------------------------------------- B producer ----
    if (lane == 0) {
      Cur t, pb;  // pb runs one ring ahead: its chunks are prefetched to L2
      cur_init(a, t);
      cur_init(a, pb);
      for (int i = 0; i < S && !pb.end; ++i) cur_next(a, pb);
      uint32_t g = 0;
      for (; !t.end && !*abort_flag; cur_next(a, t), ++g) {
        const int st = g % S;
        if (SLX_PF_L2_PREFETCH && !pb.end) {
          const int p0 = pb.c * kCPS;
          const int pn = a.nC - p0 < kCPS ? a.nC - p0 : kCPS;
          const uint8_t* ps = a.bimg + ((size_t)pb.blk * a.nC + p0) * kStageB;
          for (int ci = 0; ci < pn; ++ci)
            bulk_prefetch_l2(ps + (size_t)ci * kStageB, (uint32_t)npad16(pb.n) * kRowB);
          cur_next(a, pb);
        }
        if (!mbar_wait_sleep(&bar_empty[st], ((g / S) & 1) ^ 1, a.status)) { fail(SLX_ERR_DEVICE_TIMEOUT); break; }
        PF_STAMP(g, 0);
        const uint32_t bytes = (uint32_t)npad16(t.n) * kRowB;
        const int c0 = t.c * kCPS;
        const int nch = a.nC - c0 < kCPS ? a.nC - c0 : kCPS;
        const uint8_t* src = a.bimg + ((size_t)t.blk * a.nC + c0) * kStageB;
        mbar_arrive_expect_tx(&bar_tx[st], bytes * nch);
        for (int ci = 0; ci < nch; ++ci)
          bulk_g2s_plain(sB + ((size_t)st * kCPS + ci) * kStageB,
                         src + (size_t)ci * kStageB, bytes, &bar_tx[st]);
        PF_STAMP(g, 1);
      }
      // drain: every issued copy has landed before the CTA exits
      const uint32_t issued = g;
      for (uint32_t h = issued > S ? issued - S : 0; h < issued; ++h)
        mbar_wait(&bar_tx[h % S], (h / S) & 1, a.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issue ----
    if (lane == 0) {
      Cur t;
      cur_init(a, t);
      uint32_t g = 0;
      int jl = 0;
      bool ok = true;
      while (!t.end && ok && !*abort_flag) {
        const int buf = jl & 1;
        if (!mbar_wait(&bar_free[buf], ((jl >> 1) & 1) ^ 1, a.status)) { fail(SLX_ERR_DEVICE_TIMEOUT); break; }
        tc_fence_after();
        const uint32_t d = tmem + kAccCol + buf * kNT;
        const uint32_t idesc = idesc_f16(npad16(t.n));
        for (int sg = 0; sg < a.nStg; ++sg, ++g) {
          const int st = g % S;
          const uint32_t ph = (g / S) & 1;
          bool okw = mbar_wait(&bar_tx[st], ph, a.status);
          PF_STAMP(g, 2);
          okw = okw && mbar_wait(&bar_dq[st], ph, a.status);
          PF_STAMP(g, 3);
          if (!okw) {
            fail(SLX_ERR_DEVICE_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const int c0 = sg * kCPS;
          const int nch = a.nC - c0 < kCPS ? a.nC - c0 : kCPS;
          for (int ci = 0; ci < nch; ++ci) {
            const int c = c0 + ci;
            const int nk = c < a.nG ? 4 : bias_ksteps(a.nG, c - a.nG);
            const uint32_t b0 = smem_u32(sB + ((size_t)st * kCPS + ci) * kStageB);
            const uint32_t a0 = smem_u32(sA + ((size_t)st * kCPS + ci) * kStageA);
            for (int s = 0; s < nk; ++s) {
              const uint64_t bd = sdesc_sw128(b0 + 32 * s);
              const uint32_t acc = (c | s) != 0;
              if (ATMEM)
                tc_mma_ts(d, tmem + (st * kCPS + ci) * 32 + 8 * s, bd, idesc, acc);
              else
                tc_mma_ss(d, sdesc_sw128(a0 + 32 * s), bd, idesc, acc);
            }
          }
          tc_commit(&bar_empty[st]);
          PF_STAMP(g, 4);
        }
        if (!ok) break;
        tc_commit(&bar_full[buf]);
        ++jl;
        cur_next_item(a, t);
      }
      tc_commit(bar_done);
      mbar_wait(bar_done, 0, a.status);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------- epilogue ----
    const int q = warp & 3;
    const int te = threadIdx.x - 64;  // 0..127
    const bool issuer = te == 0;
    Cur t;
    cur_init(a, t);
    int jl = 0;
    while (!t.end) {
      const int buf = jl & 1;
      const bool ok = __all_sync(0xffffffffu,
                                 mbar_wait_sleep(&bar_full[buf], (jl >> 1) & 1, a.status));
      if (!ok) fail(SLX_ERR_DEVICE_TIMEOUT);
      bool stop = !ok || *abort_flag;
      stop = named_bar_or(1, 128, stop);
      if (stop) break;
      tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + kAccCol + buf * kNT;
      const int np = npad16(t.n);
      if (PHASE == 1) {
        if (issuer) bulk_wait_read();  // the previous item's store left hst
        named_bar(1, 128);
        const int r = 32 * (q & 1) + lane;  // I row within the block
        if (q >= 2) {
          for (int cc = 0; cc < np; cc += 16) {
            uint32_t v[16];
            tc_ld16(tq + cc, v);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              xch[r * kXchStride + cc + i] = f32_to_bf16(__uint_as_float(v[i]));
          }
        }
        named_bar(1, 128);
        if (q < 2) {
          const int pos = kpos(r);
          for (int cc = 0; cc < np; cc += 16) {
            uint32_t v[16];
            tc_ld16(tq + cc, v);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int n = cc + i;
              const float gt = round_bf16(__uint_as_float(v[i]));
              const float up = bf16_to_f32(xch[r * kXchStride + n]);
              const float h = round_bf16(silu_f32(gt) * up);
              *reinterpret_cast<uint16_t*>(hst + sw_off(n, pos)) =
                  h_bits(__float2half_rn(h));
            }
          }
          fence_proxy_async();
        }
        tc_fence_before();
        named_bar(1, 128);
        // group sums of the 64 h values of each pair -> phase 2 bias columns
        if (te < t.n) {
          const uint4* row = reinterpret_cast<const uint4*>(hst + te * kRowB);
          float s = 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 w = row[(u + te) & 7];  // 8 threads: 8 distinct units
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
              s += f.x + f.y;
            }
          }
          const __half hi = __float2half_rn(s);
          const __half lo = __float2half_rn(s - __half2float(hi));
          const int pos = 2 * (t.mb & 31);
          uint8_t* dst = a.himg + ((size_t)t.blk * a.nC2 + a.nG2 + (t.mb >> 5)) * kStageB +
                         sw_off(te, pos);
          *reinterpret_cast<uint32_t*>(dst) =
              (uint32_t)h_bits(hi) | ((uint32_t)h_bits(lo) << 16);
        }
        if (issuer) {
          bulk_s2g(a.himg + ((size_t)t.blk * a.nC2 + t.mb) * kStageB, hst,
                   (uint32_t)np * kRowB);
          bulk_commit();
        }
      } else {
        // output rows of the item's pairs, staged once (one load per thread)
        int32_t* orow = reinterpret_cast<int32_t*>(base + a.off_orow);
        if (te < t.n) {
          const int p = t.p0 + te;
          orow[te] = a.out_row ? a.out_row[p] : p;
        }
        named_bar(1, 128);
        const int hr = t.mb * 128 + 32 * q + lane;
        for (int cc = 0; cc < t.n; cc += 16) {
          uint32_t v[16];
          tc_ld16(tq + cc, v);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = cc + i;
            if (n < t.n) {
              const int row = orow[n];
              if (row >= 0 && row < a.n_out)
                a.out[(size_t)row * a.H + hr] = f32_to_bf16(__uint_as_float(v[i]));
              else if (q == 0 && lane == 0)
                set_status(a.status, SLX_ERR_OUT_OF_RANGE);
            }
          }
        }
        tc_fence_before();
        named_bar(1, 128);  // orow is rewritten by the next item
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_free[buf]);
      ++jl;
      cur_next_item(a, t);
    }
    if (PHASE == 1 && issuer) bulk_wait_all();
  } else {
    // -------------------------------------------------- dequantization ----
    // Group grp (warps 6-9 / 10-13) dequantizes chunk grp of every stage:
    // each thread one A row (TMEM lane), the row's whole 16-byte code unit.
    const int dq = threadIdx.x - 192;  // 0..255
    const int grp = (warp - 6) >> 2;   // chunk of the stage this group owns
    const int q = warp & 3;
    const int m = 32 * q + lane;       // A row = TMEM lane
    const int gt = dq & 127;           // thread within the group
    // staging, thread-contiguous (conflict-free): codes [slot][group thread]
    // 16 bytes, scale|bias words [slot][group thread] 4 bytes, per group
    uint4* stg_codes = reinterpret_cast<uint4*>(stg) + grp * kDqDepth * 128;
    uint32_t* stg_sb = reinterpret_cast<uint32_t*>(stg + 2 * kDqDepth * 128 * 16) +
                       grp * kDqDepth * 128;
    Cur pf, cu;
    cur_init(a, pf);
    cur_init(a, cu);
    RowSrc rs;
    rs.j = -1;
    auto issue = [&](int slot) {
      if (!pf.end) {
        const int c = pf.c * kCPS + grp;
        if (c < a.nG) {
          if (rs.j != pf.j) {
            row_src<PHASE>(a, pf.slot, pf.mb, m, rs);
            rs.j = pf.j;
          }
          const int u = slot * 128 + gt;
          cp_async16(smem_u32(stg_codes + u), rs.row + ((c ^ rs.swz) << 4));
          cp_async4(smem_u32(stg_sb + u), rs.sb + c * rs.sbs);
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < kDqDepth; ++s) {
      issue(s);
      cur_next(a, pf);
    }
    uint32_t g = 0;
    while (!cu.end && !__any_sync(0xffffffffu, *abort_flag != 0)) {
      cp_async_wait<kDqDepth - 1>();
      if (warp == 6 && lane == 0) PF_STAMP(g, 5);
      const int slot = g % kDqDepth;
      const int c = cu.c * kCPS + grp;
      // bias table [g][row] of this item; two buffers by item parity (the
      // other group may already be in the next item, at most a ring ahead)
      __half* bt = btab + (cu.j & 1) * a.nG * 128;
      uint4 cw = make_uint4(0, 0, 0, 0);
      uint32_t sbw = 0;
      if (c < a.nG) {
        cw = stg_codes[slot * 128 + gt];
        sbw = stg_sb[slot * 128 + gt];
      }
      issue(slot);
      cur_next(a, pf);
      const int st = g % S;
      bool ok = mbar_wait_sleep(&bar_empty[st], ((g / S) & 1) ^ 1, a.status);
      if (warp == 6 && lane == 0) PF_STAMP(g, 6);
      if (ok && c >= a.nG && c < a.nC && g > 0) {
        // bias chunk: every code chunk of the item (both groups) has written
        // its biases once the previous stage's arrivals are complete
        ok = mbar_wait_sleep(&bar_dq[(g - 1) % S], ((g - 1) / S) & 1, a.status);
      }
      if (!__all_sync(0xffffffffu, ok)) {
        fail(SLX_ERR_DEVICE_TIMEOUT);
        break;
      }
      if (c < a.nC) {
        uint32_t out[32];
        if (c < a.nG) {
          const __half s16 = __float2half_rn(bf16_lo(sbw));
          bt[c * 128 + m] = __float2half_rn(bf16_hi(sbw));
          const __half2 s2 = __half2half2(s16);
          const __half2 n2 = __half2half2(__hneg(__hmul(s16, __float2half_rn(1024.f))));
          const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t r = ((wd[i] >> (2 * j)) & 0x00030003u) | 0x64006400u;
              const __half2 h = __hfma2(*reinterpret_cast<const __half2*>(&r), s2, n2);
              out[8 * i + j] = *reinterpret_cast<const uint32_t*>(&h);
            }
          }
        } else {
          const int cb = c - a.nG;
#pragma unroll
          for (int k2 = 0; k2 < 32; ++k2) {
            const int gi = 32 * cb + k2;
            const uint32_t hb = gi < a.nG ? h_bits(bt[gi * 128 + m]) : 0u;
            out[k2] = hb | (hb << 16);
          }
        }
        if (ATMEM) {
          tc_st32(tmem + ((uint32_t)(32 * q) << 16) + (st * kCPS + grp) * 32, out);
          tc_wait_st();
          tc_fence_before();
        } else {
          uint8_t* rowp = sA + ((size_t)st * kCPS + grp) * kStageA + (m >> 3) * 1024 +
                          (m & 7) * kRowB;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int pu = u ^ (m & 7);
            *reinterpret_cast<uint4*>(rowp + pu * 16) =
                make_uint4(out[4 * u], out[4 * u + 1], out[4 * u + 2], out[4 * u + 3]);
          }
          fence_proxy_async();
        }
      }
      __syncwarp();
      if (warp == 6 && lane == 0) PF_STAMP(g, 7);
      if (lane == 0) mbar_arrive(&bar_dq[st]);
      cur_next(a, cu);
      ++g;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem, kTmemCols);
  }
}

// Phase-1 B image: pair rows of x in the permuted, swizzled fp16 layout plus
// (hi, lo) group sums.  One warp per (block, pair row); 4 groups per pass.
__global__ void __launch_bounds__(256)
    k_pf_pack_x(const uint16_t* __restrict__ x, int n_rows, int H,
                const int32_t* __restrict__ pair_row, const int4* __restrict__ blocks,
                int n_blocks, int n_pairs, int n_slots, int nG, int nC,
                uint8_t* __restrict__ img, int32_t* status) {
  const int b = blockIdx.x;
  const int n = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int4 bl = blocks[b];
  const bool ok = bl.x >= 0 && bl.x < n_slots && bl.z >= 1 && bl.z <= kNT &&
                  bl.y >= 0 && (long long)bl.y + bl.z <= n_pairs;
  if (!ok) {
    if (n == 0 && lane == 0) set_status(status, SLX_ERR_OUT_OF_RANGE);
    return;
  }
  if (n >= bl.z) return;
  const int xr = pair_row[bl.y + n];
  if (xr < 0 || xr >= n_rows) {
    if (lane == 0) set_status(status, SLX_ERR_OUT_OF_RANGE);
    return;
  }
  const uint16_t* xrow = x + (size_t)xr * H;
  uint8_t* blk = img + (size_t)b * nC * kStageB;
  const int u = lane & 7;            // 16-byte unit of the chunk row
  const int i = u >> 1, j0 = 4 * (u & 1);
  for (int c0 = 0; c0 < nG; c0 += 4) {
    const int c = c0 + (lane >> 3);
    const uint16_t* src = xrow + 64 * c + 16 * i + j0;
    const uint2 lo4 = *reinterpret_cast<const uint2*>(src);      // elements j0..j0+3
    const uint2 hi4 = *reinterpret_cast<const uint2*>(src + 8);  // j0+8..j0+11
    const uint32_t lw[4] = {lo4.x & 0xFFFFu, lo4.x >> 16, lo4.y & 0xFFFFu, lo4.y >> 16};
    const uint32_t hw[4] = {hi4.x & 0xFFFFu, hi4.x >> 16, hi4.y & 0xFFFFu, hi4.y >> 16};
    uint32_t o[4];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a0 = bf16_to_f32((uint16_t)lw[k]);
      const float a1 = bf16_to_f32((uint16_t)hw[k]);
      s += a0 + a1;
      o[k] = (uint32_t)h_bits(__float2half_rn(a0)) |
             ((uint32_t)h_bits(__float2half_rn(a1)) << 16);
    }
    *reinterpret_cast<uint4*>(blk + (size_t)c * kStageB + n * kRowB +
                              ((u ^ (n & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (u == 0) {
      const __half hi = __float2half_rn(s);
      const __half lo = __float2half_rn(s - __half2float(hi));
      const int pos = 2 * (c & 31);
      *reinterpret_cast<uint32_t*>(blk + (size_t)(nG + (c >> 5)) * kStageB +
                                   n * kRowB + ((((pos >> 3) ^ (n & 7))) << 4) +
                                   ((pos & 7) << 1)) =
          (uint32_t)h_bits(hi) | ((uint32_t)h_bits(lo) << 16);
    }
  }
}

// ------------------------------------------------------------ launchers --

namespace {

int pf_chunks(int nG) { return nG + (nG + 31) / 32; }

struct SmemPlan {
  int off_b, off_a, off_stg, off_btab, off_xch, off_hst, off_orow, bytes;
};

SmemPlan plan_smem(int phase, bool atmem, int nG) {
  SmemPlan p = {};
  int o = 0;
  p.off_b = o;   o += stages(atmem) * kCPS * kStageB;
  p.off_hst = o; if (phase == 1) o += kStageB;
  p.off_a = o;   if (!atmem) o += stages(atmem) * kCPS * kStageA;
  p.off_stg = o; o += 2 * kDqDepth * 128 * (16 + 4);
  p.off_btab = o; o += 2 * nG * 128 * 2;
  o = (o + 15) & ~15;
  p.off_xch = o; if (phase == 1) o += 64 * kXchStride * 2;
  o = (o + 15) & ~15;
  p.off_orow = o; if (phase == 2) o += kNT * 4;
  // + barrier area (256) + worst-case 1024 alignment; at least 120 KB so one
  // CTA (and one 512-column TMEM allocation) per SM
  int bytes = o + 256 + 1024;
  if (bytes < 120 * 1024) bytes = 120 * 1024;
  p.bytes = bytes;
  return p;
}

int g_num_sms_pf = 0;

template <int PHASE, bool ATMEM>
int launch_phase(PrefillArgs a, int smem, cudaStream_t s) {
  static int attr_set = 0;
  if (!attr_set) {
    if (cudaFuncSetAttribute(k_prefill<PHASE, ATMEM>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return SLX_ERR_CUDA;
    attr_set = 1;
  }
  if (a.n_items == 0) return SLX_OK;
  const int grid = a.n_items < g_num_sms_pf ? a.n_items : g_num_sms_pf;
  k_prefill<PHASE, ATMEM><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace

size_t prefill_scratch_bytes(int n_blocks, int H, int I) {
  const size_t c1 = pf_chunks(H / 64), c2 = pf_chunks(I / 64);
  return (size_t)n_blocks * (c1 + c2) * kStageB;
}

int launch_prefill(const uint8_t* bank, long long slot_stride, int n_slots,
                   int H, int I, const uint16_t* x, int n_rows,
                   const int32_t* pair_row, int n_pairs, const int4* blocks,
                   int n_blocks, const int32_t* out_row, uint16_t* out,
                   int n_out, uint8_t* scratch, int32_t* status, int a_tmem,
                   cudaStream_t s) {
  if (g_num_sms_pf == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&g_num_sms_pf, cudaDevAttrMultiProcessorCount,
                               dev) != cudaSuccess)
      return SLX_ERR_CUDA;
  }
  const int nG1 = H / 64, nG2 = I / 64;
  if (nG1 > 64 || nG2 > 64) return SLX_ERR_UNSUPPORTED;
  PrefillArgs a = {};
  a.bank = bank;
  a.slot_stride = slot_stride;
  a.n_slots = n_slots;
  a.H = H;
  a.I = I;
  a.blocks = blocks;
  a.n_blocks = n_blocks;
  a.n_pairs = n_pairs;
  a.status = status;
  a.nG2 = nG2;
  a.nC2 = pf_chunks(nG2);
  uint8_t* ximg = scratch;
  uint8_t* himg = scratch + (size_t)n_blocks * pf_chunks(nG1) * kStageB;
  a.himg = himg;
  a.out = out;
  a.out_row = out_row;
  a.n_out = n_out;

  // phase 0: gather x rows into phase 1's B image
  {
    dim3 grid(n_blocks, kNT / 8);
    k_pf_pack_x<<<grid, 256, 0, s>>>(x, n_rows, H, pair_row, blocks, n_blocks,
                                     n_pairs, n_slots, nG1, pf_chunks(nG1),
                                     ximg, status);
    if (cudaGetLastError() != cudaSuccess) return SLX_ERR_CUDA;
  }
  // phase 1: gate/up -> SwiGLU -> phase 2's B image
  {
    PrefillArgs p = a;
    p.nG = nG1;
    p.nC = pf_chunks(nG1);
    p.nStg = (p.nC + kCPS - 1) / kCPS;
    p.n_mb = I / 64;
    p.n_items = n_blocks * p.n_mb;
    p.bimg = ximg;
    const SmemPlan sp = plan_smem(1, a_tmem != 0, nG1);
    p.off_b = sp.off_b; p.off_a = sp.off_a; p.off_stg = sp.off_stg;
    p.off_btab = sp.off_btab; p.off_xch = sp.off_xch; p.off_hst = sp.off_hst;
    p.off_orow = sp.off_orow;
    if (sp.bytes > 227 * 1024) return SLX_ERR_UNSUPPORTED;
    const int rc = a_tmem ? launch_phase<1, true>(p, sp.bytes, s)
                          : launch_phase<1, false>(p, sp.bytes, s);
    if (rc) return rc;
  }
  // phase 2: down projection -> per-pair outputs
  {
    PrefillArgs p = a;
    p.nG = nG2;
    p.nC = pf_chunks(nG2);
    p.nStg = (p.nC + kCPS - 1) / kCPS;
    p.n_mb = H / 128;
    p.n_items = n_blocks * p.n_mb;
    p.bimg = himg;
    const SmemPlan sp = plan_smem(2, a_tmem != 0, nG2);
    p.off_b = sp.off_b; p.off_a = sp.off_a; p.off_stg = sp.off_stg;
    p.off_btab = sp.off_btab; p.off_xch = sp.off_xch; p.off_hst = sp.off_hst;
    p.off_orow = sp.off_orow;
    if (sp.bytes > 227 * 1024) return SLX_ERR_UNSUPPORTED;
    const int rc = a_tmem ? launch_phase<2, true>(p, sp.bytes, s)
                          : launch_phase<2, false>(p, sp.bytes, s);
    if (rc) return rc;
  }
  return SLX_OK;
}

}  // namespace slx
