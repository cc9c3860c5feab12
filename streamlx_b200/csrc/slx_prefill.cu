// Expert-major prefill (K3): the grouped quantized SwitchGLU of every
// (token, expert) pair of a prefill chunk, pairs grouped by expert, on the
// 5th-generation tensor cores (tcgen05.mma, fp32 accumulators in TMEM).
//
// Reference: streamlx/integrate.py:141-232 (_expert_sweep) runs
// switch_forward (streamlx/pool.py:30-50: gather_qmm gate/up, swiglu,
// gather_qmm down) over the pairs of each 16-expert batch.  Here one launch
// pair covers every pair of the chunk whose expert has a slot:
//
//   k_pf_pack_x   gathers each pair's token row into phase 1's activation
//                 image (fp16, 128-byte swizzled K-major rows, one 64-column
//                 chunk per quantization group) plus per-group sums;
//   k_prefill<1>  D[128 pairs x 256] = X x [gate rows r..r+127 ; up rows
//                 r..r+127]^T over K = hidden; SwiGLU in the epilogue (a
//                 thread = one pair holds both its gate and up values),
//                 written as phase 2's activation image + group sums;
//   k_prefill<2>  D[128 pairs x 256] = Hact x [down rows h..h+255]^T over
//                 K = inter, rounded to bf16 and stored per pair.
//
// The pairs of one expert (up to 128, a block) are the MMA's M side and 256
// weight rows its N side: a tcgen05.mma costs about the same whether N is
// 64 or 256 here, so the widest N halves the instructions per layer.
//
// Exact affine arithmetic on fp16 tensor cores.  MLX affine 2-bit weights
// are w = s*q + b per group of 64 (s, b bf16, q in 0..3).  s*q has at most
// 8 + 2 significant bits, so it is EXACT in fp16 (11 bits) whenever
// 2^-17 <= |s| (its last bit >= the fp16 subnormal step 2^-24); the dequant
// warps produce it with one fp16 FMA on the magic-number expansion
// (1024 + q) * s - 1024 * s, whose addend 1024 * s must itself be finite:
// |s| < 64.  The bias term b * sum(x over the group) rides on extra K
// columns: per group two columns, weights (b, b), activations (hi, lo) with
// hi + lo = the fp32 group sum; b is exact in fp16 for 2^-17 <= |b| <
// 65504.  Activations and SwiGLU outputs enter as fp16 (bf16 values are
// exact there for 2^-17 <= |x| < 65504; a smaller one is off by < 2^-25),
// and a group sum must stay below 65504.  The kernels check every scale,
// bias, activation and group sum against those bounds (s = 0 and b = 0 are
// exact) and report SLX_ERR_RANGE instead of a wrong result; the host then
// runs the call on the GEMV kernels, whose scale/bias arithmetic is fp32.
// So each
// output is sum_i s*q_i*x_i + b*sum x accumulated in fp32 -- the value MLX's
// quantized matrix-vector product forms (scale * dot(q, x) + bias * sum(x))
// -- and the rounding points are those of switch_forward: gate / up to bf16,
// silu(gate)*up to bf16, down output to bf16.
//
// Inside each 16-code word the K order is permuted so a code pair
// (q[j], q[j+8]) -- one AND of the packed word -- fills one 32-bit column;
// the activation images use the same order (position 16i + 2j + t <-
// element 16i + j + 8t).
//
// Warp roles (448 threads, one CTA per SM, persistent over work items):
//   warp 0      TMEM allocation; lane 0 streams activation chunks
//               (cp.async.bulk, the TMA engine) into a 4-stage ring, with
//               an L2 prefetch of the chunks one ring ahead (a copy takes
//               ~3 us to land);
//   warp 1      lane 0 issues the MMAs (M128 x N256 x K16, kind::f16, both
//               operands in shared memory) and commits them to the ring /
//               accumulator barriers;
//   warps 2-5   epilogue: each thread one pair (TMEM lane), tcgen05.ld of
//               its 256 accumulator columns (two TMEM buffers, so the next
//               item's MMAs overlap it);
//   warps 6-13  dequantization: each thread one weight row; its 16-byte
//               code unit and scale|bias word prefetched with cp.async four
//               chunks ahead; fp16 weights written into a ring of
//               swizzled K-major chunks (a 3-stage ring).
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

constexpr int kNT = 128;            // max pairs per block (MMA M)
constexpr int kNW = 256;            // weight rows per item (MMA N)
constexpr int kRowB = 128;          // bytes of one 64-column fp16 chunk row
constexpr int kActB = kNT * kRowB;  // activation chunk (16 KB)
constexpr int kWB = kNW * kRowB;    // weight chunk (32 KB)
#ifndef SLX_PF_SX
#define SLX_PF_SX 4
#endif
#ifndef SLX_PF_SW
#define SLX_PF_SW 3
#endif
constexpr int kSX = SLX_PF_SX;      // activation ring stages (one chunk each)
constexpr int kSW = SLX_PF_SW;      // weight ring stages (one chunk each)
constexpr int kThreads = 448;
constexpr int kDqThreads = 256;     // one weight row each
constexpr int kDqDepth = 4;         // cp.async chunks in flight per thread
constexpr int kTmemCols = 512;      // two 256-column accumulators
constexpr float kF16Max = 65504.f;   // largest finite fp16
constexpr float kTiny = 7.62939453125e-06f;  // 2^-17: smaller loses bits

// Tuning (compile-time; the defaults are the shipped configuration).
#ifndef SLX_PF_L2_PREFETCH
#define SLX_PF_L2_PREFETCH 1  // prefetch activation chunks one ring ahead into L2
#endif
#ifndef SLX_PF_SLEEP_WAIT
#define SLX_PF_SLEEP_WAIT 1   // barrier polls with a suspend-time hint
#endif

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
  int nG, nC;          // this phase: groups along K, chunks incl. bias chunks
  const uint8_t* ximg; // this phase's activation image [n_blocks][nC][kNT][128]
  uint8_t* himg;       // phase 1 output: phase 2's activation image
  int nG2, nC2;
  uint16_t* out;       // phase 2: [n_out, H] bf16
  const int32_t* out_row;
  int n_out;
  int32_t* status;
  int off_x, off_w, off_stg, off_btab;  // from the aligned base
};

namespace {

SLX_DEV bool block_ok(const PrefillArgs& a, int4 bl) {
  return bl.x >= 0 && bl.x < a.n_slots && bl.z >= 1 && bl.z <= kNT &&
         bl.y >= 0 && (long long)bl.y + bl.z <= a.n_pairs;
}

// Cursor over this CTA's (item, chunk) tasks; invalid blocks are skipped by
// every role alike.  An item is (block, 128 I rows) in phase 1 and
// (block, 256 H rows) in phase 2.
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
SLX_DEV void cur_next(const PrefillArgs& a, Cur& t) {
  if (++t.c == a.nC) cur_next_item(a, t);
}

SLX_DEV int npad16(int n) { return (n + 15) & ~15; }
SLX_DEV int bias_ksteps(int nG, int cb) {  // issued K steps of bias chunk cb
  const int cols = 2 * nG - 64 * cb;
  const int k = (cols + 15) / 16;
  return k > 4 ? 4 : k;
}

// Where weight row n (this thread) of an item reads its packed codes: the
// row's first byte, its swizzle key, and its scale|bias word of group 0
// with the word stride between groups (computed once per item).
struct RowSrc {
  const uint8_t* row;
  const uint32_t* sb;
  int swz, sbs, j;
};
template <int PHASE>
SLX_DEV void row_src(const PrefillArgs& a, int slot, int mb, int n, RowSrc& o) {
  const uint8_t* e = a.bank + (size_t)slot * a.slot_stride;
  if (PHASE == 1) {  // n < 128: gate row mb*128 + n, else up row mb*128 + n - 128
    const int RB = tile_rb(a.H, 2);
    const int r = mb * 128 + (n & 127), mat = n >> 7;
    const int t = r >> 4, tr = r & 15;
    const uint8_t* base = e + (size_t)t * pair_tile_bytes(a.H, 2);
    o.row = base + (size_t)(mat * 16 + tr) * RB;
    o.swz = tile_swizzled(a.H, 2) ? (tr & 7) : 0;
    o.sb = reinterpret_cast<const uint32_t*>(base + 32 * RB) + mat * 16 + tr;
    o.sbs = 32;
  } else {           // down row mb*256 + n
    const int RB = tile_rb(a.I, 2);
    const int r = mb * kNW + n;
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

template <int PHASE>
__global__ void __launch_bounds__(kThreads, 1)
    k_prefill(const __grid_constant__ PrefillArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint64_t* bar_tx = reinterpret_cast<uint64_t*>(smem_raw);  // [kSX] activations landed
  uint64_t* bar_xfree = bar_tx + kSX;                        // [kSX] activation slot consumed
  uint64_t* bar_dq = bar_xfree + kSX;                        // [kSW] weights written
  uint64_t* bar_wfree = bar_dq + kSW;                        // [kSW] weight slot consumed
  uint64_t* bar_full = bar_wfree + kSW;                      // [2] accumulator ready
  uint64_t* bar_free = bar_full + 2;                         // [2] accumulator drained
  uint64_t* bar_done = bar_free + 2;                         // all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // 1024-aligned region for the swizzled operand rings
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - ((raw + 256u) & 1023u)) & 1023u) + 256;
  uint8_t* sX = base + a.off_x;
  uint8_t* sW = base + a.off_w;
  uint8_t* stg = base + a.off_stg;
  __half* btab = reinterpret_cast<__half*>(base + a.off_btab);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSX; ++i) {
      mbar_init(&bar_tx[i], 1);
      mbar_init(&bar_xfree[i], 1);
    }
    for (int i = 0; i < kSW; ++i) {
      mbar_init(&bar_dq[i], kDqThreads / 32);
      mbar_init(&bar_wfree[i], 1);
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
    // ------------------------------------------- activation producer ----
    if (lane == 0) {
      Cur t, pb;  // pb runs one ring ahead: its chunks are prefetched to L2
      cur_init(a, t);
      cur_init(a, pb);
      for (int i = 0; i < kSX && !pb.end; ++i) cur_next(a, pb);
      uint32_t g = 0;
      for (; !t.end && !*abort_flag; cur_next(a, t), ++g) {
        const int st = g % kSX;
        if (SLX_PF_L2_PREFETCH && !pb.end) {
          bulk_prefetch_l2(a.ximg + ((size_t)pb.blk * a.nC + pb.c) * kActB,
                           (uint32_t)npad16(pb.n) * kRowB);
          cur_next(a, pb);
        }
        if (!mbar_wait_sleep(&bar_xfree[st], ((g / kSX) & 1) ^ 1, a.status)) {
          fail(SLX_ERR_DEVICE_TIMEOUT);
          break;
        }
        PF_STAMP(g, 0);
        const uint32_t bytes = (uint32_t)npad16(t.n) * kRowB;
        mbar_arrive_expect_tx(&bar_tx[st], bytes);
        bulk_g2s_plain(sX + (size_t)st * kActB,
                       a.ximg + ((size_t)t.blk * a.nC + t.c) * kActB, bytes,
                       &bar_tx[st]);
        PF_STAMP(g, 1);
      }
      // drain: every issued copy has landed before the CTA exits
      const uint32_t issued = g;
      for (uint32_t h = issued > kSX ? issued - kSX : 0; h < issued; ++h)
        mbar_wait(&bar_tx[h % kSX], (h / kSX) & 1, a.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issue ----
    if (lane == 0) {
      Cur t;
      cur_init(a, t);
      uint32_t g = 0;
      int jl = 0;
      bool ok = true;
      const uint32_t idesc = idesc_f16(kNW);  // M 128 pairs, N 256 weight rows
      while (!t.end && ok && !*abort_flag) {
        const int buf = jl & 1;
        if (!mbar_wait(&bar_free[buf], ((jl >> 1) & 1) ^ 1, a.status)) {
          fail(SLX_ERR_DEVICE_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * kNW;
        for (int c = 0; c < a.nC; ++c, ++g) {
          const int sx = g % kSX, sw = g % kSW;
          bool okw = mbar_wait(&bar_tx[sx], (g / kSX) & 1, a.status);
          PF_STAMP(g, 2);
          okw = okw && mbar_wait(&bar_dq[sw], (g / kSW) & 1, a.status);
          PF_STAMP(g, 3);
          if (!okw) {
            fail(SLX_ERR_DEVICE_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const int nk = c < a.nG ? 4 : bias_ksteps(a.nG, c - a.nG);
          const uint32_t x0 = smem_u32(sX + (size_t)sx * kActB);
          const uint32_t w0 = smem_u32(sW + (size_t)sw * kWB);
          for (int s = 0; s < nk; ++s)
            tc_mma_ss(d, sdesc_sw128(x0 + 32 * s), sdesc_sw128(w0 + 32 * s),
                      idesc, (c | s) != 0);
          tc_commit(&bar_xfree[sx]);
          tc_commit(&bar_wfree[sw]);
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
    // thread = pair m of the block (TMEM lane); columns = weight rows
    const int q = warp & 3;
    const int m = 32 * q + lane;
    Cur t;
    cur_init(a, t);
    int jl = 0;
    while (!t.end) {
      const int buf = jl & 1;
      const bool ok = __all_sync(0xffffffffu,
                                 mbar_wait_sleep(&bar_full[buf], (jl >> 1) & 1, a.status));
      if (!ok) fail(SLX_ERR_DEVICE_TIMEOUT);
      if (__any_sync(0xffffffffu, !ok || *abort_flag != 0)) break;
      tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + buf * kNW;
      const bool valid = m < t.n;
      if (PHASE == 1) {
        // columns 0..127 gate, 128..255 up of I rows mb*128 + 0..127: two
        // groups of 64 = two chunks of phase 2's activation image
        for (int jg = 0; jg < 2; ++jg) {
          const int chunk = t.mb * 2 + jg;
          uint8_t* dst = a.himg + ((size_t)t.blk * a.nC2 + chunk) * kActB +
                         (size_t)m * kRowB;
          float hs = 0.f;
          for (int cc = 0; cc < 64; cc += 16) {
            uint32_t gv[16], uv[16];
            tc_ld16(tq + 64 * jg + cc, gv);
            tc_ld16(tq + 128 + 64 * jg + cc, uv);
            tc_wait_ld();
            float h[16];
            bool big = false;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float gt = round_bf16(__uint_as_float(gv[i]));
              const float up = round_bf16(__uint_as_float(uv[i]));
              h[i] = round_bf16(silu_f32(gt) * up);
              hs += h[i];
              big |= !(fabsf(h[i]) < kF16Max);
            }
            if (valid && (big || !(fabsf(hs) < kF16Max)))
              set_status(a.status, SLX_ERR_RANGE);
            // 16 I rows 16w..16w+15 of the group fill positions 16w..16w+15
            // (permuted order): word j = (h[j], h[j+8]), units 2w and 2w+1
            uint32_t hw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              hw[j] = (uint32_t)h_bits(__float2half_rn(h[j])) |
                      ((uint32_t)h_bits(__float2half_rn(h[j + 8])) << 16);
            if (valid) {
              const int w = cc >> 4;
              *reinterpret_cast<uint4*>(dst + (((2 * w) ^ (m & 7)) << 4)) =
                  make_uint4(hw[0], hw[1], hw[2], hw[3]);
              *reinterpret_cast<uint4*>(dst + (((2 * w + 1) ^ (m & 7)) << 4)) =
                  make_uint4(hw[4], hw[5], hw[6], hw[7]);
            }
          }
          if (valid) {
            const __half hi = __float2half_rn(hs);
            const __half lo = __float2half_rn(hs - __half2float(hi));
            uint8_t* bd = a.himg +
                          ((size_t)t.blk * a.nC2 + a.nG2 + (chunk >> 5)) * kActB +
                          sw_off(m, 2 * (chunk & 31));
            *reinterpret_cast<uint32_t*>(bd) =
                (uint32_t)h_bits(hi) | ((uint32_t)h_bits(lo) << 16);
          }
        }
      } else {
        int row = -1;
        if (valid) {
          const int p = t.p0 + m;
          row = a.out_row ? a.out_row[p] : p;
          if (row < 0 || row >= a.n_out) {
            set_status(a.status, SLX_ERR_OUT_OF_RANGE);
            row = -1;
          }
        }
        uint16_t* orow = row >= 0 ? a.out + (size_t)row * a.H + t.mb * kNW : nullptr;
        for (int cc = 0; cc < kNW; cc += 16) {
          uint32_t v[16];
          tc_ld16(tq + cc, v);
          tc_wait_ld();
          if (orow) {
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              o[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
            uint4* dp = reinterpret_cast<uint4*>(orow + cc);
            dp[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dp[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_free[buf]);
      ++jl;
      cur_next_item(a, t);
    }
  } else {
    // -------------------------------------------------- dequantization ----
    const int n = threadIdx.x - 192;  // weight row of the item, 0..255
    // staging, thread-contiguous (conflict-free): codes [slot][row] 16
    // bytes, then scale|bias words [slot][row] 4 bytes
    uint4* stg_codes = reinterpret_cast<uint4*>(stg);
    uint32_t* stg_sb = reinterpret_cast<uint32_t*>(stg + kDqDepth * kDqThreads * 16);
    Cur pf, cu;
    cur_init(a, pf);
    cur_init(a, cu);
    RowSrc rs;
    rs.j = -1;
    auto issue = [&](int slot) {
      if (!pf.end && pf.c < a.nG) {
        if (rs.j != pf.j) {
          row_src<PHASE>(a, pf.slot, pf.mb, n, rs);
          rs.j = pf.j;
        }
        const int u = slot * kDqThreads + n;
        cp_async16(smem_u32(stg_codes + u), rs.row + ((pf.c ^ rs.swz) << 4));
        cp_async4(smem_u32(stg_sb + u), rs.sb + pf.c * rs.sbs);
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
      const int c = cu.c;
      uint4 cw = make_uint4(0, 0, 0, 0);
      uint32_t sbw = 0;
      if (c < a.nG) {
        cw = stg_codes[slot * kDqThreads + n];
        sbw = stg_sb[slot * kDqThreads + n];
      }
      issue(slot);
      cur_next(a, pf);
      const int sw = g % kSW;
      const bool ok = mbar_wait_sleep(&bar_wfree[sw], ((g / kSW) & 1) ^ 1, a.status);
      if (warp == 6 && lane == 0) PF_STAMP(g, 6);
      if (!__all_sync(0xffffffffu, ok)) {
        fail(SLX_ERR_DEVICE_TIMEOUT);
        break;
      }
      uint32_t out[32];
      if (c < a.nG) {
        {  // operand range of the exact fp16 affine form (see the top)
          const float fs = fabsf(bf16_lo(sbw)), fb = fabsf(bf16_hi(sbw));
          const bool bad = !(fs < 64.f) || (fs != 0.f && fs < kTiny) ||
                           !(fb < kF16Max) || (fb != 0.f && fb < kTiny);
          if (__any_sync(0xffffffffu, bad) && lane == 0)
            set_status(a.status, SLX_ERR_RANGE);
        }
        const __half s16 = __float2half_rn(bf16_lo(sbw));
        // this thread's row only: written here, read back at the bias chunk
        btab[c * kDqThreads + n] = __float2half_rn(bf16_hi(sbw));
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
          const uint32_t hb = gi < a.nG ? h_bits(btab[gi * kDqThreads + n]) : 0u;
          out[k2] = hb | (hb << 16);
        }
      }
      uint8_t* rowp = sW + (size_t)sw * kWB + (n >> 3) * 1024 + (n & 7) * kRowB;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int pu = u ^ (n & 7);
        *reinterpret_cast<uint4*>(rowp + pu * 16) =
            make_uint4(out[4 * u], out[4 * u + 1], out[4 * u + 2], out[4 * u + 3]);
      }
      fence_proxy_async();
      __syncwarp();
      if (warp == 6 && lane == 0) PF_STAMP(g, 7);
      if (lane == 0) mbar_arrive(&bar_dq[sw]);
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
  // a bad row index is reported and the pair's image row written as zeros,
  // so its (skipped-in-spirit) output is deterministic
  const bool row_ok = xr >= 0 && xr < n_rows;
  if (!row_ok && lane == 0) set_status(status, SLX_ERR_OUT_OF_RANGE);
  const uint16_t* xrow = x + (size_t)(row_ok ? xr : 0) * H;
  uint8_t* blk = img + (size_t)b * nC * kActB;
  const int u = lane & 7;            // 16-byte unit of the chunk row
  const int i = u >> 1, j0 = 4 * (u & 1);
  bool big = false;
  for (int c0 = 0; c0 < nG; c0 += 4) {
    const int c = c0 + (lane >> 3);
    const uint16_t* src = xrow + 64 * c + 16 * i + j0;
    uint2 lo4 = make_uint2(0, 0), hi4 = make_uint2(0, 0);
    if (row_ok) {
      lo4 = *reinterpret_cast<const uint2*>(src);      // elements j0..j0+3
      hi4 = *reinterpret_cast<const uint2*>(src + 8);  // j0+8..j0+11
    }
    const uint32_t lw[4] = {lo4.x & 0xFFFFu, lo4.x >> 16, lo4.y & 0xFFFFu, lo4.y >> 16};
    const uint32_t hw[4] = {hi4.x & 0xFFFFu, hi4.x >> 16, hi4.y & 0xFFFFu, hi4.y >> 16};
    uint32_t o[4];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a0 = bf16_to_f32((uint16_t)lw[k]);
      const float a1 = bf16_to_f32((uint16_t)hw[k]);
      big |= !(fabsf(a0) < kF16Max) || !(fabsf(a1) < kF16Max);
      s += a0 + a1;
      o[k] = (uint32_t)h_bits(__float2half_rn(a0)) |
             ((uint32_t)h_bits(__float2half_rn(a1)) << 16);
    }
    *reinterpret_cast<uint4*>(blk + (size_t)c * kActB + n * kRowB +
                              ((u ^ (n & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    big |= !(fabsf(s) < kF16Max);
    if (u == 0) {
      const __half hi = __float2half_rn(s);
      const __half lo = __float2half_rn(s - __half2float(hi));
      const int pos = 2 * (c & 31);
      *reinterpret_cast<uint32_t*>(blk + (size_t)(nG + (c >> 5)) * kActB +
                                   n * kRowB + ((((pos >> 3) ^ (n & 7))) << 4) +
                                   ((pos & 7) << 1)) =
          (uint32_t)h_bits(hi) | ((uint32_t)h_bits(lo) << 16);
    }
  }
  if (__any_sync(0xffffffffu, big) && lane == 0 && row_ok)
    set_status(status, SLX_ERR_RANGE);
}

// ------------------------------------------------------------ launchers --

namespace {

int pf_chunks(int nG) { return nG + (nG + 31) / 32; }

struct SmemPlan {
  int off_x, off_w, off_stg, off_btab, bytes;
};

SmemPlan plan_smem(int nG) {
  SmemPlan p = {};
  int o = 0;
  p.off_x = o;    o += kSX * kActB;
  p.off_w = o;    o += kSW * kWB;
  p.off_stg = o;  o += kDqDepth * kDqThreads * (16 + 4);
  p.off_btab = o; o += nG * kDqThreads * 2;
  // + barrier area (256) + worst-case 1024 alignment; at least 120 KB so one
  // CTA (and one 512-column TMEM allocation) per SM
  int bytes = o + 256 + 1024;
  if (bytes < 120 * 1024) bytes = 120 * 1024;
  p.bytes = bytes;
  return p;
}

PerDevice g_num_sms_pf;

template <int PHASE>
int launch_phase(PrefillArgs a, int smem, cudaStream_t s, int n_sms) {
  static PerDevice attr_set;
  std::atomic<int>& slot = attr_set.here();
  if (!slot.load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(k_prefill<PHASE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return SLX_ERR_CUDA;
    slot.store(1, std::memory_order_relaxed);
  }
  if (a.n_items == 0) return SLX_OK;
  const int grid = a.n_items < n_sms ? a.n_items : n_sms;
  k_prefill<PHASE><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? SLX_OK : SLX_ERR_CUDA;
}

}  // namespace

size_t prefill_scratch_bytes(int n_blocks, int H, int I) {
  const size_t c1 = pf_chunks(H / 64), c2 = pf_chunks(I / 64);
  return (size_t)n_blocks * (c1 + c2) * kActB;
}

int launch_prefill(const uint8_t* bank, long long slot_stride, int n_slots,
                   int H, int I, const uint16_t* x, int n_rows,
                   const int32_t* pair_row, int n_pairs, const int4* blocks,
                   int n_blocks, const int32_t* out_row, uint16_t* out,
                   int n_out, uint8_t* scratch, int32_t* status,
                   cudaStream_t s) {
  std::atomic<int>& sm_slot = g_num_sms_pf.here();
  int n_sms = sm_slot.load(std::memory_order_relaxed);
  if (n_sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount,
                               dev) != cudaSuccess || n_sms <= 0)
      return SLX_ERR_CUDA;
    sm_slot.store(n_sms, std::memory_order_relaxed);
  }
  const int nG1 = H / 64, nG2 = I / 64;
  if (nG1 > 64 || nG2 > 64 || I % 128 || H % kNW) return SLX_ERR_UNSUPPORTED;
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
  uint8_t* himg = scratch + (size_t)n_blocks * pf_chunks(nG1) * kActB;
  a.himg = himg;
  a.out = out;
  a.out_row = out_row;
  a.n_out = n_out;

  // phase 0: gather x rows into phase 1's activation image
  {
    dim3 grid(n_blocks, kNT / 8);
    k_pf_pack_x<<<grid, 256, 0, s>>>(x, n_rows, H, pair_row, blocks, n_blocks,
                                     n_pairs, n_slots, nG1, pf_chunks(nG1),
                                     ximg, status);
    if (cudaGetLastError() != cudaSuccess) return SLX_ERR_CUDA;
  }
  // phase 1: gate/up -> SwiGLU -> phase 2's activation image
  {
    PrefillArgs p = a;
    p.nG = nG1;
    p.nC = pf_chunks(nG1);
    p.n_mb = I / 128;
    p.n_items = n_blocks * p.n_mb;
    p.ximg = ximg;
    const SmemPlan sp = plan_smem(nG1);
    p.off_x = sp.off_x; p.off_w = sp.off_w; p.off_stg = sp.off_stg;
    p.off_btab = sp.off_btab;
    if (sp.bytes > 227 * 1024) return SLX_ERR_UNSUPPORTED;
    const int rc = launch_phase<1>(p, sp.bytes, s, n_sms);
    if (rc) return rc;
  }
  // phase 2: down projection -> per-pair outputs
  {
    PrefillArgs p = a;
    p.nG = nG2;
    p.nC = pf_chunks(nG2);
    p.n_mb = H / kNW;
    p.n_items = n_blocks * p.n_mb;
    p.ximg = himg;
    const SmemPlan sp = plan_smem(nG2);
    p.off_x = sp.off_x; p.off_w = sp.off_w; p.off_stg = sp.off_stg;
    p.off_btab = sp.off_btab;
    if (sp.bytes > 227 * 1024) return SLX_ERR_UNSUPPORTED;
    const int rc = launch_phase<2>(p, sp.bytes, s, n_sms);
    if (rc) return rc;
  }
  return SLX_OK;
}

}  // namespace slx
