// Shared device helpers for the streamlx B200 kernels (sm_100a).
//
// Everything here is hand-written PTX or plain CUDA: mbarrier + bulk-copy
// (TMA engine, one CTA per copy) staging, mma.sync bf16 fragments, and the
// magic-number unpack of MLX-affine 2/4/8-bit codes into bf16 pairs.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "../../include/streamlx_cuda.h"

#define SLX_DEV __device__ __forceinline__
#define SLX_HOST_DEV __host__ __device__ __forceinline__

namespace slx {

// ----------------------------------------------------------------- bf16 ---

SLX_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
SLX_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
SLX_DEV float bf16_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

SLX_DEV uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&b);
}
SLX_DEV float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

SLX_DEV uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

// ------------------------------------------------------------ addresses ---

SLX_DEV uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// -------------------------------------------------------------- mbarrier ---

SLX_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

SLX_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

SLX_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

SLX_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

SLX_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

SLX_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait in these kernels is bounded: after kWaitLimitNs the waiter
// records SLX_ERR_DEVICE_TIMEOUT in the caller's status word and gives up,
// so a logic error surfaces as a status code instead of a hung GPU.
constexpr uint64_t kWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

SLX_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicCAS(status, 0, SLX_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------------------ bulk copy ---

// L2 policy for streamed-once weight bytes.
SLX_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy on the TMA engine, completion counted on `bar`.
// dst, src and bytes must be 16-byte aligned / multiples of 16.
SLX_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                      uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes."
      "L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Same without an L2 policy (data that other CTAs read too).
SLX_DEV void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes,
                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Generic-proxy global writes before async-proxy (bulk copy) accesses.
SLX_DEV void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Start reading [src, src + bytes) from DRAM into L2 (no completion to
// wait for).  src and bytes: 16-byte aligned / multiple of 16.
SLX_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes)
               : "memory");
}

// ------------------------------------------------------------------ PDL ---
//
// Every kernel of the library lets its dependent grid launch at once
// (launch_dependents at entry) and executes griddepcontrol.wait before it
// reads anything a preceding kernel wrote or writes any global memory; only
// reads of immutable weights may come before the wait.  Both instructions
// are no-ops for a grid launched without the programmatic-serialization
// attribute, so the same code is correct with and without PDL.

SLX_DEV void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
SLX_DEV void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launch setting of the calling host thread (slx_set_pdl).
bool pdl_enabled();

// A launcher's one-time per-device value (function attributes and occupancy
// apply per device context; slots for devices 0..63, 0 = not yet known).
constexpr int kMaxDevices = 64;
struct PerDevice {
  std::atomic<int> v[kMaxDevices];
  // the slot of the calling thread's current device
  std::atomic<int>& here() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) d = 0;
    return v[d];
  }
};

// <<<>>> replacement that adds the PDL attribute when pdl_enabled().
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                     size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------ MMA ---

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
SLX_DEV void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                           uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                           const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// ------------------------------------------------------- affine unpack ---
//
// A code q sitting at bit s of a 16-bit half, with every other bit of that
// half clear, is the IEEE fp16 subnormal q * 2^s * 2^-24 -- exactly, for
// q * 2^s < 1024.  So a single AND with a two-lane mask turns two packed
// codes (one per 16-bit half of a word) into an fp16 pair the tensor core
// multiplies exactly: no offset to cancel, no conversion instructions.  The
// 2^s factor is undone by pre-scaling the matching activation by 2^-s
// (power of two: exact), and the common 2^-24 by scaling the group's fp32
// result by 2^24 in the fold (slx_qgemv.cu).

constexpr float kSubnormalUnit = 16777216.0f;  // 2^24

// 2-bit: word holds 16 codes (code v at bits 2v).  R[j] = {q[v], q[v+8]}
// times 4^c, with v = j, c = j for j < 5 (no shift) and v = j, c = j - 5 on
// the word shifted right by 10 (j = 5..7).
SLX_DEV void unpack2(uint32_t w, uint32_t (&r)[8]) {
  const uint32_t w10 = w >> 10;
  r[0] = w & 0x00030003u;
  r[1] = w & 0x000C000Cu;
  r[2] = w & 0x00300030u;
  r[3] = w & 0x00C000C0u;
  r[4] = w & 0x03000300u;
  r[5] = w10 & 0x00030003u;
  r[6] = w10 & 0x000C000Cu;
  r[7] = w10 & 0x00300030u;
}

// 4-bit: two words (8 codes each, code v at bits 4v) -> 8 pairs.
// R[j] = {q0[j], q0[j+4]} * 16^(j&1) for j < 4, R[4+j] likewise from w1.
SLX_DEV void unpack4(uint32_t w0, uint32_t w1, uint32_t (&r)[8]) {
  const uint32_t a8 = w0 >> 8, b8 = w1 >> 8;
  r[0] = w0 & 0x000F000Fu;
  r[1] = w0 & 0x00F000F0u;
  r[2] = a8 & 0x000F000Fu;
  r[3] = a8 & 0x00F000F0u;
  r[4] = w1 & 0x000F000Fu;
  r[5] = w1 & 0x00F000F0u;
  r[6] = b8 & 0x000F000Fu;
  r[7] = b8 & 0x00F000F0u;
}

// 8-bit: four words (4 codes each) -> 8 pairs; R[2i] = {b0, b2} of word i,
// R[2i+1] = {b1, b3}.  Codes < 256 < 1024: no scaling.
SLX_DEV void unpack8(const uint32_t (&w)[4], uint32_t (&r)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r[2 * i] = w[i] & 0x00FF00FFu;
    r[2 * i + 1] = (w[i] >> 8) & 0x00FF00FFu;
  }
}

// Local column (0..15 within a thread's 16-column slice of a group) carried
// by the low / high half of unpack register j, per bit width.
SLX_DEV int col_lo(int bits, int j) {
  if (bits == 2) return j;
  if (bits == 4) return j < 4 ? j : 8 + (j - 4);
  return 4 * (j >> 1) + (j & 1);  // 8-bit
}
SLX_DEV int col_hi(int bits, int j) {
  if (bits == 2) return j + 8;
  if (bits == 4) return col_lo(4, j) + 4;
  return col_lo(8, j) + 2;
}
// factor applied to the activation matching local column c (inverse of the
// power of two the unpack leaves on that code)
SLX_DEV float act_scale(int bits, int c) {
  if (bits == 2) {
    const int j = c & 7;
    const int k = j < 5 ? j : j - 5;
    return __int_as_float((127 - 2 * k) << 23);  // 4^-k
  }
  if (bits == 4) return (c & 1) ? 0.0625f : 1.f;
  return 1.f;
}

SLX_DEV uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

SLX_DEV float silu_f32(float g) { return g / (1.f + __expf(-g)); }

// Timeline trace points: compiled out unless the library is built with
// -DSLX_TRACE (a diagnostics build; records %globaltimer per CTA).
#ifdef SLX_TRACE
#define SLX_TRACE_POINT(K, I)                                          \
  do {                                                                 \
    if (threadIdx.x == 32 && blockIdx.x < 160)                         \
      ::g_slx_trace[K][blockIdx.x][I] = slx::globaltimer_ns();         \
  } while (0)
#define SLX_TRACE_AT(K, I, V)                                          \
  do {                                                                 \
    if (blockIdx.x < 160) ::g_slx_trace[K][blockIdx.x][I] = (V);       \
  } while (0)
#define SLX_TRACE_SMID(K)                                              \
  do {                                                                 \
    unsigned smid_;                                                    \
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid_));                 \
    if (threadIdx.x == 32 && blockIdx.x < 160)                         \
      ::g_slx_trace[K][blockIdx.x][15] = smid_;                        \
  } while (0)
#else
#define SLX_TRACE_POINT(K, I) \
  do {                        \
  } while (0)
#define SLX_TRACE_SMID(K) \
  do {                    \
  } while (0)
#define SLX_TRACE_AT(K, I, V) \
  do {                        \
  } while (0)
#endif

// Ticket of a "last CTA finishes the job" pattern: call after a
// __syncthreads() that follows the CTA's global writes, from one thread.
// The release half publishes this CTA's writes (ordered before it by the
// barrier); the acquire half lets the last CTA read every other CTA's
// writes (through L2: use ld.cg / __ldcg) after its own __syncthreads().
SLX_DEV int ticket_acq_rel(int32_t* counter) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
               : "=r"(old) : "l"(counter) : "memory");
  return old;
}

SLX_DEV void set_status(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace slx
