// extern "C" entry points of libstreamlx_cuda.so (declared in
// include/streamlx_cuda.h).  Host-side argument checks, then the launchers.
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <vector>

#include "slx_kernels.cuh"
#include "slx_tiles.cuh"

namespace {

thread_local std::string g_err;
thread_local int g_pdl = 0;
thread_local int g_fused = 1;
thread_local int g_glu_kernels = 0;  // kernels the last slx_switchglu launched

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_check(int rc, const char* what) {
  if (rc == SLX_ERR_CUDA) {
    cudaError_t e = cudaGetLastError();
    return fail(rc, "%s: %s", what, cudaGetErrorString(e));
  }
  if (rc == SLX_ERR_UNSUPPORTED) return fail(rc, "%s: unsupported shape", what);
  if (rc != SLX_OK) return fail(rc, "%s: error %d", what, rc);
  return SLX_OK;
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

bool qmat_ok(const slx_qmat& m) {
  return m.weight && m.scales && m.biases && aligned16(m.weight) &&
         aligned16(m.scales) && aligned16(m.biases);
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

namespace slx {
bool pdl_enabled() { return g_pdl != 0; }
}  // namespace slx

extern "C" {

int slx_version(void) { return 1; }

int slx_set_pdl(int on) {
  const int prev = g_pdl;
  g_pdl = on ? 1 : 0;
  return prev;
}

const char* slx_last_error_string(void) { return g_err.c_str(); }

// scratch = SwiGLU output of every routed unit and of the shared expert, in
// the down projection's fragment layout: per unit (in/64) x 32 words of fp16
// pairs + (in/64) x 4 partial sums.
size_t slx_switchglu_scratch_bytes(int T, int k, int inter, int shared_inter) {
  if (T < 0 || k < 0 || inter < 0 || shared_inter < 0) return 0;
  const size_t u = (size_t)T * k, ng = inter / 64, ngs = shared_inter / 64;
  // the first 256 bytes: grid-barrier words of the fused decode kernel (at
  // a fixed place, so calls of any shape sharing one scratch agree on them)
  return 256 + align256(u * ng * 128) + align256(u * ng * 16) +
         align256((size_t)T * ngs * 128) + align256((size_t)T * ngs * 16);
}

size_t slx_expert_tiled_bytes(int hidden, int inter, int bits) {
  if (hidden <= 0 || inter <= 0 || hidden % 64 || inter % 64) return 0;
  return slx::expert_tiled_bytes(hidden, inter, bits);
}

size_t slx_dense_tiled_bytes(int out_features, int in_features, int bits) {
  if (out_features <= 0 || in_features <= 0 || in_features % 64) return 0;
  return slx::dense_tiled_bytes(out_features, in_features, bits);
}

int slx_pack_experts(const slx_qmat* gate, const slx_qmat* up,
                     const slx_qmat* down, int n, int hidden, int inter,
                     int bits, void* const* dst, void* stream) {
  g_err.clear();
  if (n < 0 || (n > 0 && (!gate || !up || !down || !dst)))
    return fail(SLX_ERR_INVALID, "pack_experts: bad arrays");
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(SLX_ERR_UNSUPPORTED, "bits %d", bits);
  if (hidden <= 0 || inter <= 0 || hidden % 64 || inter % 64)
    return fail(SLX_ERR_INVALID, "hidden %d inter %d", hidden, inter);
  std::vector<const void*> v[9];
  for (int e = 0; e < n; ++e) {
    const slx_qmat* m[3] = {&gate[e], &up[e], &down[e]};
    for (int p = 0; p < 3; ++p) {
      if (!qmat_ok(*m[p])) return fail(SLX_ERR_INVALID, "expert %d part %d", e, p);
      v[3 * p].push_back(m[p]->weight);
      v[3 * p + 1].push_back(m[p]->scales);
      v[3 * p + 2].push_back(m[p]->biases);
    }
    if (!dst[e] || !aligned16(dst[e]))
      return fail(SLX_ERR_INVALID, "dst[%d] NULL or misaligned", e);
  }
  if (n == 0) return SLX_OK;
  const int rc = slx::launch_pack_experts(
      v[0].data(), v[1].data(), v[2].data(), v[3].data(), v[4].data(),
      v[5].data(), v[6].data(), v[7].data(), v[8].data(), dst, n, hidden,
      inter, bits, reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_pack_experts") : SLX_OK;
}

int slx_pack_dense(const slx_qmat* w, int out_features, int in_features,
                   int bits, void* dst, void* stream) {
  g_err.clear();
  if (!w || !qmat_ok(*w) || !dst || !aligned16(dst))
    return fail(SLX_ERR_INVALID, "pack_dense: bad pointers");
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(SLX_ERR_UNSUPPORTED, "bits %d", bits);
  if (out_features <= 0 || in_features <= 0 || in_features % 64)
    return fail(SLX_ERR_INVALID, "pack_dense shape %d x %d", out_features,
                in_features);
  const int rc = slx::launch_pack_dense(w->weight, w->scales, w->biases,
                                        out_features, in_features, bits, dst,
                                        reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_pack_dense") : SLX_OK;
}

static int switchglu_impl(const slx_expert_bank* bank,
                          const slx_shared_expert* shared, const void* x,
                          int T, int k, const int32_t* ids, const float* scores,
                          const int32_t* slot_table, int n_table, void* out,
                          void* scratch, size_t scratch_bytes, int32_t* status,
                          void* stream, const slx_fill_service* svc,
                          const slx_ep_exchange* ep = nullptr);

static bool ep_ok(const slx_ep_exchange* ep) {
  if (!ep || ep->n_ranks < 1 || ep->n_ranks > SLX_EP_MAX_RANKS ||
      ep->rank < 0 || ep->rank >= ep->n_ranks || ep->layer < 0 ||
      ep->layer >= ep->n_layers || !ep->stamp || ep->grid < 0 ||
      ep->wait_ns <= 0)
    return false;
  for (int r = 0; r < ep->n_ranks; ++r)
    if (!ep->recv[r] || !ep->count[r] || !aligned16(ep->recv[r])) return false;
  return true;
}

int slx_ep_grid(void) {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
          cudaSuccess)
    return fail(SLX_ERR_CUDA, "slx_ep_grid: no device");
  return n;
}

int slx_switchglu_ep(const slx_expert_bank* bank,
                     const slx_shared_expert* shared, const void* x, int k,
                     const int32_t* ids, const float* scores,
                     const int32_t* slot_table, int n_table, void* scratch,
                     size_t scratch_bytes, int32_t* status,
                     const slx_ep_exchange* ep, void* stream) {
  g_err.clear();
  if (!ep_ok(ep)) return fail(SLX_ERR_INVALID, "switchglu_ep: bad exchange");
  if (!scores || !slot_table)
    return fail(SLX_ERR_INVALID, "switchglu_ep: scores and slot_table are "
                "required");
  if (ep->grid != slx_ep_grid())
    return fail(SLX_ERR_INVALID, "switchglu_ep: grid %d != %d", ep->grid,
                slx_ep_grid());
  // out is not written in this mode; the scratch doubles as a dummy
  return switchglu_impl(bank, shared, x, 1, k, ids, scores, slot_table,
                        n_table, scratch, scratch, scratch_bytes, status,
                        stream, nullptr, ep);
}

int slx_ep_combine_rmsnorm(const slx_ep_exchange* ep, const float* scores,
                           int k, int hidden, int has_shared,
                           const void* h_in, const void* weight, float eps,
                           void* h_out, void* y, int32_t* status,
                           void* stream) {
  g_err.clear();
  if (!ep_ok(ep)) return fail(SLX_ERR_INVALID, "ep_combine: bad exchange");
  if (!scores || !h_in || !weight || !h_out || !y || k < 1 ||
      !aligned16(h_in) || !aligned16(h_out) || !aligned16(y) ||
      !aligned16(weight))
    return fail(SLX_ERR_INVALID, "ep_combine: NULL/misaligned or k %d", k);
  const int rc = slx::launch_ep_combine_rmsnorm(
      *ep, scores, k, hidden, has_shared ? 1 : 0,
      reinterpret_cast<const uint16_t*>(h_in),
      reinterpret_cast<const uint16_t*>(weight), eps,
      reinterpret_cast<uint16_t*>(h_out), reinterpret_cast<uint16_t*>(y),
      status, reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_ep_combine_rmsnorm") : SLX_OK;
}

int slx_ipc_handle(const void* dev_ptr, void* handle64, int64_t* offset) {
  g_err.clear();
  if (!dev_ptr || !handle64 || !offset)
    return fail(SLX_ERR_INVALID, "ipc_handle: NULL");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SLX_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  // the handle names the whole allocation: locate dev_ptr inside it (the
  // driver call is reached through the runtime, so the library does not
  // link the driver and still loads on machines without one)
  using range_fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault,
                              &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn) {
    cudaGetLastError();
    return fail(SLX_ERR_CUDA, "cuMemGetAddressRange entry point not found");
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (reinterpret_cast<range_fn>(fn)(&base, &size, (CUdeviceptr)dev_ptr) !=
      CUDA_SUCCESS)
    return fail(SLX_ERR_CUDA, "cuMemGetAddressRange failed");
  std::memcpy(handle64, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)dev_ptr - base);
  return SLX_OK;
}

int slx_ipc_open(const void* handle64, void** base) {
  g_err.clear();
  if (!handle64 || !base) return fail(SLX_ERR_INVALID, "ipc_open: NULL");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  const cudaError_t e =
      cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SLX_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  }
  return SLX_OK;
}

int slx_ipc_close(void* base) {
  g_err.clear();
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SLX_ERR_CUDA, "cudaIpcCloseMemHandle: %s",
                cudaGetErrorString(e));
  }
  return SLX_OK;
}

int slx_switchglu(const slx_expert_bank* bank, const slx_shared_expert* shared,
                  const void* x, int T, int k, const int32_t* ids,
                  const float* scores, const int32_t* slot_table, int n_table,
                  void* out, void* scratch, size_t scratch_bytes,
                  int32_t* status, void* stream) {
  g_err.clear();
  return switchglu_impl(bank, shared, x, T, k, ids, scores, slot_table,
                        n_table, out, scratch, scratch_bytes, status, stream,
                        nullptr);
}

int slx_switchglu_serviced(const slx_expert_bank* bank,
                           const slx_shared_expert* shared, const void* x,
                           int k, const int32_t* ids, const float* scores,
                           int32_t* slot_table, int n_table, void* out,
                           void* scratch, size_t scratch_bytes,
                           int32_t* status, const slx_fill_service* svc,
                           void* stream) {
  g_err.clear();
  if (!svc) return fail(SLX_ERR_INVALID, "switchglu_serviced: svc is NULL");
  if (!scores || !slot_table)
    return fail(SLX_ERR_INVALID, "switchglu_serviced: scores and slot_table "
                "are required");
  if (k < 1 || k > SLX_FILL_MAX_K)
    return fail(SLX_ERR_UNSUPPORTED, "switchglu_serviced: k %d (1..%d)", k,
                SLX_FILL_MAX_K);
  if (svc->layer < 0 || svc->layer > 255 || svc->max_items < 0)
    return fail(SLX_ERR_INVALID, "switchglu_serviced: layer %d max_items %d",
                svc->layer, svc->max_items);
  if (!svc->stamp || !svc->park || !svc->release || !svc->desc || !svc->go ||
      !aligned16(svc->desc) || svc->wait_ns <= 0)
    return fail(SLX_ERR_INVALID, "switchglu_serviced: NULL/misaligned "
                "service pointer or wait_ns <= 0");
  if ((svc->pred_ids == nullptr) != (svc->pred_scores == nullptr))
    return fail(SLX_ERR_INVALID, "switchglu_serviced: pred_ids and "
                "pred_scores go together");
  return switchglu_impl(bank, shared, x, 1, k, ids, scores, slot_table,
                        n_table, out, scratch, scratch_bytes, status, stream,
                        svc);
}

static int switchglu_impl(const slx_expert_bank* bank,
                          const slx_shared_expert* shared, const void* x,
                          int T, int k, const int32_t* ids, const float* scores,
                          const int32_t* slot_table, int n_table, void* out,
                          void* scratch, size_t scratch_bytes, int32_t* status,
                          void* stream, const slx_fill_service* svc,
                          const slx_ep_exchange* ep) {
  if (!bank) return fail(SLX_ERR_INVALID, "slx_switchglu: bank is NULL");
  const int H = bank->hidden, I = bank->inter, bits = bank->bits;
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(SLX_ERR_UNSUPPORTED, "bits %d (2/4/8)", bits);
  if (H <= 0 || I <= 0 || H % 64 || I % 64)
    return fail(SLX_ERR_INVALID, "hidden %d / inter %d must be multiples of 64",
                H, I);
  if (T < 0 || k < 1 || bank->n_slots < 1)
    return fail(SLX_ERR_INVALID, "T %d k %d n_slots %d", T, k, bank->n_slots);
  if (bank->slot_stride < (int64_t)slx::expert_tiled_bytes(H, I, bits) ||
      bank->slot_stride % 16)
    return fail(SLX_ERR_INVALID, "slot_stride %lld", (long long)bank->slot_stride);
  if (T == 0) return SLX_OK;
  if (!x || !ids || !out || !aligned16(x) || !aligned16(out))
    return fail(SLX_ERR_INVALID, "x/ids/out NULL or not 16-byte aligned");
  if (!bank->base || !aligned16(bank->base))
    return fail(SLX_ERR_INVALID, "bank base NULL or misaligned");
  if (slot_table && n_table < 1)
    return fail(SLX_ERR_INVALID, "n_table %d", n_table);
  const bool use_shared = scores && shared;
  const int Is = use_shared ? shared->inter : 0;
  if (use_shared) {
    if (Is <= 0 || Is % 64) return fail(SLX_ERR_INVALID, "shared inter %d", Is);
    if (!shared->base || !aligned16(shared->base))
      return fail(SLX_ERR_INVALID, "shared expert base NULL or misaligned");
  }
  const size_t need = slx_switchglu_scratch_bytes(T, k, I, Is);
  if (!scratch || scratch_bytes < need || !aligned16(scratch))
    return fail(SLX_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  const size_t nu = (size_t)T * k, ng = I / 64, ngs = Is / 64;
  uint8_t* sp = reinterpret_cast<uint8_t*>(scratch);
  void* gbar = sp;  // 64-bit arrival counter of the fused kernel's barrier
  sp += 256;
  uint32_t* hfrag = reinterpret_cast<uint32_t*>(sp);
  sp += align256(nu * ng * 128);
  float* hpart = reinterpret_cast<float*>(sp);
  sp += align256(nu * ng * 16);
  uint32_t* hfrag_sh = reinterpret_cast<uint32_t*>(sp);
  sp += align256((size_t)T * ngs * 128);
  float* hpart_sh = reinterpret_cast<float*>(sp);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  slx::GemvArgs a = {};
  a.mode = SLX_GEMV_GLU;
  a.x = reinterpret_cast<const uint16_t*>(x);
  a.T = T;
  a.in = H;
  a.ids = ids;
  a.k = k;
  a.slot_table = slot_table;
  a.n_table = n_table;
  a.n_slots = bank->n_slots;
  a.bank = reinterpret_cast<const uint8_t*>(bank->base);
  a.slot_stride = bank->slot_stride;
  a.I = I;
  a.shared = use_shared ? reinterpret_cast<const uint8_t*>(shared->base) : nullptr;
  a.Is = Is;
  a.hfrag = hfrag;
  a.hpart = hpart;
  a.hfrag_sh = hfrag_sh;
  a.hpart_sh = hpart_sh;
  a.unit_frag_words = (int)ng * 32;
  a.unit_part_floats = (int)ng * 4;
  a.shared_frag_words = (int)ngs * 32;
  a.shared_part_floats = (int)ngs * 4;
  a.status = status;
  a.n_tiles = T * k * (I / 16) + T * (Is / 16);

  slx::DownArgs d = {};
  d.T = T;
  d.k = k;
  d.H = H;
  d.I = I;
  d.Is = Is;
  d.ids = ids;
  d.slot_table = slot_table;
  d.n_table = n_table;
  d.n_slots = bank->n_slots;
  d.scores = scores;
  d.bank = a.bank;
  d.slot_stride = bank->slot_stride;
  d.shared = a.shared;
  d.hfrag = hfrag;
  d.hpart = hpart;
  d.hfrag_sh = hfrag_sh;
  d.hpart_sh = hpart_sh;
  d.unit_frag_words = a.unit_frag_words;
  d.unit_part_floats = a.unit_part_floats;
  d.shared_frag_words = a.shared_frag_words;
  d.shared_part_floats = a.shared_part_floats;
  d.out = reinterpret_cast<uint16_t*>(out);
  d.status = status;
  d.n_items = T * (H / 16);
  d.n_units = k + (Is > 0 ? 1 : 0);
  d.pdl = 1;
  int rc = SLX_ERR_UNSUPPORTED;
  if ((g_fused || svc || ep) && T == 1) {
    // one cooperative launch for both phases when the token's tiles fit
    d.tile_bytes = (int)slx::single_tile_bytes(I, bits);
    d.tile_bytes_sh = Is ? (int)slx::single_tile_bytes(Is, bits) : 0;
    d.a_bytes = (long long)slx::expert_a_bytes(H, I, bits);
    d.a_bytes_sh = Is ? (long long)slx::expert_a_bytes(H, Is, bits) : 0;
    rc = slx::launch_switchglu_fused(a, d, gbar, bits, s, svc, ep);
    if (rc != SLX_ERR_UNSUPPORTED) {
      g_glu_kernels = rc ? 0 : 1;
      return rc ? cuda_check(rc, "slx_switchglu fused") : SLX_OK;
    }
  }
  if (svc || ep)
    return fail(SLX_ERR_UNSUPPORTED, "switchglu (serviced / ep): the token's "
                "tiles do not fit the single-launch form");
  g_glu_kernels = 0;
  rc = slx::launch_gemv(a, bits, s, /*pdl_secondary=*/true);
  if (rc) return cuda_check(rc, "slx_switchglu gate/up");
  rc = slx::launch_down(d, bits, s);
  if (!rc) g_glu_kernels = 2;
  return rc ? cuda_check(rc, "slx_switchglu down") : SLX_OK;
}

int slx_switchglu_last_kernels(void) { return g_glu_kernels; }

int slx_host_device_ptr(const void* host, void** dev) {
  g_err.clear();
  if (!host || !dev) return fail(SLX_ERR_INVALID, "host_device_ptr: NULL");
  const cudaError_t e =
      cudaHostGetDevicePointer(dev, const_cast<void*>(host), 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SLX_ERR_CUDA, "cudaHostGetDevicePointer: %s",
                cudaGetErrorString(e));
  }
  return SLX_OK;
}

size_t slx_prefill_scratch_bytes(int n_blocks, int hidden, int inter,
                                 int bits) {
  if (n_blocks < 0 || bits != 2 || hidden <= 0 || inter <= 0 ||
      hidden % 512 || inter % 512)
    return 0;
  return slx::prefill_scratch_bytes(n_blocks, hidden, inter);
}

int slx_prefill_grouped(const slx_expert_bank* bank, const void* x,
                        int n_rows, const int32_t* pair_row, int n_pairs,
                        const int32_t* blocks, int n_blocks,
                        const int32_t* out_row, void* out, int n_out,
                        void* scratch, size_t scratch_bytes, int32_t* status,
                        void* stream) {
  g_err.clear();
  if (!bank) return fail(SLX_ERR_INVALID, "slx_prefill_grouped: bank is NULL");
  const int H = bank->hidden, I = bank->inter;
  if (bank->bits != 2)
    return fail(SLX_ERR_UNSUPPORTED, "prefill: bits %d (2-bit experts only)",
                bank->bits);
  if (H <= 0 || I <= 0 || H % 512 || I % 512 || H > 4096 || I > 4096)
    return fail(SLX_ERR_UNSUPPORTED,
                "prefill: hidden %d / inter %d must be multiples of 512, <= 4096",
                H, I);
  if (bank->n_slots < 1 || bank->slot_stride % 16 ||
      bank->slot_stride < (int64_t)slx::expert_tiled_bytes(H, I, 2))
    return fail(SLX_ERR_INVALID, "prefill: n_slots %d slot_stride %lld",
                bank->n_slots, (long long)bank->slot_stride);
  if (n_blocks < 0 || n_pairs < 0 || n_rows < 0 || n_out < 0)
    return fail(SLX_ERR_INVALID, "prefill: negative count");
  if (n_blocks == 0) return SLX_OK;
  if (!bank->base || !aligned16(bank->base) || !x || !aligned16(x) ||
      !pair_row || !blocks || !aligned16(blocks) || !out || !aligned16(out))
    return fail(SLX_ERR_INVALID, "prefill: NULL or misaligned pointer");
  const size_t need = slx::prefill_scratch_bytes(n_blocks, H, I);
  if (!scratch || scratch_bytes < need || (reinterpret_cast<uintptr_t>(scratch) & 127))
    return fail(SLX_ERR_SCRATCH, "prefill: scratch %zu < %zu bytes (128-aligned)",
                scratch_bytes, need);
  const int rc = slx::launch_prefill(
      reinterpret_cast<const uint8_t*>(bank->base), bank->slot_stride,
      bank->n_slots, H, I, reinterpret_cast<const uint16_t*>(x), n_rows,
      pair_row, n_pairs, reinterpret_cast<const int4*>(blocks), n_blocks,
      out_row, reinterpret_cast<uint16_t*>(out), n_out,
      reinterpret_cast<uint8_t*>(scratch), status,
      reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_prefill_grouped") : SLX_OK;
}

int slx_set_switchglu_fused(int on) {
  const int prev = g_fused;
  g_fused = on ? 1 : 0;
  return prev;
}

int slx_qlinear(const void* w_tiled, int out_features, int in_features,
                int bits, const void* x, int T, void* y, int32_t* status,
                void* stream) {
  g_err.clear();
  if (!w_tiled || !aligned16(w_tiled))
    return fail(SLX_ERR_INVALID, "qlinear: weight NULL or misaligned");
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(SLX_ERR_UNSUPPORTED, "bits %d", bits);
  if (in_features <= 0 || in_features % 64 || out_features <= 0 ||
      out_features % 16)
    return fail(SLX_ERR_INVALID, "qlinear shape out %d in %d", out_features,
                in_features);
  if (T < 0) return fail(SLX_ERR_INVALID, "T %d", T);
  if (T == 0) return SLX_OK;
  if (!x || !y || !aligned16(x)) return fail(SLX_ERR_INVALID, "x/y");
  slx::GemvArgs a = {};
  a.mode = SLX_GEMV_LINEAR;
  a.x = reinterpret_cast<const uint16_t*>(x);
  a.T = T;
  a.in = in_features;
  a.lin = reinterpret_cast<const uint8_t*>(w_tiled);
  a.out_features = out_features;
  a.y = reinterpret_cast<uint16_t*>(y);
  a.status = status;
  a.n_tiles = T * ((out_features + 31) / 32);
  const int rc = slx::launch_gemv(a, bits, reinterpret_cast<cudaStream_t>(stream),
                                  /*pdl_secondary=*/false);
  return rc ? cuda_check(rc, "slx_qlinear") : SLX_OK;
}

int slx_dequant_rows(const slx_qmat* w, int in_features, int bits,
                     int group_size, const int32_t* rows, int nrows,
                     int n_src_rows, void* out, int out_bf16, int32_t* status,
                     void* stream) {
  g_err.clear();
  if (!w || !w->weight || !w->scales || !w->biases || !out)
    return fail(SLX_ERR_INVALID, "dequant: NULL pointer");
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(SLX_ERR_UNSUPPORTED, "bits %d", bits);
  if (group_size <= 0 || in_features % group_size || (in_features * bits) % 32)
    return fail(SLX_ERR_INVALID, "dequant shape in %d gs %d", in_features,
                group_size);
  if (nrows < 0 || n_src_rows < 0) return fail(SLX_ERR_INVALID, "rows");
  const int rc = slx::launch_dequant_rows(
      (const uint32_t*)w->weight, (const uint16_t*)w->scales,
      (const uint16_t*)w->biases, in_features, bits, group_size, rows, nrows,
      n_src_rows, out, out_bf16, status, reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_dequant_rows") : SLX_OK;
}

// Router scratch: [T, E] logits, then (one token) the E logit bounds of
// the many-SM form, then the T tickets.
static size_t router_bound_bytes(int T, int n_experts) {
  return T == 1 ? align256((size_t)n_experts * 4) : 0;
}

size_t slx_router_scratch_bytes(int T, int n_experts) {
  if (T < 0 || n_experts < 0) return 0;
  return align256((size_t)T * n_experts * 4) + router_bound_bytes(T, n_experts) +
         align256((size_t)T * 4);
}

int slx_router_topk(const void* x, const void* ratio, const void* w_gate,
                    const float* bias, int T, int H, int E, int k,
                    int norm_topk, const int32_t* force,
                    const int32_t* forced_ids, int32_t* out_ids,
                    float* out_scores, void* scratch, size_t scratch_bytes,
                    int32_t* status, void* stream) {
  g_err.clear();
  if (!x || !w_gate || !out_ids || !out_scores)
    return fail(SLX_ERR_INVALID, "router: NULL pointer");
  if (!aligned16(x) || !aligned16(w_gate) || (ratio && !aligned16(ratio)))
    return fail(SLX_ERR_INVALID, "router: x / w_gate / ratio not 16-byte aligned");
  if (T < 0 || H <= 0 || H % 8 || E < 1 || k < 1 || k > E)
    return fail(SLX_ERR_INVALID, "router shape T %d H %d E %d k %d", T, H, E, k);
  if (force && !forced_ids) return fail(SLX_ERR_INVALID, "force without ids");
  if (T == 0) return SLX_OK;
  const size_t need = slx_router_scratch_bytes(T, E);
  if (!scratch || scratch_bytes < need)
    return fail(SLX_ERR_SCRATCH, "router scratch %zu < %zu", scratch_bytes, need);
  slx::RouterArgs a = {};
  a.x = (const uint16_t*)x;
  a.ratio = (const uint16_t*)ratio;
  a.w = (const uint16_t*)w_gate;
  a.bias = bias;
  a.T = T;
  a.H = H;
  a.E = E;
  a.k = k;
  a.norm_topk = norm_topk;
  a.force = force;
  a.forced_ids = forced_ids;
  a.out_ids = out_ids;
  a.out_scores = out_scores;
  a.logits = reinterpret_cast<float*>(scratch);
  a.bound = T == 1 ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) +
                                               align256((size_t)T * E * 4))
                   : nullptr;
  a.tickets = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(scratch) +
                                         align256((size_t)T * E * 4) +
                                         router_bound_bytes(T, E));
  a.status = status;
  const int rc = slx::launch_router(a, reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_router_topk") : SLX_OK;
}

static int router_multi_impl(const slx_router_head* heads, int n_heads,
                             const void* x, int T, int H, int E, int k,
                             int norm_topk, int32_t* status, void* stream,
                             const slx::RouterNorm* norm);

int slx_router_topk_multi(const slx_router_head* heads, int n_heads,
                          const void* x, int T, int H, int E, int k,
                          int norm_topk, int32_t* status, void* stream) {
  g_err.clear();
  return router_multi_impl(heads, n_heads, x, T, H, E, k, norm_topk, status,
                           stream, nullptr);
}

int slx_router_topk_multi_norm(const slx_router_head* heads, int n_heads,
                               const void* h_in, const void* delta,
                               const void* norm_weight, float eps,
                               void* h_out, void* x_out, int H, int E, int k,
                               int norm_topk, int32_t* status, void* stream) {
  g_err.clear();
  if (!h_in || !norm_weight || !h_out || !x_out)
    return fail(SLX_ERR_INVALID, "router_multi_norm: NULL pointer");
  if (!aligned16(h_in) || !aligned16(norm_weight) || !aligned16(h_out) ||
      !aligned16(x_out) || (delta && !aligned16(delta)))
    return fail(SLX_ERR_INVALID, "router_multi_norm: operands not 16-byte aligned");
  if (h_out == h_in)
    return fail(SLX_ERR_INVALID, "router_multi_norm: h_out may not alias h_in");
  const slx::RouterNorm nm = {(const uint16_t*)h_in, (const uint16_t*)delta,
                              (const uint16_t*)norm_weight, eps,
                              (uint16_t*)h_out, (uint16_t*)x_out};
  return router_multi_impl(heads, n_heads, x_out, 1, H, E, k, norm_topk,
                           status, stream, &nm);
}

static int router_multi_impl(const slx_router_head* heads, int n_heads,
                             const void* x, int T, int H, int E, int k,
                             int norm_topk, int32_t* status, void* stream,
                             const slx::RouterNorm* norm) {
  if (!heads || n_heads < 1 || n_heads > 2)
    return fail(SLX_ERR_INVALID, "router_multi: 1 or 2 heads");
  if (!x || !aligned16(x))
    return fail(SLX_ERR_INVALID, "router_multi: x NULL or not 16-byte aligned");
  if (T < 0 || H <= 0 || H % 8 || E < 1 || k < 1 || k > E)
    return fail(SLX_ERR_INVALID, "router shape T %d H %d E %d k %d", T, H, E, k);
  if (T == 0) return SLX_OK;
  const size_t need = slx_router_scratch_bytes(T, E);
  slx::RouterArgs a[2] = {};
  for (int i = 0; i < n_heads; ++i) {
    const slx_router_head& h = heads[i];
    if (!h.w_gate || !h.out_ids || !h.out_scores)
      return fail(SLX_ERR_INVALID, "router_multi head %d: NULL pointer", i);
    if (!aligned16(h.w_gate) || (h.ratio && !aligned16(h.ratio)))
      return fail(SLX_ERR_INVALID, "router_multi head %d: not 16-byte aligned", i);
    if (h.force && !h.forced_ids)
      return fail(SLX_ERR_INVALID, "router_multi head %d: force without ids", i);
    if (!h.scratch || h.scratch_bytes < need)
      return fail(SLX_ERR_SCRATCH, "router_multi head %d: scratch %zu < %zu",
                  i, h.scratch_bytes, need);
    for (int j = 0; j < i; ++j)
      if (heads[j].scratch == h.scratch)
        return fail(SLX_ERR_INVALID, "router_multi: heads share scratch");
    a[i].x = (const uint16_t*)x;
    a[i].ratio = (const uint16_t*)h.ratio;
    a[i].w = (const uint16_t*)h.w_gate;
    a[i].bias = h.bias;
    a[i].T = T;
    a[i].H = H;
    a[i].E = E;
    a[i].k = k;
    a[i].norm_topk = norm_topk;
    a[i].force = h.force;
    a[i].forced_ids = h.forced_ids;
    a[i].out_ids = h.out_ids;
    a[i].out_scores = h.out_scores;
    a[i].logits = reinterpret_cast<float*>(h.scratch);
    a[i].bound = T == 1 ? reinterpret_cast<float*>(
                              reinterpret_cast<uint8_t*>(h.scratch) +
                              align256((size_t)T * E * 4))
                        : nullptr;
    a[i].tickets = reinterpret_cast<int32_t*>(
        reinterpret_cast<uint8_t*>(h.scratch) + align256((size_t)T * E * 4) +
        router_bound_bytes(T, E));
    a[i].status = status;
  }
  const int rc = slx::launch_router_heads(
      a, n_heads, reinterpret_cast<cudaStream_t>(stream), norm);
  if (rc == SLX_ERR_UNSUPPORTED && norm)
    return fail(rc, "router_multi_norm: one token, H <= 8192, H %% 32 == 0");
  return rc ? cuda_check(rc, "slx_router_topk_multi") : SLX_OK;
}

int slx_add_rmsnorm_out(const void* h_in, const void* delta,
                        const void* weight, int T, int H, float eps,
                        void* h_out, void* y, void* stream) {
  g_err.clear();
  if (!h_in || !weight || !y || !h_out) return fail(SLX_ERR_INVALID, "rmsnorm: NULL");
  if (!aligned16(h_in) || !aligned16(h_out) || !aligned16(weight) ||
      !aligned16(y) || (delta && !aligned16(delta)))
    return fail(SLX_ERR_INVALID, "rmsnorm: operands must be 16-byte aligned");
  const int rc = slx::launch_add_rmsnorm(
      (const uint16_t*)h_in, (const uint16_t*)delta, (const uint16_t*)weight,
      T, H, eps, (uint16_t*)h_out, (uint16_t*)y,
      reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_add_rmsnorm") : SLX_OK;
}

int slx_add_rmsnorm(void* h, const void* delta, const void* weight, int T,
                    int H, float eps, void* y, void* stream) {
  return slx_add_rmsnorm_out(h, delta, weight, T, H, eps, h, y, stream);
}

int slx_event_record_external(void* event, void* stream) {
  g_err.clear();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &cs);
  if (e != cudaSuccess)
    return fail(SLX_ERR_CUDA, "event record: %s", cudaGetErrorString(e));
  // outside a capture the flag is not accepted; a plain record is the same
  e = cs == cudaStreamCaptureStatusActive
          ? cudaEventRecordWithFlags(reinterpret_cast<cudaEvent_t>(event), s,
                                     cudaEventRecordExternal)
          : cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), s);
  return e == cudaSuccess ? SLX_OK
                          : fail(SLX_ERR_CUDA, "event record: %s",
                                 cudaGetErrorString(e));
}

int slx_event_elapsed_many(void* const* start, void* const* end, int n,
                           float* out_ms) {
  g_err.clear();
  for (int i = 0; i < n; ++i) {
    const cudaError_t e =
        cudaEventElapsedTime(&out_ms[i], reinterpret_cast<cudaEvent_t>(start[i]),
                             reinterpret_cast<cudaEvent_t>(end[i]));
    if (e != cudaSuccess)
      return fail(SLX_ERR_CUDA, "elapsed[%d]: %s", i, cudaGetErrorString(e));
  }
  return SLX_OK;
}

int slx_qk_norm_rope_cache(void* qkv, int T, int n_q, int n_kv, int head_dim,
                           const void* q_norm, const void* k_norm, float eps,
                           const float* inv_freq, const int32_t* pos,
                           int max_len, void* k_cache, void* v_cache,
                           int32_t* status, void* stream) {
  g_err.clear();
  if (!qkv || !q_norm || !k_norm || !inv_freq || !pos || !k_cache || !v_cache)
    return fail(SLX_ERR_INVALID, "rope: NULL");
  if (n_q < 1 || n_kv < 1 || n_q % n_kv) return fail(SLX_ERR_INVALID, "heads");
  const int rc = slx::launch_qk_rope_cache(
      (uint16_t*)qkv, T, n_q, n_kv, head_dim, (const uint16_t*)q_norm,
      (const uint16_t*)k_norm, eps, inv_freq, pos, max_len,
      (uint16_t*)k_cache, (uint16_t*)v_cache, status,
      reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_qk_norm_rope_cache") : SLX_OK;
}

int slx_attn_decode(const void* qkv, int T, int n_q, int n_kv, int head_dim,
                    const void* k_cache, const void* v_cache,
                    const int32_t* pos, int max_len, void* out, void* stream) {
  g_err.clear();
  if (!qkv || !k_cache || !v_cache || !pos || !out)
    return fail(SLX_ERR_INVALID, "attn: NULL");
  if (n_q < 1 || n_kv < 1 || n_q % n_kv) return fail(SLX_ERR_INVALID, "heads");
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(SLX_ERR_INVALID, "attn: caches not 16-byte aligned");
  const int rc = slx::launch_attn_decode(
      (const uint16_t*)qkv, T, n_q, n_kv, head_dim, (const uint16_t*)k_cache,
      (const uint16_t*)v_cache, pos, max_len, (uint16_t*)out,
      reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_attn_decode") : SLX_OK;
}

int slx_attn_rope_decode(const void* qkv, int n_q, int n_kv, int head_dim,
                         const void* q_norm, const void* k_norm, float eps,
                         const float* inv_freq, const int32_t* pos,
                         int max_len, void* k_cache, void* v_cache, void* out,
                         int32_t* status, void* stream) {
  g_err.clear();
  if (!qkv || !q_norm || !k_norm || !inv_freq || !pos || !k_cache ||
      !v_cache || !out)
    return fail(SLX_ERR_INVALID, "attn_rope: NULL");
  if (n_q < 1 || n_kv < 1 || n_q % n_kv) return fail(SLX_ERR_INVALID, "heads");
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(qkv))
    return fail(SLX_ERR_INVALID, "attn_rope: qkv / caches not 16-byte aligned");
  const int rc = slx::launch_attn_rope_decode(
      (const uint16_t*)qkv, n_q, n_kv, head_dim, (const uint16_t*)q_norm,
      (const uint16_t*)k_norm, eps, inv_freq, pos, max_len,
      (uint16_t*)k_cache, (uint16_t*)v_cache, (uint16_t*)out, status,
      reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_attn_rope_decode") : SLX_OK;
}

int slx_argmax(const void* logits, int T, int V, int32_t* out, void* stream) {
  g_err.clear();
  if (!logits || !out || V < 1) return fail(SLX_ERR_INVALID, "argmax");
  const int rc = slx::launch_argmax((const uint16_t*)logits, T, V, out,
                                    reinterpret_cast<cudaStream_t>(stream));
  return rc ? cuda_check(rc, "slx_argmax") : SLX_OK;
}

int slx_copy_many(void* const* dst, const void* const* src,
                  const size_t* bytes, int n, void* stream) {
  g_err.clear();
  if (n < 0 || (n > 0 && (!dst || !src || !bytes)))
    return fail(SLX_ERR_INVALID, "copy_many: bad arrays");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    if (!bytes[i]) continue;
    const cudaError_t e =
        cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyDefault, s);
    if (e != cudaSuccess)
      return fail(SLX_ERR_CUDA, "copy_many[%d]: %s", i, cudaGetErrorString(e));
  }
  return SLX_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Router without caller scratch.  The logits and the per-token tickets live
// in this file's own static device array; the tickets start at zero (module
// load) and every router launch leaves them zero.
namespace {

constexpr int kNoAllocLogits = 32768;   // max T * n_experts
constexpr int kNoAllocTokens = 1024;    // max T
constexpr size_t kNoAllocTicketOff = (size_t)kNoAllocLogits * 4;
constexpr size_t kNoAllocBytes = kNoAllocTicketOff + (size_t)kNoAllocTokens * 4;
constexpr int kNoAllocDevices = 64;

static __device__ __align__(256) unsigned char g_router_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocDevices] = {};

}  // namespace

extern "C" int slx_router_topk_noalloc(
    const void* x, const void* ratio, const void* w_gate, const float* bias,
    int T, int H, int E, int k, int norm_topk, const int32_t* force,
    const int32_t* forced_ids, int32_t* out_ids, float* out_scores,
    int32_t* status, void* stream) {
  g_err.clear();
  if (T < 0 || E < 1) return fail(SLX_ERR_INVALID, "router_noalloc: T %d E %d", T, E);
  if (T > kNoAllocTokens || (long long)T * E > kNoAllocLogits)
    return fail(SLX_ERR_SCRATCH,
                "router_noalloc: T %d x E %d exceeds the static scratch "
                "(%d logits, %d tokens); use slx_router_topk with caller "
                "scratch", T, E, kNoAllocLogits, kNoAllocTokens);
  int dev = -1;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess)
    return fail(SLX_ERR_CUDA, "router_noalloc: %s", cudaGetErrorString(ce));
  if (dev < 0 || dev >= kNoAllocDevices)
    return fail(SLX_ERR_UNSUPPORTED, "router_noalloc: device %d", dev);
  void* base;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      ce = cudaGetSymbolAddress(&p, g_router_scratch);
      if (ce != cudaSuccess || !p)
        return fail(SLX_ERR_CUDA, "router_noalloc: symbol address: %s",
                    cudaGetErrorString(ce));
      g_noalloc_addr[dev] = p;
    }
    base = g_noalloc_addr[dev];
  }
  // slx_router_topk puts the tickets right after the 256-aligned logits
  // (and, for one token, the logit bounds); start the logits so that the
  // tickets land on the fixed ticket words.
  const size_t logit_bytes =
      align256((size_t)T * E * 4) + router_bound_bytes(T, E);
  if (logit_bytes > kNoAllocTicketOff)
    return fail(SLX_ERR_SCRATCH, "router_noalloc: E %d too large", E);
  unsigned char* scr = (unsigned char*)base + kNoAllocTicketOff - logit_bytes;
  return slx_router_topk(x, ratio, w_gate, bias, T, H, E, k, norm_topk, force,
                         forced_ids, out_ids, out_scores, scr,
                         slx_router_scratch_bytes(T, E), status, stream);
}
