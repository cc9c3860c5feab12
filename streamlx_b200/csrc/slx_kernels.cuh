// Argument blocks and host launchers shared by the kernel translation units
// and the C ABI (slx_api.cu).
#pragma once
#include "slx_common.cuh"

namespace slx {

struct GemvArgs {
  int mode;  // SLX_GEMV_GLU or SLX_GEMV_LINEAR
  const uint16_t* x;
  int T;
  int in;
  // GLU: routed experts (tile-format slot pool)
  const int32_t* ids;
  int k;
  const int32_t* slot_table;  // [n_table] expert -> slot, or null (ids are slots)
  int n_table;
  int n_slots;
  const uint8_t* bank;
  long long slot_stride;
  int I;
  // GLU: shared expert (tile format, same hidden/bits)
  const uint8_t* shared;
  int Is;
  // SwiGLU output, written directly as the down projection's activation
  // fragments (+ per-16-column partial sums), see slx_qgemv.cu
  uint32_t* hfrag;
  float* hpart;
  uint32_t* hfrag_sh;
  float* hpart_sh;
  int unit_frag_words, unit_part_floats;      // per routed unit
  int shared_frag_words, shared_part_floats;  // per token (shared expert)
  // LINEAR: dense tile-format matrix
  const uint8_t* lin;
  int out_features;
  uint16_t* y;  // [T, out_features]
  int32_t* status;
  int n_tiles;
  int n_stages;
  int stage_bytes;
  int tile_bytes;
  int wait_primary;  // 1: kernel was launched as a PDL secondary
};

struct DownArgs {
  int T, k, H, I, Is;
  const int32_t* ids;
  const int32_t* slot_table;
  int n_table, n_slots;
  const float* scores;  // [T,k]; null -> per-expert output [T,k,H]
  const uint8_t* bank;
  long long slot_stride;
  long long a_bytes;     // bytes of an expert's gate/up region
  const uint8_t* shared;
  long long a_bytes_sh;
  const uint32_t* hfrag;
  const float* hpart;
  const uint32_t* hfrag_sh;
  const float* hpart_sh;
  int unit_frag_words, unit_part_floats, shared_frag_words, shared_part_floats;
  uint16_t* out;
  int32_t* status;
  int n_items, n_units, n_stages, stage_bytes, tile_bytes, tile_bytes_sh;
  int pdl;  // launched as PDL secondary of phase A
};

struct RouterArgs {
  const uint16_t* x;      // [T, H] bf16
  const uint16_t* ratio;  // [H] bf16 or null: x' = bf16(x * ratio)
  const uint16_t* w;      // [E, H] bf16
  const float* bias;      // [E] or null
  int T, H, E, k, norm_topk;
  const int32_t* force;      // [T] flags or null
  const int32_t* forced_ids; // [T, k]
  int32_t* out_ids;          // [T, k]
  float* out_scores;         // [T, k]
  float* logits;             // scratch [T, E]
  float* bound;              // scratch [E] when T == 1 (else null)
  int32_t* tickets;          // scratch [T], zero on entry, zero on exit
  int32_t* status;
};


int launch_gemv(GemvArgs a, int bits, cudaStream_t stream, bool pdl_secondary);
int launch_down(DownArgs a, int bits, cudaStream_t stream);
int launch_switchglu_fused(const GemvArgs& a, const DownArgs& d, void* bar,
                           int bits, cudaStream_t stream,
                           const slx_fill_service* svc = nullptr,
                           const slx_ep_exchange* ep = nullptr);
int launch_ep_combine_rmsnorm(const slx_ep_exchange& ep, const float* scores,
                              int k, int H, int has_shared,
                              const uint16_t* h_in, const uint16_t* w,
                              float eps, uint16_t* h_out, uint16_t* y,
                              int32_t* status, cudaStream_t s);
int launch_dequant_rows(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                        int in, int bits, int gs, const int32_t* rows,
                        int nrows, int n_src_rows, void* out, int out_bf16,
                        int32_t* status, cudaStream_t stream);
int launch_router(const RouterArgs& a, cudaStream_t stream);
// The residual add + RMSNorm that produces a one-token router's input.
struct RouterNorm {
  const uint16_t* h_in;   // [H]
  const uint16_t* delta;  // [H] or null
  const uint16_t* w;      // [H] norm weight
  float eps;
  uint16_t* h_out;        // [H] h_in + delta (may not alias h_in)
  uint16_t* y;            // [H] the normalised x
};

int launch_router_heads(const RouterArgs* heads, int n_heads,
                        cudaStream_t stream, const RouterNorm* norm = nullptr);
int launch_pack_experts(const void* const* gw, const void* const* gs,
                        const void* const* gb, const void* const* uw,
                        const void* const* us, const void* const* ub,
                        const void* const* dw, const void* const* ds,
                        const void* const* db, void* const* dst, int n, int H,
                        int I, int bits, cudaStream_t stream);
int launch_pack_dense(const void* w, const void* s, const void* b, int out,
                      int in, int bits, void* dst, cudaStream_t stream);
int launch_add_rmsnorm(const uint16_t* h_in, const uint16_t* d,
                       const uint16_t* w, int T, int H, float eps,
                       uint16_t* h_out, uint16_t* y, cudaStream_t s);
int launch_qk_rope_cache(uint16_t* qkv, int T, int nq, int nkv, int hd,
                         const uint16_t* qn, const uint16_t* kn, float eps,
                         const float* inv_freq, const int32_t* pos,
                         int max_len, uint16_t* kc, uint16_t* vc,
                         int32_t* status, cudaStream_t s);
int launch_attn_decode(const uint16_t* qkv, int T, int nq, int nkv, int hd,
                       const uint16_t* kc, const uint16_t* vc,
                       const int32_t* pos, int max_len, uint16_t* out,
                       cudaStream_t s);
int launch_attn_rope_decode(const uint16_t* qkv, int nq, int nkv, int hd,
                            const uint16_t* qn, const uint16_t* kn, float eps,
                            const float* inv_freq, const int32_t* pos,
                            int max_len, uint16_t* kc, uint16_t* vc,
                            uint16_t* out, int32_t* status, cudaStream_t s);
int launch_argmax(const uint16_t* logits, int T, int V, int32_t* out,
                  cudaStream_t s);
size_t prefill_scratch_bytes(int n_blocks, int H, int I);
int launch_prefill(const uint8_t* bank, long long slot_stride, int n_slots,
                   int H, int I, const uint16_t* x, int n_rows,
                   const int32_t* pair_row, int n_pairs, const int4* blocks,
                   int n_blocks, const int32_t* out_row, uint16_t* out,
                   int n_out, uint8_t* scratch, int32_t* status,
                   cudaStream_t s);

}  // namespace slx
