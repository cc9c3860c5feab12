/*
 * streamlx_cuda.h -- C ABI of libstreamlx_cuda.so, the sm_100a (B200) kernels
 * behind the streamlx quantized mixture-of-experts expert path.
 *
 * Conventions
 *   - Every pointer argument named x / w / out / scratch / status ... is a
 *     DEVICE pointer unless the comment says "host".  bf16 data is passed as
 *     raw 16-bit words (uint16_t / void*), quantized weights as raw bytes.
 *   - Quantized weights use the MLX "affine" layout: a matrix [out, in] is
 *     `weight` uint32 [out, in*bits/32] (codes packed low bits first),
 *     `scales` and `biases` bf16 [out, in/group_size]; w = scale*q + bias.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Every call is asynchronous on `stream`, allocates nothing and does not
 *     synchronise.  The return value is 0 (SLX_OK) or a negative SLX_ERR_*;
 *     errors found on the device (unmapped expert, out-of-range index, a
 *     bounded wait that expired) are written to the int32 `status` word
 *     (first error wins) -- read it after the stream completes.
 *   - Thread-compatible: concurrent calls need distinct streams / scratch.
 *
 * Reference interfaces these replace are cited per entry point
 * (paths inside the streamlx project).
 */
#ifndef STREAMLX_CUDA_H_
#define STREAMLX_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SLX_OK 0
#define SLX_ERR_INVALID (-1)         /* bad argument (host-side check) */
#define SLX_ERR_UNSUPPORTED (-2)     /* shape / bit width not implemented */
#define SLX_ERR_CUDA (-3)            /* CUDA runtime error (see string) */
#define SLX_ERR_OUT_OF_RANGE (-4)    /* device: index outside its table */
#define SLX_ERR_UNMAPPED_EXPERT (-5) /* device: expert id has no pool slot */
#define SLX_ERR_DEVICE_TIMEOUT (-6)  /* device: a bounded wait expired */
#define SLX_ERR_SCRATCH (-7)         /* scratch buffer too small */
#define SLX_ERR_IO (-8)              /* host file read failed or was short */
#define SLX_ERR_RANGE (-9)           /* device: an operand outside the range
                                        a kernel computes exactly (fp16
                                        operands: see the kernel's entry) */

#define SLX_GEMV_GLU 0
#define SLX_GEMV_LINEAR 1

/* One quantized matrix in the MLX affine layout. */
typedef struct slx_qmat {
  const void* weight; /* uint32 codes */
  const void* scales; /* bf16 */
  const void* biases; /* bf16 */
} slx_qmat;

/* HBM slot pool of one MoE layer, every slot one expert in the TILE format
 * produced by slx_pack_experts (16-row tiles streamed by the kernels in one
 * piece; see streamlx_b200/csrc/slx_tiles.cuh).  Replaces the per-part slot
 * tensors of streamlx/pool.py:71-77 (StreamingSwitchMLP.pool[proj][part]). */
typedef struct slx_expert_bank {
  const void* base;    /* n_slots x slot_stride bytes */
  int64_t slot_stride; /* >= slx_expert_tiled_bytes(...), multiple of 16 */
  int32_t n_slots;
  int32_t hidden;
  int32_t inter;
  int32_t bits; /* 2, 4 or 8; group size is 64 */
} slx_expert_bank;

/* Always-on shared expert (weight 1.0 in the combine), tile format, same
 * hidden size and bit width as the routed experts. */
typedef struct slx_shared_expert {
  const void* base;
  int32_t inter;
} slx_shared_expert;

int slx_version(void);

/* Programmatic dependent launch for the calling host thread's subsequent
 * launches (0 = off, the default).  With it on, each kernel may start while
 * the previous one on the stream drains: it streams its fixed weights early
 * and waits (griddepcontrol.wait) before touching anything the previous
 * kernel wrote, so results are the same either way.  Returns the previous
 * setting. */
int slx_set_pdl(int on);

/* Last host-side error message of the calling thread ("" if none). */
const char* slx_last_error_string(void);

/* Bytes of one expert (gate/up/down, group 64) in the tile format; equal to
 * its bytes in the MLX layout. */
size_t slx_expert_tiled_bytes(int hidden, int inter, int bits);

/* Bytes of a dense [out, in] quantized matrix in the tile format (rows
 * padded to a multiple of 32). */
size_t slx_dense_tiled_bytes(int out_features, int in_features, int bits);

/* Repack n experts from the MLX affine layout (the safetensors row ranges of
 * streamlx/stindex.py:31-39, already in device memory) into tile-format
 * slots dst[i] (device pointers, 16-byte aligned).  gate/up/down/dst are
 * HOST arrays of n entries.  The slot-fill step of the pool
 * (streamlx/pool.py:196-199, 295-297). */
int slx_pack_experts(const slx_qmat* gate, const slx_qmat* up,
                     const slx_qmat* down, int n, int hidden, int inter,
                     int bits, void* const* dst, void* stream);

/* Repack a dense [out, in] matrix (MLX layout, device) into the tile format
 * at dst (slx_dense_tiled_bytes bytes). */
int slx_pack_dense(const slx_qmat* w, int out_features, int in_features,
                   int bits, void* dst, void* stream);

/* Scratch bytes slx_switchglu needs for T tokens (activations h). */
size_t slx_switchglu_scratch_bytes(int T, int k, int inter, int shared_inter);

/* Fused quantized SwitchGLU for decode / small batches (K2).
 * Replaces streamlx/pool.py:30-50 switch_forward (three gather_qmm + swiglu)
 * together with the id->slot remap of streamlx/integrate.py:90-95 and the
 * score-weighted combine of the mlx-lm MoE block (streamlx/integrate.py:5-7).
 *   x        [T, hidden] bf16
 *   ids      [T, k] int32 expert ids (or slot ids when slot_table == NULL)
 *   slot_table [n_table] int32 expert -> slot (-1 = not resident) or NULL
 *   scores   [T, k] fp32 router weights, or NULL for the drop-in mode that
 *            returns per-expert UNWEIGHTED outputs out[T, k, hidden]
 *            (SwitchGLU.__call__ semantics); with scores, out is the combined
 *            [T, hidden] = sum_j scores*expert_j(x) (+ shared expert).
 *   shared   optional shared expert (ignored when scores == NULL)
 *   scratch  >= slx_switchglu_scratch_bytes(...) device bytes
 * An id without a slot sets SLX_ERR_UNMAPPED_EXPERT in *status and
 * contributes zeros. */
int slx_switchglu(const slx_expert_bank* bank, const slx_shared_expert* shared,
                  const void* x, int T, int k, const int32_t* ids,
                  const float* scores, const int32_t* slot_table, int n_table,
                  void* out, void* scratch, size_t scratch_bytes,
                  int32_t* status, void* stream);

/* In-kernel slot fill of a graph-launched decode step.  Replaces, for the
 * CUDA-graph decoder, the per-layer host round trip of
 * streamlx/integrate.py:234-250 (host sync on the routed ids, then
 * touch/ensure) and its hits-first overlap (streamlx/integrate.py:97-139):
 * a layer whose routed experts all have slots never waits on the host; a
 * layer with a miss parks in its own SwitchGLU launch until the host has run
 * the pool bookkeeping up to that layer, and then repacks the newly read
 * experts into their slots itself.
 *
 * Protocol (one decode token = one step, stamped by the host):
 *   1. On entry, CTA 0 writes this layer's record to `log` (host-mapped):
 *      word 1 = 1 when some routed id has no slot, word 2 = k, words
 *      4..4+k = routed ids, 20..20+k = predicted next-layer ids, 36..36+k =
 *      their fp32 scores (bit patterns); word 0 (written last) = the stamp.
 *   2. If an id has no slot, CTA 0 writes park[1] = layer, park[2] = stamp
 *      and then park[0] = ticket = (stamp << 8) | layer, and every CTA waits
 *      (bounded by wait_ns) until the device word `release` equals the
 *      ticket (-ticket aborts: the layer then reports
 *      SLX_ERR_UNMAPPED_EXPERT).
 *   3. The host writes the descriptor `desc` (slx_fill_header, then
 *      max_items slx_fill_item, then n_table int32 of the new expert -> slot
 *      table) and the raw MLX bytes of the experts it names into device
 *      memory with copies on a stream of its own, and then the ticket into
 *      `release` on that same stream.
 *   4. The kernel repacks each item into its slot, installs the new table
 *      into slot_table and continues with the layer.
 * The host must not touch `desc`, `release` or the slots of this layer's
 * pool while the layer runs, except through step 3. */
#define SLX_FILL_LOG_WORDS 64
#define SLX_FILL_MAX_K 16

typedef struct slx_fill_header {
  int32_t ticket;  /* must equal the parked kernel's ticket */
  int32_t layer;
  int32_t n_items; /* <= max_items */
  int32_t n_table; /* == n_table of the call */
  int32_t pad[4];
} slx_fill_header;

typedef struct slx_fill_item {
  int32_t slot;
  int32_t pad;
  /* device pointers (16-byte aligned) to the expert's MLX rows: gate
   * weight, scales, biases, up weight, scales, biases, down weight, scales,
   * biases */
  const void* part[9];
} slx_fill_item;

typedef struct slx_fill_service {
  int32_t layer;          /* 0..255 */
  int32_t max_items;      /* items the descriptor has room for */
  const int32_t* stamp;   /* device int32: the step's stamp, < 2^23 */
  int32_t* log;           /* host-mapped int32[SLX_FILL_LOG_WORDS] or NULL */
  const int32_t* pred_ids;  /* device [k] next-layer prediction, or NULL */
  const float* pred_scores; /* device [k] or NULL */
  int32_t* park;          /* host-mapped int32[4] */
  const int32_t* release; /* device int32 */
  const void* desc;       /* device descriptor (see above) */
  int32_t* go;            /* device int32 scratch word of this service */
  int64_t wait_ns;        /* bound of the park wait */
} slx_fill_service;

/* slx_switchglu for one decode token (T = 1, scores given: combined
 * output + shared expert) with the in-kernel slot fill described above.
 * slot_table is written by the kernel when it parks.  Needs the fused
 * single-launch form (SLX_ERR_UNSUPPORTED otherwise) and k <=
 * SLX_FILL_MAX_K. */
int slx_switchglu_serviced(const slx_expert_bank* bank,
                           const slx_shared_expert* shared, const void* x,
                           int k, const int32_t* ids, const float* scores,
                           int32_t* slot_table, int n_table, void* out,
                           void* scratch, size_t scratch_bytes,
                           int32_t* status, const slx_fill_service* svc,
                           void* stream);

/* Expert-parallel decode over NVLink peer memory (no reference counterpart:
 * the reference runs on one device).  Every rank runs the trunk and the
 * router (identical results on every rank) and the SwitchGLU of the routed
 * experts it owns (its slot table maps only those); the launch writes each
 * owned unit's bf16 output rows into EVERY rank's receive block of this
 * step and layer, then each of its CTAs adds 1 to every rank's counter of
 * the layer (system-scope release).  slx_ep_combine_rmsnorm on each rank
 * waits (bounded) until its counter of the stamp's parity reaches
 * ((stamp + 1) / 2) * n_ranks * grid (the steps of that parity so far), sums the
 * rows in unit order exactly as the single-GPU kernel does (so the result
 * does not depend on n_ranks), adds the residual and applies the next
 * RMSNorm.  Receive block layout per rank: [2 (stamp parity)][n_layers]
 * [k + 1][hidden] bf16 (row k = the shared expert, written by every rank
 * for itself); counters: uint32 [2][n_layers] (stamp parity), zero before
 * the first step.  A rank can only count itself for step s + 1 at a layer
 * after every rank has combined step s there, and parity-split counters keep
 * those early counts out of the step-s wait.
 * recv/count hold peer addresses (slx_ipc_open) except entry `rank`. */
#define SLX_EP_MAX_RANKS 8

typedef struct slx_ep_exchange {
  int32_t rank, n_ranks;   /* n_ranks <= SLX_EP_MAX_RANKS */
  int32_t layer, n_layers;
  const int32_t* stamp;    /* device int32: step stamp, 1, 2, 3, ... */
  void* recv[SLX_EP_MAX_RANKS];
  uint32_t* count[SLX_EP_MAX_RANKS];
  int32_t grid;            /* CTAs of the SwitchGLU launch (slx_ep_grid) */
  int64_t wait_ns;         /* bound of the combine's wait */
} slx_ep_exchange;

/* CTAs of the single-launch decode SwitchGLU on the current device (every
 * rank must agree). */
int slx_ep_grid(void);

/* slx_switchglu for one decode token in expert-parallel mode (above): the
 * combined output is formed by slx_ep_combine_rmsnorm, `scores` is still
 * required for the shared expert's presence only. */
int slx_switchglu_ep(const slx_expert_bank* bank,
                     const slx_shared_expert* shared, const void* x, int k,
                     const int32_t* ids, const float* scores,
                     const int32_t* slot_table, int n_table, void* scratch,
                     size_t scratch_bytes, int32_t* status,
                     const slx_ep_exchange* ep, void* stream);

/* Wait for every rank's rows of this step and layer, then
 * delta = bf16(sum_j scores[j] * row_j (+ shared row)), h_out = bf16(h_in +
 * delta), y = RMSNorm(h_out) * weight (one token).  With ep->grid == 0 the
 * wait is skipped (a warm-up launch). */
int slx_ep_combine_rmsnorm(const slx_ep_exchange* ep, const float* scores,
                           int k, int hidden, int has_shared,
                           const void* h_in, const void* weight, float eps,
                           void* h_out, void* y, int32_t* status,
                           void* stream);

/* CUDA IPC for the receive blocks: the handle (64 bytes) of the allocation
 * holding dev_ptr and dev_ptr's offset inside it; open maps a peer's
 * allocation (returns its base); close unmaps. */
int slx_ipc_handle(const void* dev_ptr, void* handle64, int64_t* offset);
int slx_ipc_open(const void* handle64, void** base);
int slx_ipc_close(void* base);

/* Device address of page-locked host memory (cudaHostGetDevicePointer):
 * the `log` and `park` words of slx_fill_service live in host memory that
 * the kernel writes.  Returns SLX_ERR_CUDA if `host` is not mapped. */
int slx_host_device_ptr(const void* host, void** dev);

/* Decode calls (T == 1) of slx_switchglu run both phases in one cooperative
 * launch when the token's tiles fit one CTA per SM; the first 256 bytes of
 * the scratch hold that launch's grid-barrier words and must be zero before
 * the first call (every call, of any shape, leaves them reusable).  on = 0 forces the
 * two-launch path for the calling host thread.  Returns the previous
 * setting. */
int slx_set_switchglu_fused(int on);

/* Kernels the calling thread's last successful slx_switchglu launched
 * (1 fused, 2 two-phase; launch accounting). */
int slx_switchglu_last_kernels(void);

/* Scratch bytes slx_prefill_grouped needs for n_blocks pair blocks (0 for
 * an unsupported shape): the fp16 operand images of both phases. */
size_t slx_prefill_scratch_bytes(int n_blocks, int hidden, int inter,
                                 int bits);

/* Expert-major prefill (K3) on the tcgen05 tensor cores.  Replaces the
 * per-batch switch_forward of streamlx/integrate.py:141-232 (_expert_sweep:
 * pairs grouped by expert, streamlx/pool.py:30-50 gather_qmm gate/up,
 * swiglu, gather_qmm down) for every pair whose expert has a slot.
 *   x        [n_rows, hidden] bf16 token rows
 *   pair_row [n_pairs] int32: x row of each (token, expert) pair, pairs
 *            grouped by expert
 *   blocks   [n_blocks][4] int32 {slot, first pair, pairs (1..128), 0}: runs
 *            of consecutive pairs of one expert (a longer run is split)
 *   out_row  [n_pairs] int32 output row of each pair, or NULL (= pair index)
 *   out      [n_out, hidden] bf16 per-pair UNWEIGHTED expert outputs
 * Rounding as switch_forward: gate/up -> bf16, silu(gate)*up -> bf16,
 * down -> bf16.  2-bit experts, hidden and inter multiples of 512 (<= 4096).
 * A block with a bad slot / range, or a pair row out of range, sets
 * SLX_ERR_OUT_OF_RANGE in *status and is skipped. */
int slx_prefill_grouped(const slx_expert_bank* bank, const void* x,
                        int n_rows, const int32_t* pair_row, int n_pairs,
                        const int32_t* blocks, int n_blocks,
                        const int32_t* out_row, void* out, int n_out,
                        void* scratch, size_t scratch_bytes, int32_t* status,
                        void* stream);

/* Dense quantized linear y[T, out] = x[T, in] @ dequant(W)^T (bf16 out,
 * fp32 accumulate) over a tile-format matrix (slx_pack_dense).  Trunk
 * projections of the decoder around the expert path (no reference
 * counterpart: mlx-lm's QuantizedLinear). */
int slx_qlinear(const void* w_tiled, int out_features, int in_features,
                int bits, const void* x, int T, void* y, int32_t* status,
                void* stream);

/* Bit-exact affine dequantisation of rows `rows[0..nrows)` (device int32
 * indices, or NULL for rows 0..nrows-1) of a quantized [n_src_rows, in]
 * matrix into fp32 (out_bf16 = 0) or bf16 (1) out[nrows, in].  The MLX
 * affine semantics of mx.gather_qmm's weight operand (streamlx/pool.py:43-45);
 * also the quantized embedding lookup. */
int slx_dequant_rows(const slx_qmat* w, int in_features, int bits,
                     int group_size, const int32_t* rows, int nrows,
                     int n_src_rows, void* out, int out_bf16, int32_t* status,
                     void* stream);

/* Scratch bytes slx_router_topk needs (logits + per-token tickets).  The
 * ticket part must be zero before the first call; every call leaves it zero. */
size_t slx_router_scratch_bytes(int T, int n_experts);

/* Router GEMV + softmax + top-k (K1).  Replaces the mlx-lm MoE router that
 * produces `indices` for streamlx/integrate.py:234 and the next-layer
 * predictor streamlx/integrate.py:60-88 (pass ratio = bf16(w_next/w_this)).
 *   x [T, H] bf16, ratio [H] bf16 or NULL, w_gate [E, H] bf16, bias [E] fp32
 *   or NULL.  logits = fp32(fp64 dot) + bias; ids = top-k by logit,
 *   descending, ties to the lower id; scores = softmax(logits)[ids]
 *   (renormalised to sum 1 when norm_topk).  force [T] (nullable) selects
 *   tokens whose ids are copied from forced_ids [T, k] instead (the
 *   temporal-reuse routing override); their scores still come from this
 *   token's softmax.  out_ids may alias forced_ids. */
int slx_router_topk(const void* x, const void* ratio, const void* w_gate,
                    const float* bias, int T, int H, int E, int k,
                    int norm_topk, const int32_t* force,
                    const int32_t* forced_ids, int32_t* out_ids,
                    float* out_scores, void* scratch, size_t scratch_bytes,
                    int32_t* status, void* stream);

/* One router "head": a gate [E, H] bf16 (+ bias [E] fp32, nullable), an
 * optional ratio [H] bf16 applied to x first (next-layer predictor), the
 * optional forced-ids override, outputs, and this head's own scratch of
 * slx_router_scratch_bytes(T, E) bytes. */
typedef struct slx_router_head {
  const void* w_gate;
  const float* bias;
  const void* ratio;
  const int32_t* force;
  const int32_t* forced_ids;
  int32_t* out_ids;
  float* out_scores;
  void* scratch;
  size_t scratch_bytes;
} slx_router_head;

/* slx_router_topk for 1 or 2 heads over the same x [T, H] in one launch:
 * the decode layer's router and its next-layer predictor
 * (streamlx/integrate.py:60-88 runs the predictor's gate on the same
 * MoE input).  Each head's results equal a slx_router_topk call. */
int slx_router_topk_multi(const slx_router_head* heads, int n_heads,
                          const void* x, int T, int H, int E, int k,
                          int norm_topk, int32_t* status, void* stream);

/* One decode token: the residual add + RMSNorm that produces the router's
 * input (h_out = h_in + delta, x_out = RMSNorm(h_out) * norm_weight, as
 * slx_add_rmsnorm_out computes them, bit for bit) and the 1-2 router heads
 * on x_out, in one launch.  h_out may not alias h_in.  The router's input
 * norm is mlx-lm's (the reference's MoE block sits after it). */
int slx_router_topk_multi_norm(const slx_router_head* heads, int n_heads,
                               const void* h_in, const void* delta,
                               const void* norm_weight, float eps,
                               void* h_out, void* x_out, int H, int E, int k,
                               int norm_topk, int32_t* status, void* stream);

/* Router GEMV + softmax + top-k exactly as slx_router_topk, for callers
 * that hold no device allocator: a host binding that reaches the library
 * only through this C ABI (ctypes, cgo, JNI) and would otherwise have to
 * call cudaMalloc itself and track the buffer per device, or a serving loop
 * that must not allocate device memory once it is warm.  No counterpart in
 * the reference.  Scratch is a static device array inside the library:
 * T <= 1024 and T * E <= 32768 (e.g. 128 tokens at 256 experts); larger
 * calls return SLX_ERR_SCRATCH.  Nothing needs zeroing by the caller.  All
 * calls on one device share that array, so calls that overlap (two streams,
 * or two host threads) race: order them on one stream.  The first call on
 * each device looks up the array's address (loading the module) and should
 * come before any stream capture.  The address is kept for the life of the
 * process: do not use this entry point across a cudaDeviceReset. */
int slx_router_topk_noalloc(const void* x, const void* ratio,
                            const void* w_gate, const float* bias, int T,
                            int H, int E, int k, int norm_topk,
                            const int32_t* force, const int32_t* forced_ids,
                            int32_t* out_ids, float* out_scores,
                            int32_t* status, void* stream);

/* Trunk helpers (no reference counterpart; mlx-lm's model code). */
int slx_add_rmsnorm(void* h, const void* delta, const void* weight, int T,
                    int H, float eps, void* y, void* stream);
/* h_out = h_in + delta (delta nullable), y = RMSNorm(h_out) * weight; all
 * operands 16-byte aligned, H % 8 == 0, H <= 8192; h_out may alias h_in. */
int slx_add_rmsnorm_out(const void* h_in, const void* delta,
                        const void* weight, int T, int H, float eps,
                        void* h_out, void* y, void* stream);
int slx_qk_norm_rope_cache(void* qkv, int T, int n_q, int n_kv, int head_dim,
                           const void* q_norm, const void* k_norm, float eps,
                           const float* inv_freq, const int32_t* pos,
                           int max_len, void* k_cache, void* v_cache,
                           int32_t* status, void* stream);
/* Batch-1 decode attention (GQA, head_dim 128, n_q / n_kv <= 8) over
 * positions 0..pos[t] of the caches; one 8-CTA cluster per (token, kv
 * head) splits the positions and merges in distributed shared memory. */
int slx_attn_decode(const void* qkv, int T, int n_q, int n_kv, int head_dim,
                    const void* k_cache, const void* v_cache,
                    const int32_t* pos, int max_len, void* out, void* stream);
/* One decode token (T = 1): slx_qk_norm_rope_cache and slx_attn_decode in
 * one launch.  Each cluster normalises and rotates its q heads and its kv
 * head's key, appends key and value at position pos[0] of the caches and
 * attends over positions 0..pos[0] (the new row taken from shared memory);
 * results equal the two-launch form bit for bit.  The trunk of the
 * synthetic decoders (mlx-lm's model code in the reference).
 * Under programmatic dependent launch (slx_set_pdl) pos[0] and the cache
 * rows before it are read before the kernel waits on the preceding one:
 * they must be complete before that kernel's chain started (written in an
 * earlier step, with a stream synchronisation, a graph boundary or a
 * launch without programmatic serialisation in between). */
int slx_attn_rope_decode(const void* qkv, int n_q, int n_kv, int head_dim,
                         const void* q_norm, const void* k_norm, float eps,
                         const float* inv_freq, const int32_t* pos,
                         int max_len, void* k_cache, void* v_cache, void* out,
                         int32_t* status, void* stream);
int slx_argmax(const void* logits, int T, int V, int32_t* out, void* stream);

/* Read n byte ranges of files: fds[i] from offsets[i], sizes[i] bytes,
 * into dsts[i], on up to `threads` native threads (a pool shared by all
 * callers; the caller works too).  Replaces the per-span os.pread tasks of
 * streamlx/reader.py:80-100.  Returns SLX_ERR_IO with *failed_index and
 * *failed_errno (0 = end of file before the range ended) on the first
 * failure.  Host code only: usable without a GPU. */
int slx_pread_many(const int* fds, const int64_t* offsets,
                   const int64_t* sizes, void* const* dsts, int n, int threads,
                   int* failed_index, int* failed_errno);

/* Issue n host->device / device->device / device->host copies, one
 * cudaMemcpyAsync each, on `stream` (host arrays of device/host pointers).
 * The slot-fill path of the pool (streamlx/pool.py:196-199 slot writes,
 * pinned staging -> HBM). */
int slx_copy_many(void* const* dst, const void* const* src,
                  const size_t* bytes, int n, void* stream);

/* Timing helpers for graph-launched steps: record a CUDA event on a
 * stream -- as a timestamp node (cudaEventRecordExternal) while the stream
 * is being captured, as a plain record otherwise; read n start/end event
 * pairs in one call. */
int slx_event_record_external(void* event, void* stream);
int slx_event_elapsed_many(void* const* start, void* const* end, int n,
                           float* out_ms);

#ifdef __cplusplus
}
#endif

#endif /* STREAMLX_CUDA_H_ */
