/*
 * gdn_b200.h - C ABI of the B200 gated delta-rule (GDN) forward library
 * (libgdn_b200.so).
 *
 * Plain pointers and sizes only; no torch types.  Every tensor is a dense,
 * row-major (C-contiguous) device buffer in the reference's shapes.  Callers
 * allocate every input, output and workspace buffer; the library never
 * allocates or frees device memory and keeps no pointer after a call returns.
 * Work is enqueued on the caller's stream (`stream` is a cudaStream_t passed
 * as void*; NULL = legacy default stream) and calls do not synchronise.
 *
 * Return codes: GDN_OK (0) or a negative GDN_ERR_*; gdn_last_error() gives a
 * thread-local message for the last failing call on this thread.
 *
 * Reference interfaces replaced (paths inside the torch_mlu_ops package):
 *   gdn_chunk_fwd          <- triton_ops.py:81-165 chunk_gated_delta_rule
 *                             -> triton/fla/chunk.py:10-74 chunk_gated_delta_rule_fwd
 *   gdn_chunk_bwd          <- triton/fla/chunk.py:239-251 ChunkGatedDeltaRuleFunction.backward
 *                             -> triton/fla/chunk.py:76-186 chunk_gated_delta_rule_bwd
 *   gdn_chunk_fwd_host     <- no reference counterpart (host-memory prefill, pipelined copies)
 *   gdn_fused_recurrent_fwd<- triton_ops.py:228-285 fused_recurrent_gated_delta_rule_fn
 *                             -> triton/fla/fused_recurrent_fn.py:161-233
 *   gdn_chunk_fwd_h        <- triton/fla/chunk_delta_h.py:200-271 chunk_gated_delta_rule_fwd_h
 *                             (the state-recurrence stage, with its USE_GK branch)
 *   gdn_recurrent_plain_fwd<- triton_ops.py:168-226 fused_recurrent_gated_delta_rule
 *                             -> triton/fla/fused_recurrent.py:134-187
 *   gdn_solve_tril         <- include/torch_mlu_ops.h:1052-1054 tmo::torch_api::solve_tril
 *                             (Python: _ops.py:6232-6257; AOTI shim config_inductor.py:484-490)
 *   gdn_causal_conv1d_fwd  <- triton_ops.py:287-363 causal_conv1d
 *                             -> triton/conv/ops.py:35-99 causal_conv1d_fwd_fla
 *   gdn_causal_conv1d_fn   <- triton_ops.py:366-459 causal_conv1d_fn
 *                             -> triton/conv/ops.py:101-349 causal_conv1d_fwd_vllm
 *   gdn_causal_conv1d_update <- triton/conv/ops.py:584-644 causal_conv1d_update
 *   gdn_conv_chunk_fwd     <- no single reference counterpart: causal_conv1d_fn
 *                             (triton_ops.py:366-459) followed by chunk_gated_delta_rule
 *                             (triton_ops.py:81-165) on the conv output's q/k/v split,
 *                             as the GDN layer calls them, in one pass
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 3

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

enum {
  GDN_OK = 0,
  GDN_ERR_INVALID = -1,      /* bad argument: null pointer, shape, dtype */
  GDN_ERR_UNSUPPORTED = -2,  /* valid for the reference but not built here */
  GDN_ERR_CUDA = -3,         /* a CUDA runtime call failed */
  GDN_ERR_WORKSPACE = -4,    /* workspace missing or smaller than required */
  GDN_ERR_DEVICE = -5        /* a kernel reported a failure in the error word */
};

/* Element types of tensor arguments. */
enum { GDN_F32 = 0, GDN_BF16 = 1, GDN_F16 = 2, GDN_I32 = 3, GDN_I64 = 4 };

/*
 * Chunked prefill.  Shapes (C-contiguous):
 *   q, k [B, T, H, K]; v, o [B, T, HV, V] (all of qkv_dtype: f32/bf16/f16)
 *   g, beta [B, T, HV] f32 (g: log decay; beta: write strength)
 *   initial_state / final_state f32 [N, HV, K, V], or [N, HV, V, K] when
 *   state_v_first; either may be NULL (zeros in / no state out).
 *   cu_seqlens [N+1] (cu_dtype I32/I64) or NULL: with it B must be 1 and the
 *   N sequences are packed along T; without it N = B sequences of T tokens.
 * HV must be a multiple of H (v-head hv reads q/k head hv / (HV/H)).
 * K, V <= 128.  scale <= 0 selects K^-0.5.  With use_qk_l2norm, q and k rows
 * are divided by sqrt(sum(x^2) + 1e-6) first.  Chunk size is 64 tokens.
 */
typedef struct gdn_chunk_args {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* initial_state;
  void* o;
  float* final_state;
  const void* cu_seqlens;
  void* workspace;
  size_t workspace_bytes;
  int64_t B, T, N;
  int32_t H, HV, K, V;
  int32_t qkv_dtype;
  int32_t cu_dtype;
  float scale;
  int32_t use_qk_l2norm;
  int32_t state_v_first;
  int32_t force_generic;  /* 1: use the SIMT fp32 path even where tcgen05 applies */
  /* Optional instrumentation: an array of n_stage_events cudaEvent_t
   * handles.  When non-NULL, event i is recorded on `stream` just before the
   * i-th kernel of the call and the last event after the final kernel
   * (recording stops when the array runs out).  NULL for normal use. */
  void* const* stage_events;
  int32_t n_stage_events;
  /* Token (row) strides of q, k and v in elements; 0 means packed (H*K,
   * H*K, HV*V).  Within a row the heads stay packed (unit stride over K, K
   * between heads), so q, k and v may be views of one [T, 2*H*K + HV*V]
   * projection.  Strided rows are read in place by the tensor-core path
   * (strides >= the packed width and multiples of 8); the other paths and
   * gdn_chunk_fwd_host take packed rows only. */
  int64_t q_token_stride, k_token_stride, v_token_stride;
} gdn_chunk_args;

/* Workspace bytes gdn_chunk_fwd needs for these arguments (pointer fields
 * are ignored).  Returns 0 and sets the last error for invalid arguments. */
GDN_API size_t gdn_chunk_workspace_size(const gdn_chunk_args* args);

GDN_API int gdn_chunk_fwd(const gdn_chunk_args* args, void* stream);

/*
 * Allocation-free variant of gdn_chunk_fwd (no counterpart in the reference).
 * For callers that cannot allocate device memory: C hosts that link this
 * library without a device allocator of their own, and serving engines that
 * give all of the GPU's memory to their own pool at start-up (cudaMalloc
 * fails there, and would synchronise the device in the request path).
 * args->workspace and args->workspace_bytes are ignored; the workspace comes
 * from a 32 MiB scratch array built into the library (held on every GPU that
 * loads the library until exit).  Calls whose workspace
 * (gdn_chunk_workspace_size) exceeds 32 MiB return GDN_ERR_WORKSPACE.  The
 * first call on a device looks up the array's device address (make it before
 * any stream capture).  All calls share the one array: calls that overlap on
 * the GPU race and must be serialised by the caller.  Allocates nothing.
 */
GDN_API int gdn_chunk_fwd_noalloc(const gdn_chunk_args* args, void* stream);

/* gdn_chunk_check_device_error for the scratch of gdn_chunk_fwd_noalloc on
 * the current device (no counterpart in the reference): reads back
 * (synchronously, on `stream`) and clears the error word of the last
 * allocation-free call. */
GDN_API int gdn_chunk_noalloc_check_device_error(void* stream);

/*
 * Test hook for the failure path (no counterpart in the reference, whose
 * kernels have no bounded waits): gdn_chunk_fwd on the tensor-core path
 * (bf16/f16, K = V = 128) in which the first block of the state kernel does
 * not issue the operand copies of its chunk `stall_chunk`, and bounds every
 * wait of that block by `wait_limit_cycles` SM clocks (1e3 .. 2e9) instead of
 * about one second.  That block's wait for the missing operands runs out:
 * it records code 1, site 4 in the workspace error word, waits for the work
 * it did issue, and exits without writing its remaining outputs or its final
 * state.  No copy, MMA or fault is left behind, so the context stays usable;
 * gdn_chunk_check_device_error then returns GDN_ERR_DEVICE.  For tests only.
 */
GDN_API int gdn_chunk_fwd_test_stall(const gdn_chunk_args* args, int64_t stall_chunk,
                                     int64_t wait_limit_cycles, void* stream);

/*
 * Backward of gdn_chunk_fwd (the autograd backward of chunk_gated_delta_rule).
 * Inputs q, k, v, g, beta, initial_state, cu_seqlens and the sizes mean what
 * they mean in gdn_chunk_args (the forward's arguments, unchanged).
 *   dout [B, T, HV, V] (qkv_dtype): gradient of o.
 *   dht: gradient of final_state in the state layout, or NULL (zero).
 *   dq, dk, dv: outputs of qkv_dtype in the shapes of q, k, v.
 *   dg, dbeta [B, T, HV] f32: gradients of g and beta.
 *   dh0: gradient of initial_state in the state layout, or NULL (not
 *   written).  With use_qk_l2norm the gradients of q and k are taken
 *   through the normalisation.
 * The forward intermediates are recomputed in fp32 inside the call; the
 * workspace (gdn_chunk_bwd_workspace_size) holds them and the backward's own
 * fp32 buffers.  Every output element is written (no accumulation).
 */
typedef struct gdn_chunk_bwd_args {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* initial_state;
  const void* cu_seqlens;
  const void* dout;
  const float* dht;
  void* dq;
  void* dk;
  void* dv;
  float* dg;
  float* dbeta;
  float* dh0;
  void* workspace;
  size_t workspace_bytes;
  int64_t B, T, N;
  int32_t H, HV, K, V;
  int32_t qkv_dtype;
  int32_t cu_dtype;
  float scale;
  int32_t use_qk_l2norm;
  int32_t state_v_first;
} gdn_chunk_bwd_args;

/* Workspace bytes gdn_chunk_bwd needs (0 and the last error for invalid
 * arguments). */
GDN_API size_t gdn_chunk_bwd_workspace_size(const gdn_chunk_bwd_args* args);

GDN_API int gdn_chunk_bwd(const gdn_chunk_bwd_args* args, void* stream);

/*
 * Chunked prefill from host memory (no counterpart in the reference, whose
 * ops take device tensors only).  For callers whose q/k/v sit in host
 * memory, such as offline prefill of long prompts or a CPU-side engine that
 * streams requests to the GPU: the host link, not the kernels, bounds such a
 * call, so the copies are pipelined against the kernels.
 * args: as for gdn_chunk_fwd, except that q, k, v, g, beta, initial_state,
 * o, final_state and cu_seqlens are HOST pointers (page-locked memory lets
 * the copies run asynchronously and overlap; pageable memory also works),
 * and workspace / workspace_bytes is a DEVICE buffer of at least
 * gdn_chunk_fwd_host_buffer_size(args, segment_tokens) bytes.
 * The tokens are cut into pieces of about segment_tokens tokens (a positive
 * multiple of 64): a single sequence (B = 1, no cu_seqlens) along time, the
 * fp32 state handed from piece to piece on the device, its last
 * segment_tokens tokens in halving pieces down to 512 tokens (the last piece's
 * compute and copy-out are not overlapped, so it is kept short); an equal-length batch
 * into groups of sequences; a packed batch into groups of consecutive
 * sequences.  Each piece is one gdn_chunk_fwd call on device copies (same
 * results as the device entry point).  Copy-in of piece p+1, compute of
 * piece p (on `stream`) and copy-out of piece p-1 overlap; the copies run on
 * two streams the library creates once per device.  Before returning, the
 * call makes `stream` wait for all of its copies: the host outputs are
 * complete, and the host inputs may be reused, once `stream` reaches this
 * point (for example after cudaStreamSynchronize(stream)).
 */
GDN_API size_t gdn_chunk_fwd_host_buffer_size(const gdn_chunk_args* args, int64_t segment_tokens);
GDN_API int gdn_chunk_fwd_host(const gdn_chunk_args* args, int64_t segment_tokens, void* stream);

/* Reads back (synchronously, on `stream`) the device error word that the
 * chunk kernels keep at the start of `workspace` (no counterpart in the
 * reference, whose kernels cannot report a failure); returns GDN_OK or
 * GDN_ERR_DEVICE and clears the word.  Every gdn_chunk_fwd call clears the
 * word before its first kernel, so the word describes the last call that
 * used this workspace.  A kernel that gives up on a wait (a bounded
 * mbarrier wait that timed out) records code 1, the site, the block and the
 * thread, and leaves its outputs incomplete. */
GDN_API int gdn_chunk_check_device_error(void* workspace, void* stream);

/*
 * The inter-chunk state recurrence as a stage (chunk_gated_delta_rule_fwd_h,
 * triton/fla/chunk_delta_h.py:200-271), with the per-key decay gk of its
 * KDA branch (USE_GK, :155-171).  64-token chunks.  Shapes (C-contiguous,
 * k, w, u, h, v_new of `dtype` F32/BF16/F16):
 *   k [B, T, Hg, K]; w [B, T, H, K]; u [B, T, H, V]  (head h reads k head
 *   h / (H / Hg));
 *   g: chunk-local cumsum of the log decay in the reference's head-major
 *   layout [H, B*T] f32, or NULL; gk: per-key cumsum [B, T, H, K] f32 or NULL;
 *   initial_state / final_state f32 [N, H, K, V] ([N, H, V, K] with
 *   state_v_first), either NULL;
 *   h: the state before every chunk, [B, NT, H, K, V] ([.., V, K] with
 *   state_v_first), NT = chunks per sequence (or the packed batch's total
 *   chunk count with cu_seqlens), or NULL;
 *   v_new [B, T, H, V] = u - w S per chunk, or NULL;
 *   cu_seqlens [N+1] (cu_dtype) or NULL as for gdn_chunk_fwd.
 * Per chunk: S <- S exp(g_last) exp(gk_last)[:, None] + k^T (v_new *
 * exp(g_last - g)), the products in fp32 with S and v_new~ rounded to
 * `dtype` where the reference rounds them.  K, V <= 128.
 */
typedef struct gdn_chunk_h_args {
  const void* k;
  const void* w;
  const void* u;
  const float* g;
  const float* gk;
  const float* initial_state;
  void* h;
  void* v_new;
  float* final_state;
  const void* cu_seqlens;
  int64_t B, T, N;
  int32_t Hg, H, K, V;
  int32_t dtype, cu_dtype;
  int32_t state_v_first;
} gdn_chunk_h_args;

GDN_API int gdn_chunk_fwd_h(const gdn_chunk_h_args* args, void* stream);

/*
 * Recurrent forward with a V-first state cache: the slot-indexed decode of
 * fused_recurrent_gated_delta_rule_fn.
 *   q, k [B, T, H, K]; v, o [B, T, HV, V] (qkv_dtype); g [B, T, HV] f32 or NULL;
 *   beta [B, T, HV] f32, or [B, T, HV, V] when beta_per_v.
 *   initial_state f32 rows of [HV, V, K], row r at initial_state +
 *   r * stride_init_state_token (elements); NULL = zero state.
 *   final_state: with inplace_final_state the per-token state of token t of
 *   sequence n is written to row ssm_state_indices[n, t] (skipped when
 *   negative), usually aliasing initial_state; otherwise to row bos + t.
 *   ssm_state_indices [N] or [N, *] (idx_dtype I32/I64, strides in elements)
 *   or NULL (then the initial state row of sequence n is bos, as in the
 *   reference).  num_accepted_tokens [N] (nacc_dtype) or NULL: the initial
 *   state is read from column num_accepted_tokens[n]-1 of the index row.
 *   A sequence whose initial index is negative (PAD) is skipped and its
 *   output rows are set to zero.
 *   gk [B, T, HV, K] f32 or NULL: per-key log decays (the IS_KDA branch of
 *   fused_recurrent_fn.py:77-80,115-120: S <- S * exp(gk)[None, :] each
 *   token); applied together with g when both are given.
 *   num_slots > 0 declares the number of state rows: an initial index >=
 *   num_slots makes the sequence be skipped like PAD (outputs zero, state
 *   untouched) and a final index >= num_slots skips that store; both record
 *   error code 2 (site 9 initial, 10 final, block = sequence, info = index)
 *   in `err`.  num_slots <= 0 checks nothing (the reference's behaviour).
 *   err: NULL or a device int32[4] error word that the caller zeroes; the
 *   kernels only write it on a failure (the first one wins): code 1 = a
 *   bounded wait of the streaming kernel gave up (site 7 or 8), code 2 = a
 *   state index out of range.
 * K, V <= 128 and K a multiple of 4.
 */
typedef struct gdn_recurrent_args {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* initial_state;
  void* o;
  float* final_state;
  const void* cu_seqlens;
  const void* ssm_state_indices;
  const void* num_accepted_tokens;
  int64_t B, T, N;
  int32_t H, HV, K, V;
  int32_t qkv_dtype, cu_dtype, idx_dtype, nacc_dtype;
  int64_t stride_init_state_token;
  int64_t stride_final_state_token;
  int64_t stride_indices_seq;
  int64_t stride_indices_tok;
  float scale;
  int32_t use_qk_l2norm;
  int32_t beta_per_v;
  int32_t inplace_final_state;
  int64_t num_slots;
  int32_t* err;
  const float* gk;
} gdn_recurrent_args;

GDN_API int gdn_fused_recurrent_fwd(const gdn_recurrent_args* args, void* stream);

/*
 * Plain recurrence with a K-first state, fused_recurrent_gated_delta_rule.
 *   q, k [B, T, H, K]; v, o [B, T, HV, V]; g [B, T, HV] f32 or NULL;
 *   gk [B, T, HV, K] f32 or NULL; gv [B, T, HV, V] f32 or NULL;
 *   beta [B, T, HV] f32, or [B, T, HV, V] when beta_per_v.
 *   initial_state [N, HV, K, V] f32 or NULL; final_state [N, HV, K, V] f32 or
 *   NULL.  scale <= 0 selects K^-0.5.
 */
typedef struct gdn_recurrent_plain_args {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* gk;
  const float* gv;
  const float* beta;
  const float* initial_state;
  void* o;
  float* final_state;
  const void* cu_seqlens;
  int64_t B, T, N;
  int32_t H, HV, K, V;
  int32_t qkv_dtype, cu_dtype;
  float scale;
  int32_t use_qk_l2norm;
  int32_t beta_per_v;
} gdn_recurrent_plain_args;

GDN_API int gdn_recurrent_plain_fwd(const gdn_recurrent_plain_args* args, void* stream);

/*
 * (I + A)^-1 for every BT x BT chunk block of a strictly lower-triangular A.
 *   A f32 [B, T, H, BT]; out [B, T, H, BT] of out_dtype (F32/BF16/F16);
 *   cu_seqlens [N+1] (I32/I64, B == 1) or NULL.  BT in {16, 32, 64}.
 * Entries above the diagonal and columns past a partial chunk's end are
 * written as zero.  Mirrors solve_tril(input, output, cu_seqlens).
 */
GDN_API int gdn_solve_tril(const float* A, void* out, int32_t out_dtype,
                   const void* cu_seqlens, int32_t cu_dtype, int64_t N,
                   int64_t B, int64_t T, int32_t H, int32_t BT, void* stream);

/* ------------------------------------------------------------------------
 * Causal depthwise conv1d (the short convolution before the GDN layer)
 * ------------------------------------------------------------------------ */
#define GDN_ACT_NONE 0
#define GDN_ACT_SILU 1 /* "silu" / "swish": y / (1 + exp(-y)) */

/* causal_conv1d (FLA layout).  y_t = sum_i x_{t-W+1+i} w_i, then + bias,
 * activation, + residual, per channel.  Tokens before a sequence start come
 * from initial_state or are zero.
 *   x, residual, y  [B, T, D] of x_dtype (residual may be NULL);
 *   weight [D, W], bias [D] (or NULL) of w_dtype;
 *   initial_state [N, D, W] of state_dtype or NULL (column j = token j - W);
 *   cu_seqlens [N+1] (I32/I64) or NULL: with it, B == 1 and the T tokens are
 *   N packed sequences.  1 <= W <= 16. */
typedef struct gdn_conv1d_args {
  const void* x;
  const void* weight;
  const void* bias;
  const void* residual;
  const void* initial_state;
  void* y;
  const void* cu_seqlens;
  int64_t B, T, N, D;
  int32_t W;
  int32_t x_dtype, w_dtype, state_dtype, cu_dtype;
  int32_t activation; /* GDN_ACT_* */
} gdn_conv1d_args;
GDN_API int gdn_causal_conv1d_fwd(const gdn_conv1d_args* args, void* stream);

/* causal_conv1d_fn (vLLM layout, continuous batching, slot-indexed state).
 *   x (dim, total) with unit channel stride: element (c, t) at
 *     x[t * stride_x_token + c]; out likewise with stride_o_token;
 *   weight (dim, W) row-major, bias (dim) or NULL, both of w_dtype;
 *   conv_states (lines, dim, >= W-1) of state_dtype with unit channel
 *     stride: element (l, c, j) at l * stride_state_seq + j * stride_state_tok
 *     + c; updated in place to each processed sequence's last W-1 tokens;
 *   query_start_loc [batch+1] (qsl_dtype I32/I64); cache_indices [batch]
 *     (idx_dtype) or NULL for line = sequence; has_initial_state [batch]
 *     bytes (bool) or NULL for none.
 * A sequence whose line equals null_block_id (when has_null_block) or
 * pad_slot_id is skipped: its out tokens are written as zero and its line is
 * left alone.  2 <= W <= 4.
 * Prefix caching (block_idx_last non-NULL; all four block arrays [batch] of
 * apc_dtype): cache_indices is (batch, blocks) with row stride
 * stride_cache_indices; the initial window comes from line
 * cache_indices[s, initial_state_idx[s]], the final state goes to
 * cache_indices[s, block_idx_last[s]], and the W-1 inputs before each
 * block_size_to_align-aligned block end j < last - first go to
 * cache_indices[s, block_idx_first[s] + j] (triton/conv/kernels.py:254-289,
 * 519-554). */
typedef struct gdn_conv1d_fn_args {
  const void* x;
  void* out;
  const void* weight;
  const void* bias;
  void* conv_states;
  const void* query_start_loc;
  const void* cache_indices;
  const uint8_t* has_initial_state;
  int64_t stride_x_token, stride_o_token;
  int64_t stride_state_seq, stride_state_tok, num_cache_lines;
  int64_t batch, dim, total_tokens;
  int64_t pad_slot_id, null_block_id;
  int32_t has_null_block;
  int32_t W;
  int32_t x_dtype, w_dtype, state_dtype, qsl_dtype, idx_dtype;
  int32_t activation;
  const void* block_idx_first;
  const void* block_idx_last;
  const void* initial_state_idx;
  const void* num_computed_tokens;
  int64_t stride_cache_indices; /* elements between rows of cache_indices */
  int64_t block_size_to_align;
  int32_t apc_dtype;
} gdn_conv1d_fn_args;
GDN_API int gdn_causal_conv1d_fn(const gdn_conv1d_fn_args* args, void* stream);

/* causal_conv1d_update: one decode token per sequence.
 *   x [N, D] (row stride stride_x_n), residual [N, D] (or NULL), y [N, D]
 *     contiguous, all of x_dtype;
 *   cache [N, D, W] of cache_dtype (or NULL: an all-zero window, no state),
 *     shifted left by one with x entering the last column, in place;
 *   weight [D, W] (or NULL: taps of one), bias [D] (or NULL) of w_dtype. */
typedef struct gdn_conv1d_update_args {
  const void* x;
  void* cache;
  const void* residual;
  const void* weight;
  const void* bias;
  void* y;
  int64_t stride_x_n;
  int64_t N, D;
  int32_t W;
  int32_t x_dtype, cache_dtype, w_dtype;
  int32_t activation;
} gdn_conv1d_update_args;
GDN_API int gdn_causal_conv1d_update(const gdn_conv1d_update_args* args, void* stream);

/* Causal conv1d fused into the chunked prefill (no single reference
 * counterpart).  Computes what causal_conv1d_fn(x, ...) followed by
 * gdn_chunk_fwd on the q/k/v split of its output computes, bit for bit,
 * without writing the conv output: the prefill's WY kernel applies the conv
 * (and SiLU) to x as it loads its q, k and v tiles.
 *   args: as for gdn_chunk_fwd, except that q, k and v are not read (the
 *     conv output supplies them); bf16/f16 with K = V = 128, a packed batch
 *     (B = 1, cu_seqlens), workspace of gdn_conv_chunk_workspace_size bytes;
 *   conv: as for gdn_causal_conv1d_fn with out = NULL; x holds, per token,
 *     dim = 2*H*K + HV*V channels [q heads | k heads | v heads]; W = 4; x,
 *     weight, bias and conv_states in the q/k/v dtype; x, its token stride,
 *     weight and bias 16-byte aligned; query_start_loc describes the same
 *     sequences as args->cu_seqlens (batch = N, total_tokens = T).
 * conv_states is updated like causal_conv1d_fn updates it (after the prefill
 * kernels have read the initial lines); PAD / null-block sequences get zero
 * conv outputs and keep their lines. */
GDN_API size_t gdn_conv_chunk_workspace_size(const gdn_chunk_args* args);
GDN_API int gdn_conv_chunk_fwd(const gdn_chunk_args* args, const gdn_conv1d_fn_args* conv, void* stream);

/* Message for the last failing call on this thread ("" if none). */
GDN_API const char* gdn_last_error(void);

/* Number of kernels this library has launched in the process so far
 * (monotonic, all threads).  Lets a caller count launches in a region. */
GDN_API uint64_t gdn_kernel_launch_count(void);

/* GDN_ABI_VERSION of the built library. */
GDN_API int gdn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
