// Internal launch interface between the C-ABI layer (gdn_api.cu) and the
// kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

// Workspace carve-up shared by the chunk paths.  Offsets are 256-byte aligned.
struct ChunkWorkspace {
  size_t err;            // int32[4] device error word
  size_t chunk_offsets;  // int64[N + 1]
  size_t gc;             // f32 [Ttot][HV] chunk-local cumsum of g
  size_t qn, kn;         // f32 [Ttot][H][K] (generic path: normalised q, k)
  size_t w, u, vnew;     // generic: f32 [Ttot][HV][K|V]
  size_t hs;             // generic: f32 [chunks][HV][K][V]
  size_t total;
};

// Backward workspace: the generic forward's intermediates followed by the
// backward's fp32 buffers.
struct BwdWorkspace {
  ChunkWorkspace fwd;
  size_t dvn;       // f32 [Ttot][HV][V] gradient of v_new
  size_t dhn;       // f32 [chunks][HV][K][V] gradient of the state after each chunk
  size_t dqh, dkh;  // f32 [Ttot][HV][K] per-v-head dq, dk
  size_t dw;        // f32 [Ttot][HV][K] gradient of W
  size_t dG;        // f32 [Ttot][HV] gradient of the chunk-local cumsum of g
  size_t tc;        // bf16/f16 with K = V = 128: the tensor-core WY workspace (W images, row scales)
  size_t himg, dhimg, vnimg, dvimg, dwimg;  // and the bf16 images of h, dh', v_new, dv, dW per (chunk, v-head)
  size_t total;
};

// Count of kernels launched by this library (gdn_kernel_launch_count).
void note_launch(int n = 1);

// Sets the thread-local message returned by gdn_last_error; returns `code`.
int set_last_error(int code, const char* fmt, ...);

// Per-call launch instrumentation: records the caller's optional stage
// events (gdn_chunk_args::stage_events) and counts launches.
struct LaunchHooks {
  void* const* events;
  int n;
  int next = 0;
  LaunchHooks(void* const* e, int count) : events(e), n(count) {}
  void pre(cudaStream_t s) {
    if (events && next < n) cudaEventRecord(static_cast<cudaEvent_t>(events[next++]), s);
    note_launch();
  }
  // a stage with no kernel of its own
  void mark(cudaStream_t s) {
    if (events && next < n) cudaEventRecord(static_cast<cudaEvent_t>(events[next++]), s);
  }
  void end(cudaStream_t s) {
    if (events && next < n) cudaEventRecord(static_cast<cudaEvent_t>(events[next++]), s);
  }
};

// Upper bound on the number of 64-token chunks of a packed batch.
inline int64_t chunk_upper_bound(int64_t total_tokens, int64_t nseq) {
  return (total_tokens + 63) / 64 + nseq;
}

ChunkWorkspace plan_generic_workspace(const gdn_chunk_args& a);
bool tc_path_applies(const gdn_chunk_args& a);
size_t tc_workspace_bytes(const gdn_chunk_args& a);

cudaError_t launch_recurrent_vfirst(const gdn_recurrent_args& a, cudaStream_t s);
bool decode_stream_applies(const gdn_recurrent_args& a);
cudaError_t launch_decode_stream(const gdn_recurrent_args& a, cudaStream_t s);
cudaError_t launch_recurrent_kfirst(const gdn_recurrent_plain_args& a, cudaStream_t s);
cudaError_t launch_chunk_generic(const gdn_chunk_args& a, const ChunkWorkspace& ws, cudaStream_t s);
// The generic forward without its output stage: leaves G, q/k, W, U, v_new
// and the per-chunk states in the workspace for the backward.
cudaError_t launch_chunk_generic_recompute(const gdn_chunk_args& a, const ChunkWorkspace& ws, cudaStream_t s);
BwdWorkspace plan_bwd_workspace(const gdn_chunk_bwd_args& a);
cudaError_t launch_chunk_bwd(const gdn_chunk_bwd_args& a, const BwdWorkspace& ws, cudaStream_t s);
// stall_chunk >= 0: test hook of gdn_chunk_fwd_test_stall (the first state
// block skips that chunk's operand fetch; its waits give up after stall_limit).
cudaError_t launch_chunk_h_stage(const gdn_chunk_h_args& a, cudaStream_t s);
// conv non-null: the causal conv1d of causal_conv1d_fn (W = 4, 16-bit data,
// conv_states of the same dtype) is applied to conv->x as the tiles are
// loaded; a.q/a.k/a.v are not read, and the cache lines are updated after the
// prefill kernels (launch_conv_fn_states).
cudaError_t launch_chunk_tc(const gdn_chunk_args& a, cudaStream_t s, int64_t stall_chunk = -1,
                            long long stall_limit = 0, const gdn_conv1d_fn_args* conv = nullptr);
size_t tc_conv_workspace_bytes(const gdn_chunk_args& a);
// causal_conv1d_fn's argument checks for the fused prefill (no `out`).
int check_conv_fn_args(const gdn_conv1d_fn_args* a);
cudaError_t launch_conv_fn_states(const gdn_conv1d_fn_args& a, cudaStream_t s);
cudaError_t launch_solve_tril(const float* A, void* out, int out_dtype, const void* cu,
                              int cu_dtype, int64_t N, int64_t B, int64_t T, int H, int BT,
                              cudaStream_t s);
// chunk_offsets[0..N] from cu_seqlens (or the equal-length batch); also
// zeroes the call's 16-byte device error word `err` when it is given, so that
// every call starts with a clear word (the plan kernel runs first), and the
// nzero ints at `zero` (per-call flags of the kernels that follow).
cudaError_t launch_chunk_plan(const void* cu, int cu_dtype, int64_t N, int64_t T,
                              int64_t* chunk_offsets, cudaStream_t s, int chunk = 64,
                              int* err = nullptr, int* zero = nullptr, int64_t nzero = 0);

}  // namespace gdn
