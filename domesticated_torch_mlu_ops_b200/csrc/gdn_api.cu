// extern "C" entry points of libgdn_b200.so: argument validation, workspace
// sizing and dispatch.  Validation mirrors the reference's host-side checks
// (K, V <= 128 asserts at triton/fla/chunk.py:27-28 and
// triton/fla/fused_recurrent_fn.py:181-182; shape errors of
// triton/fla/cumsum.py:284-289) but returns status codes instead of raising.

#include <atomic>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace {
std::atomic<uint64_t> g_launches{0};
}  // namespace

void gdn::note_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(GDN_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

bool qkv_dtype_ok(int d) { return d == GDN_F32 || d == GDN_BF16 || d == GDN_F16; }
bool idx_dtype_ok(int d) { return d == GDN_I32 || d == GDN_I64; }

int check_heads(int64_t B, int64_t T, int64_t N, int H, int HV, int K, int V, const void* cu,
                int cu_dtype) {
  if (B < 0 || T < 0 || N < 0 || H <= 0 || HV <= 0 || K <= 0 || V <= 0)
    return fail(GDN_ERR_INVALID, "non-positive dimension (B=%lld T=%lld N=%lld H=%d HV=%d K=%d V=%d)",
                (long long)B, (long long)T, (long long)N, H, HV, K, V);
  if (HV % H != 0) return fail(GDN_ERR_INVALID, "HV=%d is not a multiple of H=%d", HV, H);
  if (K > 128 || V > 128) return fail(GDN_ERR_INVALID, "K=%d, V=%d: both must be <= 128", K, V);
  if (cu) {
    if (!idx_dtype_ok(cu_dtype)) return fail(GDN_ERR_INVALID, "cu_seqlens dtype must be I32 or I64");
    if (B != 1) return fail(GDN_ERR_INVALID, "cu_seqlens requires B == 1 (got B=%lld)", (long long)B);
  } else if (N != B) {
    return fail(GDN_ERR_INVALID, "without cu_seqlens N must equal B (N=%lld B=%lld)",
                (long long)N, (long long)B);
  }
  return GDN_OK;
}

int check_chunk(const gdn_chunk_args* a) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  int rc = check_heads(a->B, a->T, a->N, a->H, a->HV, a->K, a->V, a->cu_seqlens, a->cu_dtype);
  if (rc) return rc;
  if (!qkv_dtype_ok(a->qkv_dtype)) return fail(GDN_ERR_INVALID, "qkv dtype must be F32, BF16 or F16");
  if (a->q_token_stride || a->k_token_stride || a->v_token_stride) {
    if (a->force_generic || !gdn::tc_path_applies(*a))
      return fail(GDN_ERR_UNSUPPORTED, "strided q/k/v rows are read in place on the tensor-core path only "
                                       "(bf16/f16, K = V = 128); pass packed rows");
    auto ok = [](int64_t st, int64_t width) { return st == 0 || (st >= width && st % 8 == 0); };
    if (!ok(a->q_token_stride, static_cast<int64_t>(a->H) * a->K) ||
        !ok(a->k_token_stride, static_cast<int64_t>(a->H) * a->K) ||
        !ok(a->v_token_stride, static_cast<int64_t>(a->HV) * a->V))
      return fail(GDN_ERR_INVALID, "q/k/v token strides must be 0 or multiples of 8 at least the packed row width");
  }
  return GDN_OK;
}

size_t workspace_bytes(const gdn_chunk_args& a) {
  if (!a.force_generic && gdn::tc_path_applies(a)) return gdn::tc_workspace_bytes(a);
  return gdn::plan_generic_workspace(a).total;
}

}  // namespace

int gdn::set_last_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

extern "C" {

const char* gdn_last_error(void) { return g_last_error; }

int gdn_abi_version(void) { return GDN_ABI_VERSION; }

uint64_t gdn_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t gdn_chunk_workspace_size(const gdn_chunk_args* a) {
  if (check_chunk(a)) return 0;
  return workspace_bytes(*a);
}

int gdn_chunk_fwd(const gdn_chunk_args* a, void* stream) {
  int rc = check_chunk(a);
  if (rc) return rc;
  const int64_t Ttot = a->B * a->T;
  if (Ttot > 0 && (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->o))
    return fail(GDN_ERR_INVALID, "q, k, v, g, beta and o must be non-null");
  const size_t need = workspace_bytes(*a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed",
                a->workspace_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (!a->force_generic && gdn::tc_path_applies(*a)) {
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!aligned(a->q) || !aligned(a->k) || !aligned(a->v))
      return fail(GDN_ERR_INVALID, "q, k and v must be 16-byte aligned for the tensor-core path");
    e = gdn::launch_chunk_tc(*a, s);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_fwd (tcgen05 path)");
  } else {
    e = gdn::launch_chunk_generic(*a, gdn::plan_generic_workspace(*a), s);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_fwd (generic path)");
  }
  return GDN_OK;
}

int gdn_chunk_fwd_test_stall(const gdn_chunk_args* a, int64_t stall_chunk, int64_t wait_limit_cycles,
                             void* stream) {
  int rc = check_chunk(a);
  if (rc) return rc;
  if (a->force_generic || !gdn::tc_path_applies(*a))
    return fail(GDN_ERR_UNSUPPORTED, "the stall hook exists on the tensor-core path only (bf16/f16, K = V = 128)");
  if (stall_chunk < 0 || wait_limit_cycles < 1000 || wait_limit_cycles > 2000000000LL)
    return fail(GDN_ERR_INVALID, "stall_chunk must be >= 0 and wait_limit_cycles in [1e3, 2e9]");
  if (a->B * a->T == 0 || !a->q || !a->k || !a->v || !a->g || !a->beta || !a->o)
    return fail(GDN_ERR_INVALID, "q, k, v, g, beta and o must be non-null and the batch non-empty");
  const size_t need = workspace_bytes(*a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", a->workspace_bytes, need);
  cudaError_t e = gdn::launch_chunk_tc(*a, static_cast<cudaStream_t>(stream), stall_chunk, wait_limit_cycles);
  if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_fwd_test_stall");
  return GDN_OK;
}

size_t gdn_conv_chunk_workspace_size(const gdn_chunk_args* a) {
  if (check_chunk(a)) return 0;
  if (a->force_generic || !gdn::tc_path_applies(*a))
    return fail(GDN_ERR_UNSUPPORTED, "the fused conv prefill needs bf16/f16 q/k/v with K = V = 128"), 0;
  return gdn::tc_conv_workspace_bytes(*a);
}

int gdn_conv_chunk_fwd(const gdn_chunk_args* a, const gdn_conv1d_fn_args* c, void* stream) {
  int rc = check_chunk(a);
  if (rc) return rc;
  if (a->force_generic || !gdn::tc_path_applies(*a))
    return fail(GDN_ERR_UNSUPPORTED, "the fused conv prefill needs bf16/f16 q/k/v with K = V = 128");
  if ((rc = gdn::check_conv_fn_args(c)) != GDN_OK) return rc;
  if (c->out) return fail(GDN_ERR_INVALID, "conv out must be NULL: the fused prefill keeps the conv output on chip");
  if (a->B != 1 || !a->cu_seqlens)
    return fail(GDN_ERR_INVALID, "the fused conv prefill takes a packed batch (B = 1 with cu_seqlens)");
  if (c->batch != a->N || c->total_tokens != a->T)
    return fail(GDN_ERR_INVALID, "conv batch=%lld / total_tokens=%lld must equal N=%lld / T=%lld",
                (long long)c->batch, (long long)c->total_tokens, (long long)a->N, (long long)a->T);
  if (c->dim != 2LL * a->H * a->K + static_cast<int64_t>(a->HV) * a->V)
    return fail(GDN_ERR_INVALID, "conv dim=%lld must be 2*H*K + HV*V = %lld ([q | k | v] channels)",
                (long long)c->dim, 2LL * a->H * a->K + static_cast<long long>(a->HV) * a->V);
  if (c->W != 4) return fail(GDN_ERR_UNSUPPORTED, "the fused conv prefill supports kernel width 4 (W=%d)", c->W);
  if (c->x_dtype != a->qkv_dtype || c->w_dtype != a->qkv_dtype || c->state_dtype != a->qkv_dtype)
    return fail(GDN_ERR_UNSUPPORTED, "x, weight, bias and conv_states must have the q/k/v dtype");
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!aligned(c->x) || c->stride_x_token % 8 != 0 || !aligned(c->weight) || (c->bias && !aligned(c->bias)))
    return fail(GDN_ERR_INVALID, "x (and its token stride), weight and bias must be 16-byte aligned");
  if (a->T > 0 && (!a->g || !a->beta || !a->o)) return fail(GDN_ERR_INVALID, "g, beta and o must be non-null");
  const size_t need = gdn::tc_conv_workspace_bytes(*a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", a->workspace_bytes, need);
  cudaError_t e = gdn::launch_chunk_tc(*a, static_cast<cudaStream_t>(stream), -1, 0, c);
  if (e != cudaSuccess) return cuda_fail(e, "gdn_conv_chunk_fwd");
  return GDN_OK;
}

size_t gdn_chunk_bwd_workspace_size(const gdn_chunk_bwd_args* a) {
  if (!a) return fail(GDN_ERR_INVALID, "null args"), 0;
  if (check_heads(a->B, a->T, a->N, a->H, a->HV, a->K, a->V, a->cu_seqlens, a->cu_dtype)) return 0;
  if (!qkv_dtype_ok(a->qkv_dtype)) return fail(GDN_ERR_INVALID, "qkv dtype must be F32, BF16 or F16"), 0;
  return gdn::plan_bwd_workspace(*a).total;
}

int gdn_chunk_bwd(const gdn_chunk_bwd_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  int rc = check_heads(a->B, a->T, a->N, a->H, a->HV, a->K, a->V, a->cu_seqlens, a->cu_dtype);
  if (rc) return rc;
  if (!qkv_dtype_ok(a->qkv_dtype)) return fail(GDN_ERR_INVALID, "qkv dtype must be F32, BF16 or F16");
  const int64_t Ttot = a->B * a->T;
  if (Ttot > 0 && (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->dout || !a->dq || !a->dk || !a->dv ||
                   !a->dg || !a->dbeta))
    return fail(GDN_ERR_INVALID, "q, k, v, g, beta, dout, dq, dk, dv, dg and dbeta must be non-null");
  const size_t need = gdn::plan_bwd_workspace(*a).total;
  if (!a->workspace || a->workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", a->workspace_bytes, need);
  if (a->N == 0) return GDN_OK;
  cudaError_t e = gdn::launch_chunk_bwd(*a, gdn::plan_bwd_workspace(*a), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_bwd");
  return GDN_OK;
}

int gdn_chunk_check_device_error(void* workspace, void* stream) {
  if (!workspace) return fail(GDN_ERR_INVALID, "null workspace");
  int32_t h[4] = {0, 0, 0, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(h, workspace, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_check_device_error");
  if (h[0] != 0) {
    e = cudaMemsetAsync(workspace, 0, sizeof(h), s);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_check_device_error");
    return fail(GDN_ERR_DEVICE, "device error word: code %d (site %d, block %d, info %d)",
                h[0], h[1], h[2], h[3]);
  }
  return GDN_OK;
}

int gdn_chunk_fwd_h(const gdn_chunk_h_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  int rc = check_heads(a->B, a->T, a->N, a->Hg, a->H, a->K, a->V, a->cu_seqlens, a->cu_dtype);
  if (rc) return rc;
  if (!qkv_dtype_ok(a->dtype)) return fail(GDN_ERR_INVALID, "dtype must be F32, BF16 or F16");
  if (a->B * a->T > 0 && (!a->k || !a->w || !a->u))
    return fail(GDN_ERR_INVALID, "k, w and u must be non-null");
  if (a->N == 0) return GDN_OK;
  cudaError_t e = gdn::launch_chunk_h_stage(*a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_chunk_fwd_h");
  return GDN_OK;
}

int gdn_fused_recurrent_fwd(const gdn_recurrent_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  int rc = check_heads(a->B, a->T, a->N, a->H, a->HV, a->K, a->V, a->cu_seqlens, a->cu_dtype);
  if (rc) return rc;
  if (!qkv_dtype_ok(a->qkv_dtype)) return fail(GDN_ERR_INVALID, "qkv dtype must be F32, BF16 or F16");
  if (a->K % 4 != 0) return fail(GDN_ERR_UNSUPPORTED, "K=%d must be a multiple of 4", a->K);
  if (a->B * a->T > 0 && (!a->q || !a->k || !a->v || !a->beta || !a->o))
    return fail(GDN_ERR_INVALID, "q, k, v, beta and o must be non-null");
  if (a->ssm_state_indices && !idx_dtype_ok(a->idx_dtype))
    return fail(GDN_ERR_INVALID, "ssm_state_indices dtype must be I32 or I64");
  if (a->num_accepted_tokens && !idx_dtype_ok(a->nacc_dtype))
    return fail(GDN_ERR_INVALID, "num_accepted_tokens dtype must be I32 or I64");
  if (a->num_accepted_tokens && !a->ssm_state_indices)
    return fail(GDN_ERR_INVALID, "num_accepted_tokens requires ssm_state_indices");
  if (a->inplace_final_state && a->final_state && !a->ssm_state_indices)
    return fail(GDN_ERR_INVALID, "inplace_final_state requires ssm_state_indices");
  if (a->initial_state && !a->ssm_state_indices && a->stride_init_state_token <= 0)
    return fail(GDN_ERR_INVALID, "stride_init_state_token must be positive");
  if (a->N == 0 || a->B * a->T == 0) return GDN_OK;
  cudaError_t e = gdn::launch_recurrent_vfirst(*a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_fused_recurrent_fwd");
  return GDN_OK;
}

int gdn_recurrent_plain_fwd(const gdn_recurrent_plain_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  int rc = check_heads(a->B, a->T, a->N, a->H, a->HV, a->K, a->V, a->cu_seqlens, a->cu_dtype);
  if (rc) return rc;
  if (!qkv_dtype_ok(a->qkv_dtype)) return fail(GDN_ERR_INVALID, "qkv dtype must be F32, BF16 or F16");
  if (a->B * a->T > 0 && (!a->q || !a->k || !a->v || !a->beta || !a->o))
    return fail(GDN_ERR_INVALID, "q, k, v, beta and o must be non-null");
  if (a->N == 0) return GDN_OK;
  cudaError_t e = gdn::launch_recurrent_kfirst(*a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_recurrent_plain_fwd");
  return GDN_OK;
}

int gdn_solve_tril(const float* A, void* out, int32_t out_dtype, const void* cu_seqlens,
                   int32_t cu_dtype, int64_t N, int64_t B, int64_t T, int32_t H, int32_t BT,
                   void* stream) {
  if (BT != 16 && BT != 32 && BT != 64) return fail(GDN_ERR_INVALID, "BT=%d must be 16, 32 or 64", BT);
  if (B < 0 || T < 0 || H <= 0) return fail(GDN_ERR_INVALID, "bad shape");
  if (!qkv_dtype_ok(out_dtype)) return fail(GDN_ERR_INVALID, "output dtype must be F32, BF16 or F16");
  if (cu_seqlens) {
    if (!idx_dtype_ok(cu_dtype)) return fail(GDN_ERR_INVALID, "cu_seqlens dtype must be I32 or I64");
    if (B != 1) return fail(GDN_ERR_INVALID, "cu_seqlens requires B == 1");
  } else {
    N = B;
  }
  if (B * T > 0 && (!A || !out)) return fail(GDN_ERR_INVALID, "null input or output");
  cudaError_t e = gdn::launch_solve_tril(A, out, out_dtype, cu_seqlens, cu_dtype, N, B, T, H, BT,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_solve_tril");
  return GDN_OK;
}

}  // extern "C"
