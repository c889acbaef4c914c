// The inter-chunk state recurrence as a stage of its own:
// chunk_gated_delta_rule_fwd_h (triton/fla/chunk_delta_h.py:200-271, kernel
// :28-197), including its per-key decay branch USE_GK (:155-171) that the
// KDA chunk path uses.  Per (sequence, head) and chunk c of 64 tokens, with
// the state S (K x V, fp32):
//   h[c]   = S                                   (stored in the k dtype)
//   v_new  = u_c - w_c S~    (S~ = S in the w dtype, :118-130; stored)
//   v~     = v_new * exp(g_last - g)  (rows past the sequence end: 0), in the k dtype
//   S      = S * exp(g_last) * exp(gk_last)[:, None] + k_c^T v~     (:131-190)
// g (when given) is the chunk-local cumsum in the layout the reference
// passes (head-major [H, B*T], chunk.py:32); gk (when given) the per-key
// cumsum [B, T, H, K].  k has Hg heads (head h reads k head h / (H / Hg)).
//
// One CTA of 256 threads per (sequence, head, 32-column V-slice); the
// 64-row products run on warp MMA with the TF32 head/tail split
// (tile_gemm.cuh), so the fp32 path keeps fp32 accuracy.  This is the stage
// op; the fused prefill computes the same recurrence inside its own kernels.

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "tile_gemm.cuh"

namespace gdn {

namespace {

constexpr int kHCols = 32;  // state columns per CTA

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_f<T>(from_f<T>(x));
}

template <typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
chunk_h_stage_kernel(const gdn_chunk_h_args p) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* S = sm;                      // [128][kRow32] state slice (fp32)
  float* Sr = S + 128 * kRow32;       // [128][kRow32] the state in the w dtype (product operand)
  float* wc = Sr + 128 * kRow32;      // [64][kRowK] w rows
  float* kc = wc + 64 * kRowK;        // [64][kRowN] k rows
  float* us = kc + 64 * kRowN;        // [64][kRow32] u slice, then v_new, then v~
  float* gs = us + 64 * kRow32;       // [64] g of the chunk
  float* dk = gs + 64;                // [128] exp(g_last) * exp(gk_last)
  float* red = dk + 128;              // [32] reduction scratch
  const int64_t n = blockIdx.x;
  const int hh = blockIdx.y, hk = hh / (p.H / p.Hg);
  const int v0 = blockIdx.z * kHCols;
  const int vcols = V - v0 < kHCols ? V - v0 : kHCols;
  const int tid = threadIdx.x;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t BT = p.B * p.T;
  // chunk index of this sequence's first chunk in h (the reference's chunk_offsets)
  int64_t boh;
  if (p.cu_seqlens) {
    float acc = 0.f;  // chunk counts are small integers: exact in fp32 up to 2^24
    for (int64_t m = tid; m < n; m += kGemmThreads) {
      int64_t b0, e0;
      seq_bounds(p.cu_seqlens, p.cu_dtype, m, p.T, b0, e0);
      acc += static_cast<float>((e0 - b0 + kChunk - 1) / kChunk);
    }
    boh = static_cast<int64_t>(block_sum(acc, red) + 0.5f);
  } else {
    boh = n * ((p.T + kChunk - 1) / kChunk);
  }
  const T* kb = static_cast<const T*>(p.k);
  const T* wb = static_cast<const T*>(p.w);
  const T* ub = static_cast<const T*>(p.u);
  T* hb = static_cast<T*>(p.h);
  T* vnb = static_cast<T*>(p.v_new);
  const int64_t rowK = static_cast<int64_t>(p.H) * K, rowKg = static_cast<int64_t>(p.Hg) * K,
                rowV = static_cast<int64_t>(p.H) * V;
  const int64_t nh = n * p.H + hh;
  for (int e = tid; e < 128 * kHCols; e += kGemmThreads) {
    const int kk = e / kHCols, c = e % kHCols, vv = v0 + c;
    float x = 0.f;
    if (p.initial_state && kk < K && c < vcols)
      x = p.state_v_first ? p.initial_state[(nh * V + vv) * K + kk] : p.initial_state[(nh * K + kk) * V + vv];
    S[kk * kRow32 + c] = x;
  }
  const int64_t nchunks = eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0;
  for (int64_t lc = 0; lc < nchunks; ++lc) {
    const int64_t s = bos + lc * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    __syncthreads();  // the previous chunk's readers of every tile are done
    for (int e = tid; e < 64 * 128; e += kGemmThreads) {
      const int i = e >> 7, kk = e & 127;
      const bool ok = i < L && kk < K;
      wc[i * kRowK + kk] = ok ? to_f<T>(wb[(s + i) * rowK + static_cast<int64_t>(hh) * K + kk]) : 0.f;
      kc[i * kRowN + kk] = ok ? to_f<T>(kb[(s + i) * rowKg + static_cast<int64_t>(hk) * K + kk]) : 0.f;
    }
    for (int e = tid; e < 64 * kHCols; e += kGemmThreads) {
      const int i = e / kHCols, c = e % kHCols;
      us[i * kRow32 + c] = i < L && c < vcols ? to_f<T>(ub[(s + i) * rowV + static_cast<int64_t>(hh) * V + v0 + c]) : 0.f;
    }
    if (tid < 64) gs[tid] = p.g && tid < L ? p.g[static_cast<int64_t>(hh) * BT + s + tid] : 0.f;
    __syncthreads();
    const float glast = p.g ? gs[L - 1] : 0.f;
    for (int kk = tid; kk < 128; kk += kGemmThreads)
      dk[kk] = (p.g ? expf(glast) : 1.f) *
               (p.gk && kk < K ? expf(p.gk[(s + L - 1) * rowK + static_cast<int64_t>(hh) * K + kk]) : 1.f);
    // h[c] = S, and the product operand S~
    for (int e = tid; e < 128 * kHCols; e += kGemmThreads) {
      const int kk = e / kHCols, c = e % kHCols;
      const float x = S[kk * kRow32 + c];
      Sr[kk * kRow32 + c] = round_to<T>(x);
      if (hb && kk < K && c < vcols) {
        const int64_t hc = (boh + lc) * p.H + hh;
        const int vv = v0 + c;
        hb[p.state_v_first ? (hc * V + vv) * K + kk : (hc * K + kk) * V + vv] = from_f<T>(x);
      }
    }
    gemm_smem<true>(us, kRow32, 64, kHCols, K, wc, kRowK, 1, Sr, kRow32, 1, -1.f);  // v_new = u - w S~
    for (int e = tid; e < 64 * kHCols; e += kGemmThreads) {
      const int i = e / kHCols, c = e % kHCols;
      const float x = us[i * kRow32 + c];
      if (vnb && i < L && c < vcols) vnb[(s + i) * rowV + static_cast<int64_t>(hh) * V + v0 + c] = from_f<T>(x);
      us[i * kRow32 + c] = i < L ? round_to<T>(p.g ? x * expf(glast - gs[i]) : x) : 0.f;
    }
    for (int e = tid; e < 128 * kHCols; e += kGemmThreads) S[(e / kHCols) * kRow32 + e % kHCols] *= dk[e / kHCols];
    gemm_smem<true>(S, kRow32, K < 64 ? K : 64, kHCols, 64, kc, 1, kRowN, us, kRow32, 1);  // S += k^T v~
    if (K > 64) gemm_smem<true>(S + 64 * kRow32, kRow32, K - 64, kHCols, 64, kc + 64, 1, kRowN, us, kRow32, 1);
  }
  __syncthreads();
  if (p.final_state) {
    for (int e = tid; e < K * kHCols; e += kGemmThreads) {
      const int kk = e / kHCols, c = e % kHCols, vv = v0 + c;
      if (c >= vcols) continue;
      if (p.state_v_first) p.final_state[(nh * V + vv) * K + kk] = S[kk * kRow32 + c];
      else p.final_state[(nh * K + kk) * V + vv] = S[kk * kRow32 + c];
    }
  }
}

template <typename T>
cudaError_t launch_t(const gdn_chunk_h_args& a, cudaStream_t s) {
  const size_t smem = (2 * 128 * kRow32 + 64 * kRowK + 64 * kRowN + 64 * kRow32 + 64 + 128 + 32) * sizeof(float);
  auto kern = chunk_h_stage_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  note_launch();
  kern<<<dim3(static_cast<unsigned>(a.N), a.H, (a.V + kHCols - 1) / kHCols), kGemmThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_chunk_h_stage(const gdn_chunk_h_args& a, cudaStream_t s) {
  switch (a.dtype) {
    case GDN_F32: return launch_t<float>(a, s);
    case GDN_BF16: return launch_t<__nv_bfloat16>(a, s);
    case GDN_F16: return launch_t<__half>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
