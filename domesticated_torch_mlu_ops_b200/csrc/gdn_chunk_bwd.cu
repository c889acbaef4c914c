// Backward of the chunked gated delta-rule forward: the autograd backward of
// chunk_gated_delta_rule (triton/fla/chunk.py:188-251 ChunkGatedDeltaRuleFunction,
// stages at chunk.py:76-186: recompute w, u, h; chunk_bwd_dv_local;
// chunk_gated_delta_rule_bwd_dhu; chunk_bwd_dqkwg; prepare_wy_repr_bwd;
// reverse chunk-local cumsum of dg).
//
// fp32 SIMT kernels over the fp32 intermediates that the generic forward
// leaves in the workspace (chunk-local cumsum G, normalised q/k, W, U, v_new
// and the state h at every chunk start).  Per chunk of L <= 64 tokens and
// v-head, with Gam_i = exp(G_i), gam = Gam_{L-1}, D_ij = exp(G_i - G_j),
// c_i = gam / Gam_i, S = Q K^T, M = causal mask (j <= i):
//   A = tril_strict(diag(b) D * K K^T), T = (I + A)^-1
//   W = T diag(b Gam) K, U = T diag(b) V, v = U - W h
//   o = scale (diag(Gam) Q h + (M * D * S) v),  h' = gam h + K^T diag(c) v
// Given dO and dh' (the gradient of the state after the chunk):
//   bwd_dvlocal_kernel (per chunk and v-head): dv_local = scale (M * D * S)^T dO
//   bwd_state_kernel (reverse over a sequence's chunks):
//     dv = dv_local + diag(c) K dh'
//     dh = gam dh' + scale Q^T diag(Gam) dO - W^T dv          (dh0 at the first chunk)
//   bwd_dqkw_kernel (per chunk and v-head):
//     dP = scale M * D * (dO v^T)
//     dQ = scale diag(Gam) dO h^T + dP K,  dK = dP^T Q + diag(c) v dh'^T,  dW = -dv h^T
//   bwd_wy_kernel (per chunk and v-head):
//     dR_w = T^T dW, dR_u = T^T dv, dT = dW R_w^T + dv R_u^T (R_w = diag(b Gam) K,
//     R_u = diag(b) V), dA = -T^T dT T^T on the strictly lower triangle,
//     dK += diag(b Gam) dR_w + (dS + dS^T) K with dS = diag(b) D * dA, dV = diag(b) dR_u
//   dG collects every use of G (through Gam, gam, c, D) and db every use of b;
//   bwd_qk_kernel sums dq, dk over the v-heads of each q/k head (then the L2
//   norm backward when the forward normalised q, k); bwd_dg_kernel turns dG
//   into dg by a reverse cumsum within each chunk (G is a forward cumsum of g).

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_chunk_tc.cuh"
#include "tile_gemm.cuh"
#include "solve_tril.cuh"

namespace gdn {
namespace {

constexpr int kT = kGemmThreads;  // threads per CTA
constexpr int LD = kRowK;         // row stride of 64 x 128 fp32 tiles
constexpr int LQ = 130;           // the same in bwd_dqkw_kernel (six tiles must fit)
constexpr int kP = 65;            // row stride of 64 x 64 fp32 tiles
constexpr int kStage = kGemmStage;
constexpr int kVS = 32;           // V columns per bwd_state_kernel CTA

template <bool ACC, bool SPLIT = true, typename TA, typename TB>
__device__ __forceinline__ void gemm(float* C, int64_t ldc, int mc, int N, int Kd, const TA* a, int64_t asi,
                                     int64_t ask, int ma, const TB* b, int64_t bsk, int64_t bsn, int nb,
                                     float alpha, float* st) {
  gemm_staged<ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
}

struct BwdPtrs {
  const int64_t* coff;                        // chunk offsets [N + 1]
  const float *gc, *qn, *kn, *w, *vnew, *hs;  // forward intermediates
  float *dvn, *dhn, *dqh, *dkh, *dw, *dG;     // backward intermediates
};

// dv_local = scale (M * D * Q K^T)^T dO for one (chunk, v-head): the part of
// dv that does not depend on the state gradient (chunk_bwd_dv_local), into
// the dv workspace, which bwd_state_kernel then completes.  dO takes Q's
// tile once Q K^T is done, so two CTAs fit on an SM and one's loads overlap
// the other's products.
template <typename T>
__global__ void __launch_bounds__(kT, 2) bwd_dvlocal_kernel(const gdn_chunk_bwd_args p, const BwdPtrs w, float scale) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* qc = sm;             // [64][LD]; dO after Q K^T
  float* kc = qc + 64 * LD;   // [64][LD]
  float* P = kc + 64 * LD;    // [64][kP]
  float* gcs = P + 64 * kP;   // [64]
  float* dO = qc;
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int tid = threadIdx.x;
  const int64_t rowQ = static_cast<int64_t>(p.H) * K, rowV = static_cast<int64_t>(p.HV) * V;
  const T* dout = static_cast<const T*>(p.dout) + s * rowV + static_cast<int64_t>(hv) * V;
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      const bool ok = i < L;
      qc[i * LD + kk] = ok ? w.qn[(s + i) * rowQ + h * K + kk] : 0.f;
      kc[i * LD + kk] = ok ? w.kn[(s + i) * rowQ + h * K + kk] : 0.f;
    }
  }
  if (tid < 64) gcs[tid] = tid < L ? w.gc[(s + tid) * p.HV + hv] : 0.f;
  gemm_smem<false, kSplit<T>>(P, kP, 64, 64, K, qc, LD, 1, kc, 1, LD);  // Q K^T (ends with a barrier)
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      dO[i * LD + vv] = i < L ? to_f<T>(dout[i * rowV + vv]) : 0.f;
    }
  }
  for (int e = tid; e < 64 * 64; e += kT) {
    const int i = e >> 6, j = e & 63;
    P[i * kP + j] = (i < L && j <= i) ? P[i * kP + j] * expf(gcs[i] - gcs[j]) : 0.f;
  }
  gemm_smem<false, kSplit<T>>(w.dvn + s * rowV + static_cast<int64_t>(hv) * V, rowV, L, V, 64, P, 1, kP, dO, LD, 1, scale);
}

// Shared memory of bwd_state_kernel: [Q; W] (128 rows, read transposed), K
// (read row-major), the dv_local slice, G (2 stages), dh and the stacked
// right-hand side (32-column tiles read n-contiguous).
constexpr int kSqw = 128 * kRowN;
constexpr int kSk = 64 * kRowK;
constexpr int kSvec = 64 * kRow32 + 2 * 64;

// Reverse recurrence over one sequence's chunks for one (v-head, 32-column
// slice of V).  Per chunk, given dh' (gradient of the state after it):
//   dv = dv_local + diag(c) K dh'                      (stored: dv of v_new)
//   dh = gam dh' + [Q; W]^T [scale diag(Gam) dO; -dv]  (one stacked product)
// dh' is stored per chunk for the parallel kernels; dh0 at the end.  The
// [Q; W] tiles of a chunk are copied in during its dv step and the next
// chunk's K, dv_local and G during its dh step.
template <typename T>
__global__ void __launch_bounds__(kT, 1) bwd_state_kernel(const gdn_chunk_bwd_args p, const BwdPtrs w, float scale) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* qw = sm;                   // [128][kRowN]: Q rows 0..63, W rows 64..127
  float* kc = qw + kSqw;            // [64][kRowK]
  float* dvl = kc + kSk;            // [64][kRow32] dv_local slice
  float* gsb = dvl + 64 * kRow32;   // [2][64] G per stage
  float* dh = gsb + 2 * 64;         // [128][kRow32]
  float* rhs = dh + 128 * kRow32;   // [128][kRow32]: scale Gam dO rows 0..63, -dv rows 64..127
  const int64_t n = blockIdx.x;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  const int v0 = blockIdx.z * kVS;
  const int vcols = V - v0 < kVS ? V - v0 : kVS;
  const int tid = threadIdx.x;
  const int64_t rowQ = static_cast<int64_t>(p.H) * K, rowV = static_cast<int64_t>(p.HV) * V,
                rowK = static_cast<int64_t>(p.HV) * K;
  const T* dout = static_cast<const T*>(p.dout);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  for (int e = tid; e < 128 * kVS; e += kT) {
    const int kk = e / kVS, c = e % kVS, vv = v0 + c;
    float x = 0.f;
    if (p.dht && vv < V && kk < K)
      x = p.state_v_first ? p.dht[((n * p.HV + hv) * V + vv) * K + kk] : p.dht[((n * p.HV + hv) * K + kk) * V + vv];
    dh[kk * kRow32 + c] = x;
  }
  const int64_t nch = eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0;
  auto chunk_len = [&](int64_t lc) { return static_cast<int>(min64(kChunk, eos - (bos + lc * kChunk))); };
  auto issue_k = [&](int64_t lc) {  // K, dv_local slice, G of chunk lc
    const int64_t s = bos + lc * kChunk;
    const int L = chunk_len(lc);
    tile_async(kc, kRowK, w.kn + s * rowQ + h * K, rowQ, L, 64, K, K);
    tile_async(dvl, kRow32, w.dvn + s * rowV + static_cast<int64_t>(hv) * V + v0, rowV, L, 64, vcols, kVS);
    if (tid < 64) cp_async4(gsb + (lc & 1) * 64 + tid, tid < L ? w.gc + (s + tid) * p.HV + hv : w.gc, tid < L);
    cp_async_commit();
  };
  auto issue_qw = [&](int64_t lc) {  // Q and W of chunk lc
    const int64_t s = bos + lc * kChunk;
    const int L = chunk_len(lc);
    tile_async(qw, kRowN, w.qn + s * rowQ + h * K, rowQ, L, 64, K, K);
    tile_async(qw + 64 * kRowN, kRowN, w.w + s * rowK + static_cast<int64_t>(hv) * K, rowK, L, 64, K, K);
    cp_async_commit();
  };
  if (nch > 0) issue_k(nch - 1);
  for (int64_t lc = nch - 1; lc >= 0; --lc) {
    const int64_t s = bos + lc * kChunk;
    const int L = chunk_len(lc);
    const int64_t cidx = w.coff[n] + lc;
    const float* gs = gsb + (lc & 1) * 64;
    // ---- dv step: needs K, dv_local, G of this chunk
    issue_qw(lc);  // [Q; W] was last read by the previous dh step, which ended with a barrier
    cp_async_wait<1>();
    __syncthreads();
    float* dhn = w.dhn + (cidx * p.HV + hv) * static_cast<int64_t>(K) * V;
    for (int e = tid; e < K * kVS; e += kT) {
      const int kk = e / kVS, c = e % kVS;
      if (c < vcols) dhn[kk * V + v0 + c] = dh[kk * kRow32 + c];
    }
    const float glast = gs[L - 1], eg = expf(glast);
    for (int e = tid; e < 64 * kVS; e += kT) {
      const int i = e / kVS, c = e % kVS;
      const float d = (i < L && c < vcols) ? to_f<T>(dout[(s + i) * rowV + static_cast<int64_t>(hv) * V + v0 + c]) : 0.f;
      rhs[i * kRow32 + c] = i < L ? scale * expf(gs[i]) * d : 0.f;
    }
    gemm_smem<false, kSplit<T>>(rhs + 64 * kRow32, kRow32, 64, kVS, K, kc, kRowK, 1, dh, kRow32, 1);  // K dh'
    for (int e = tid; e < 64 * kVS; e += kT) {
      const int i = e / kVS, c = e % kVS;
      float x = 0.f;
      if (i < L) x = dvl[i * kRow32 + c] + expf(glast - gs[i]) * rhs[(64 + i) * kRow32 + c];
      if (i < L && c < vcols) w.dvn[(s + i) * rowV + static_cast<int64_t>(hv) * V + v0 + c] = x;
      rhs[(64 + i) * kRow32 + c] = -x;
    }
    // ---- dh step: needs [Q; W]; K, dv_local of the next chunk come in meanwhile
    __syncthreads();  // K and dv_local of this chunk are no longer read
    if (lc > 0) {
      issue_k(lc - 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    for (int e = tid; e < 128 * kVS; e += kT) dh[(e / kVS) * kRow32 + e % kVS] *= eg;
    gemm_smem<true, kSplit<T>>(dh, kRow32, min(K, 64), kVS, 128, qw, 1, kRowN, rhs, kRow32, 1);
    if (K > 64) gemm_smem<true, kSplit<T>>(dh + 64 * kRow32, kRow32, K - 64, kVS, 128, qw + 64, 1, kRowN, rhs, kRow32, 1);
  }
  __syncthreads();
  if (p.dh0) {
    for (int e = tid; e < K * kVS; e += kT) {
      const int kk = e / kVS, c = e % kVS, vv = v0 + c;
      if (c >= vcols) continue;
      if (p.state_v_first) p.dh0[((n * p.HV + hv) * V + vv) * K + kk] = dh[kk * kRow32 + c];
      else p.dh0[((n * p.HV + hv) * K + kk) * V + vv] = dh[kk * kRow32 + c];
    }
  }
}

// dq, dk (per v-head, fp32), dW and the dG terms of the output and state
// paths for one (chunk, v-head).  With dq, dk complete for these paths,
// dG_i = q_i . dq_i - k_i . dk_i, plus gam <dh', h> + sum_i E_i on the last row
// (E_i = k_i . (diag(c) v dh'^T)_i): the Q K^T products of the P path cancel
// into the two row dots.
template <typename T>
__global__ void __launch_bounds__(kT, 1) bwd_dqkw_kernel(const gdn_chunk_bwd_args p, const BwdPtrs w, float scale) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* qc = sm;               // [64][LQ]
  float* kc = qc + 64 * LQ;     // [64][LQ]
  float* dOs = kc + 64 * LQ;    // [64][LQ] dO
  float* X = dOs + 64 * LQ;     // [64][LQ] v_new, then dv
  float* dq = X + 64 * LQ;      // [64][LQ]
  float* dk = dq + 64 * LQ;     // [64][LQ]
  float* dP = dk + 64 * LQ;     // [64][kP]
  float* gcs = dP + 64 * kP;    // [64]
  float* red = gcs + 64;        // [32]
  float* st = red + 32;         // gemm staging
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t cidx = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t rowQ = static_cast<int64_t>(p.H) * K, rowV = static_cast<int64_t>(p.HV) * V,
                rowK = static_cast<int64_t>(p.HV) * K;
  const float* hst = w.hs + (cidx * p.HV + hv) * static_cast<int64_t>(K) * V;   // h [K][V]
  const float* dhn = w.dhn + (cidx * p.HV + hv) * static_cast<int64_t>(K) * V;  // dh' [K][V]
  const float* vn = w.vnew + s * rowV + static_cast<int64_t>(hv) * V;          // rows, stride rowV
  const float* dvn = w.dvn + s * rowV + static_cast<int64_t>(hv) * V;
  const T* dO = static_cast<const T*>(p.dout) + s * rowV + static_cast<int64_t>(hv) * V;
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      const bool ok = i < L;
      qc[i * LQ + kk] = ok ? w.qn[(s + i) * rowQ + h * K + kk] : 0.f;
      kc[i * LQ + kk] = ok ? w.kn[(s + i) * rowQ + h * K + kk] : 0.f;
    }
  }
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      const bool ok = i < L;
      dOs[i * LQ + vv] = ok ? to_f<T>(dO[i * rowV + vv]) : 0.f;
      X[i * LQ + vv] = ok ? vn[i * rowV + vv] : 0.f;
    }
  }
  if (tid < 64) gcs[tid] = tid < L ? w.gc[(s + tid) * p.HV + hv] : 0.f;
  gemm_smem<false, kSplit<T>>(dP, kP, 64, 64, V, dOs, LQ, 1, X, 1, LQ);  // dO v^T
  for (int e = tid; e < 64 * 64; e += kT) {
    const int i = e >> 6, j = e & 63;
    dP[i * kP + j] = (i < L && j <= i) ? scale * expf(gcs[i] - gcs[j]) * dP[i * kP + j] : 0.f;
  }
  gemm<false, kSplit<T>>(dk, LQ, 64, K, V, X, LQ, 1, 64, dhn, 1, V, K, 1.f, st);  // v dh'^T
  const float glast = gcs[L - 1], eg = expf(glast);
  float E = 0.f;
  if (tid < 64) {  // dK = diag(c) v dh'^T; E_i = k_i . dK_i
    const float c = tid < L ? expf(glast - gcs[tid]) : 0.f;
    for (int kk = 0; kk < K; ++kk) {
      const float x = c * dk[tid * LQ + kk];
      dk[tid * LQ + kk] = x;
      E = fmaf(kc[tid * LQ + kk], x, E);
    }
  }
  float part = 0.f;
  for (int e = tid; e < K * V; e += kT) part = fmaf(dhn[e], hst[e], part);
  const float hh = block_sum(part, red);  // <dh', h>
  const float Esum = block_sum(tid < 64 ? E : 0.f, red);
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {  // X <- dv
    for (int vv = tid & 31; vv < V; vv += 32) {
      X[i * LQ + vv] = i < L ? dvn[i * rowV + vv] : 0.f;
    }
  }
  gemm<false, kSplit<T>>(dq, LQ, 64, K, V, dOs, LQ, 1, 64, hst, 1, V, K, scale, st);  // scale dO h^T
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      dq[i * LQ + kk] *= i < L ? expf(gcs[i]) : 0.f;
    }
  }
  gemm_smem<true, kSplit<T>>(dq, LQ, 64, K, 64, dP, kP, 1, kc, LQ, 1);  // + dP K
  gemm_smem<true, kSplit<T>>(dk, LQ, 64, K, 64, dP, 1, kP, qc, LQ, 1);  // + dP^T Q
  // dW = -dv h^T straight to the workspace
  gemm<false, kSplit<T>>(w.dw + s * rowK + static_cast<int64_t>(hv) * K, rowK, L, K, V, X, LQ, 1, 64, hst, 1, V, K, -1.f,
              st);
  if (tid < 64) {
    float a = 0.f;
    for (int kk = 0; kk < K; ++kk) a += qc[tid * LQ + kk] * dq[tid * LQ + kk] - kc[tid * LQ + kk] * dk[tid * LQ + kk];
    if (tid == L - 1) a += eg * hh + Esum;
    if (tid < L) w.dG[(s + tid) * p.HV + hv] = a;
  }
  for (int i = tid >> 5; i < L; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      w.dqh[(s + i) * rowK + static_cast<int64_t>(hv) * K + kk] = dq[i * LQ + kk];
      w.dkh[(s + i) * rowK + static_cast<int64_t>(hv) * K + kk] = dk[i * LQ + kk];
    }
  }
}

// Backward through W = T diag(b Gam) K and U = T diag(b) V for one
// (chunk, v-head): dv, db, and the dK and dG terms of the WY form.
template <typename T>
__global__ void __launch_bounds__(kT, 1) bwd_wy_kernel(const gdn_chunk_bwd_args p, const BwdPtrs w) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* Tm = sm;                 // [64][kTS] (16-byte aligned)
  float* Zs = Tm + 64 * kTS;      // solve scratch (16-byte aligned)
  float* kc = Zs + kTrilScratch;  // [64][LD]
  float* b1 = kc + 64 * LD;       // [64][LD] dW, then dR_u
  float* b2 = b1 + 64 * LD;       // [64][LD] dR_w, then dK
  float* Sk = b2 + 64 * LD;       // [64][kP] K K^T
  float* Am = Sk + 64 * kP;       // [64][kP] A, then dS
  float* dT = Am + 64 * kP;       // [64][kP] dT, then dA
  float* tm = dT + 64 * kP;       // [64][kP]
  float* gcs = tm + 64 * kP;      // [64]
  float* bs = gcs + 64;           // [64] beta
  float* cw = bs + 64;            // [64] beta Gam
  float* db = cw + 64;            // [64]
  float* dG = db + 64;            // [64]
  float* st = dG + 64;            // gemm staging
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int tid = threadIdx.x;
  const int64_t rowQ = static_cast<int64_t>(p.H) * K, rowV = static_cast<int64_t>(p.HV) * V,
                rowK = static_cast<int64_t>(p.HV) * K;
  const T* vin = static_cast<const T*>(p.v) + s * rowV + static_cast<int64_t>(hv) * V;
  const float* dvn = w.dvn + s * rowV + static_cast<int64_t>(hv) * V;
  const float* dwp = w.dw + s * rowK + static_cast<int64_t>(hv) * K;
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      const bool ok = i < L;
      kc[i * LD + kk] = ok ? w.kn[(s + i) * rowQ + h * K + kk] : 0.f;
      b1[i * LD + kk] = ok ? dwp[i * rowK + kk] : 0.f;
    }
  }
  if (tid < 64) {
    const bool ok = tid < L;
    const float g = ok ? w.gc[(s + tid) * p.HV + hv] : 0.f;
    const float bt = ok ? p.beta[(s + tid) * p.HV + hv] : 0.f;
    gcs[tid] = g;
    bs[tid] = bt;
    cw[tid] = ok ? bt * expf(g) : 0.f;
  }
  gemm_smem<false, kSplit<T>>(Sk, kP, 64, 64, K, kc, LD, 1, kc, 1, LD);  // K K^T
  for (int e = tid; e < 64 * 64; e += kT) {
    const int i = e >> 6, j = e & 63;
    Am[i * kP + j] = (i < L && j < i) ? bs[i] * expf(gcs[i] - gcs[j]) * Sk[i * kP + j] : 0.f;
  }
  __syncthreads();
  solve_tril64_nt<kT>(Am, Tm, Zs);  // T = (I + A)^-1
  gemm_smem<false, kSplit<T>>(dT, kP, 64, 64, K, b1, LD, 1, kc, 1, LD);     // dW K^T
  gemm<false, kSplit<T>>(tm, kP, 64, 64, V, dvn, rowV, 1, L, vin, 1, rowV, L, 1.f, st);  // dv V^T
  for (int e = tid; e < 64 * 64; e += kT) {
    const int i = e >> 6, j = e & 63;
    dT[i * kP + j] = dT[i * kP + j] * cw[j] + tm[i * kP + j] * bs[j];
  }
  gemm_smem<false, kSplit<T>>(b2, LD, 64, K, 64, Tm, 1, kTS, b1, LD, 1);     // dR_w = T^T dW
  gemm<false, kSplit<T>>(b1, LD, 64, V, L, Tm, 1, kTS, 64, dvn, rowV, 1, V, 1.f, st);   // dR_u = T^T dv
  gemm_smem<false, kSplit<T>>(tm, kP, 64, 64, 64, dT, kP, 1, Tm, 1, kTS);   // dT T^T
  gemm_smem<false, kSplit<T>>(dT, kP, 64, 64, 64, Tm, 1, kTS, tm, kP, 1, -1.f);  // dA = -T^T (dT T^T)
  T* dv = static_cast<T*>(p.dv) + s * rowV + static_cast<int64_t>(hv) * V;
  for (int i = tid >> 5; i < L; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      dv[i * rowV + vv] = from_f<T>(bs[i] * b1[i * LD + vv]);
    }
  }
  if (tid < 64) {
    const int i = tid;
    float dbi = 0.f, dgi = 0.f;
    if (i < L) {
      float a = 0.f;  // U path: V_i . dR_u_i
      for (int vv = 0; vv < V; ++vv) a = fmaf(to_f<T>(vin[i * rowV + vv]), b1[i * LD + vv], a);
      float r = 0.f;  // W path: K_i . dR_w_i
      for (int kk = 0; kk < K; ++kk) r = fmaf(kc[i * LD + kk], b2[i * LD + kk], r);
      dbi = a + expf(gcs[i]) * r;
      dgi = cw[i] * r;
      float t = 0.f;  // A path: sum_j dA_ij D_ij S_ij
      for (int j = 0; j < i; ++j) t += dT[i * kP + j] * expf(gcs[i] - gcs[j]) * Sk[i * kP + j];
      dbi += t;
    }
    db[i] = dbi;
    dG[i] = dgi;
  }
  __syncthreads();
  for (int e = tid; e < 64 * 64; e += kT) {  // dS = diag(b) D * dA (strictly lower, rows < L)
    const int i = e >> 6, j = e & 63;
    Am[i * kP + j] = (i < L && j < i) ? bs[i] * expf(gcs[i] - gcs[j]) * dT[i * kP + j] : 0.f;
  }
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {  // dK = diag(b Gam) dR_w
    for (int kk = tid & 31; kk < K; kk += 32) {
      b2[i * LD + kk] *= cw[i];
    }
  }
  __syncthreads();
  if (tid < 64) {  // D path of A: F = dS * S; dG_i += sum_j F_ij - sum_j F_ji
    float f = 0.f;
    for (int j = 0; j < 64; ++j) f += Am[tid * kP + j] * Sk[tid * kP + j] - Am[j * kP + tid] * Sk[j * kP + tid];
    dG[tid] += f;
  }
  gemm_smem<true, kSplit<T>>(b2, LD, 64, K, 64, Am, kP, 1, kc, LD, 1);  // + dS K
  gemm_smem<true, kSplit<T>>(b2, LD, 64, K, 64, Am, 1, kP, kc, LD, 1);  // + dS^T K
  for (int i = tid >> 5; i < L; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      w.dkh[(s + i) * rowK + static_cast<int64_t>(hv) * K + kk] += b2[i * LD + kk];
    }
  }
  if (tid < L) {
    p.dbeta[(s + tid) * p.HV + hv] = db[tid];
    w.dG[(s + tid) * p.HV + hv] += dG[tid];
  }
}

// One warp per (token, q/k head): dq and dk summed over the head's v-heads
// in a fixed order, then the L2-norm backward dx = r (dy - y (y . dy)) with
// y = x r, r = 1 / sqrt(sum(x^2) + 1e-6) when the forward normalised q, k.
template <typename T>
__global__ void bwd_qk_kernel(const gdn_chunk_bwd_args p, const float* __restrict__ dqh,
                              const float* __restrict__ dkh, int64_t rows) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int K = p.K, G = p.HV / p.H;
  const int64_t t = row / p.H;
  const int hh = static_cast<int>(row % p.H);
  const uintptr_t al = reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
                       reinterpret_cast<uintptr_t>(p.dq) | reinterpret_cast<uintptr_t>(p.dk);
  if (K == 128 && (al & 15) == 0) {
    // four consecutive columns per lane, every load issued before the first use
    const int64_t src0 = (t * p.HV + static_cast<int64_t>(hh) * G) * K + lane * 4;
    float4 dy[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int j = 0; j < G; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(dqh + src0 + static_cast<int64_t>(j) * K);
      const float4 b = *reinterpret_cast<const float4*>(dkh + src0 + static_cast<int64_t>(j) * K);
      dy[0].x += a.x; dy[0].y += a.y; dy[0].z += a.z; dy[0].w += a.w;
      dy[1].x += b.x; dy[1].y += b.y; dy[1].z += b.z; dy[1].w += b.w;
    }
    const float4 xv[2] = {load4<T>(static_cast<const T*>(p.q) + row * K + lane * 4),
                          load4<T>(static_cast<const T*>(p.k) + row * K + lane * 4)};
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      float4 d = dy[which];
      const float4 x = xv[which];
      if (p.use_qk_l2norm) {
        const float ss = group_sum<32>(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
        const float r = 1.f / sqrtf(ss + 1e-6f);
        const float dot = group_sum<32>(r * (x.x * d.x + x.y * d.y + x.z * d.z + x.w * d.w));
        d = make_float4(r * (d.x - x.x * r * dot), r * (d.y - x.y * r * dot), r * (d.z - x.z * r * dot),
                        r * (d.w - x.w * r * dot));
      }
      T* out = static_cast<T*>(which ? p.dk : p.dq) + row * K + lane * 4;
      out[0] = from_f<T>(d.x);
      out[1] = from_f<T>(d.y);
      out[2] = from_f<T>(d.z);
      out[3] = from_f<T>(d.w);
    }
    return;
  }
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const float* src = which ? dkh : dqh;
    const T* x = static_cast<const T*>(which ? p.k : p.q) + row * K;
    T* out = static_cast<T*>(which ? p.dk : p.dq) + row * K;
    float dy[4], xv[4];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = lane + 32 * u;
      float a = 0.f, xx = 0.f;
      if (kk < K) {
        for (int j = 0; j < G; ++j) a += src[(t * p.HV + hh * G + j) * K + kk];
        xx = to_f<T>(x[kk]);
      }
      dy[u] = a;
      xv[u] = xx;
      ss = fmaf(xx, xx, ss);
    }
    if (p.use_qk_l2norm) {
      ss = group_sum<32>(ss);
      const float r = 1.f / sqrtf(ss + 1e-6f);
      float dot = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) dot = fmaf(xv[u] * r, dy[u], dot);
      dot = group_sum<32>(dot);
#pragma unroll
      for (int u = 0; u < 4; ++u) dy[u] = r * (dy[u] - xv[u] * r * dot);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int kk = lane + 32 * u;
      if (kk < K) out[kk] = from_f<T>(dy[u]);
    }
  }
}

// dg = reverse cumsum of dG within each chunk; one thread per (chunk, v-head).
__global__ void bwd_dg_kernel(const gdn_chunk_bwd_args p, const int64_t* __restrict__ coff,
                              const float* __restrict__ dG) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nchunks = coff[p.N];
  if (e >= nchunks * p.HV) return;
  const int64_t c = e / p.HV;
  const int hv = static_cast<int>(e % p.HV);
  int64_t n, lc;
  if (!locate_chunk(coff, p.N, c, n, lc)) return;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  float acc = 0.f;
  for (int i = L - 1; i >= 0; --i) {
    acc += dG[(s + i) * p.HV + hv];
    p.dg[(s + i) * p.HV + hv] = acc;
  }
}

constexpr size_t kDvlSmem = sizeof(float) * (2 * 64 * LD + 64 * kP + 64);
static_assert(2 * (kDvlSmem + 1024) <= 228 * 1024, "two bwd_dvlocal_kernel CTAs per SM");
constexpr size_t kStateSmem = sizeof(float) * (kSqw + kSk + kSvec + 2 * 128 * kRow32);
constexpr size_t kDqkwSmem = sizeof(float) * (6 * 64 * LQ + 64 * kP + 64 + 32 + kStage);
static_assert(kDqkwSmem <= 227 * 1024, "bwd_dqkw_kernel shared memory");
constexpr size_t kWySmem =
    sizeof(float) * (64 * kTS + kTrilScratch + 3 * 64 * LD + 4 * 64 * kP + 5 * 64 + kStage);
static_assert(kWySmem <= 227 * 1024, "bwd_wy_kernel shared memory");
static_assert((64 * kTS) % 4 == 0, "solve scratch must stay 16-byte aligned");

gdn_chunk_args forward_args(const gdn_chunk_bwd_args& b) {
  gdn_chunk_args a{};
  a.q = b.q;
  a.k = b.k;
  a.v = b.v;
  a.g = b.g;
  a.beta = b.beta;
  a.initial_state = b.initial_state;
  a.cu_seqlens = b.cu_seqlens;
  a.workspace = b.workspace;
  a.workspace_bytes = b.workspace_bytes;
  a.B = b.B;
  a.T = b.T;
  a.N = b.N;
  a.H = b.H;
  a.HV = b.HV;
  a.K = b.K;
  a.V = b.V;
  a.qkv_dtype = b.qkv_dtype;
  a.cu_dtype = b.cu_dtype;
  a.scale = b.scale;
  a.use_qk_l2norm = b.use_qk_l2norm;
  a.state_v_first = b.state_v_first;
  a.force_generic = 1;
  return a;
}

// bf16/fp16 with K = V = 128: the state-gradient recurrence runs on tcgen05
// (gdn_chunk_bwd_tc.cu) from the forward WY kernel's images.
bool bwd_tc_applies(const gdn_chunk_bwd_args& b) {
  return (b.qkv_dtype == GDN_BF16 || b.qkv_dtype == GDN_F16) && b.K == 128 && b.V == 128 &&
         b.B * b.T < (int64_t(1) << 31);
}

template <typename T>
cudaError_t run_bwd(const gdn_chunk_bwd_args& b, const BwdWorkspace& ws, cudaStream_t s) {
  const gdn_chunk_args a = forward_args(b);
  const bool tcb = bwd_tc_applies(b);
  // with the tensor-core path, the states and v_new come from the forward's
  // own kernels (tcgen05, bf16 roundings as in the forward); otherwise from
  // the generic fp32 recompute
  cudaError_t e = cudaSuccess;
  // the tensor-core kernels need none of the generic recompute's outputs (they
  // take q, k raw and compute the L2 norms themselves)
  if (!tcb && (e = launch_chunk_generic_recompute(a, ws.fwd, s)) != cudaSuccess) return e;
  char* base = static_cast<char*>(b.workspace);
  tc::Work tw{};
  if (tcb) {  // G from the tensor-core WY kernel; W and U of the generic one are not needed
    gdn_chunk_args fa = a;
    fa.force_generic = 0;
    if ((e = tc::launch_wy_only(fa, base + ws.tc, s, tw, reinterpret_cast<float*>(base + ws.fwd.gc))) !=
        cudaSuccess)
      return e;
    if ((e = tc::launch_state_store(fa, tw, reinterpret_cast<uint8_t*>(base + ws.himg),
                                    reinterpret_cast<uint8_t*>(base + ws.vnimg), s)) != cudaSuccess)
      return e;
  }
  BwdPtrs w;
  w.coff = tcb ? tw.coff : reinterpret_cast<const int64_t*>(base + ws.fwd.chunk_offsets);
  w.gc = reinterpret_cast<const float*>(base + ws.fwd.gc);
  w.qn = reinterpret_cast<const float*>(base + ws.fwd.qn);
  w.kn = reinterpret_cast<const float*>(base + ws.fwd.kn);
  w.w = reinterpret_cast<const float*>(base + ws.fwd.w);
  w.vnew = reinterpret_cast<const float*>(base + ws.fwd.vnew);
  w.hs = reinterpret_cast<const float*>(base + ws.fwd.hs);
  w.dvn = reinterpret_cast<float*>(base + ws.dvn);
  w.dhn = reinterpret_cast<float*>(base + ws.dhn);
  w.dqh = reinterpret_cast<float*>(base + ws.dqh);
  w.dkh = reinterpret_cast<float*>(base + ws.dkh);
  w.dw = reinterpret_cast<float*>(base + ws.dw);
  w.dG = reinterpret_cast<float*>(base + ws.dG);
  const int64_t Ttot = b.B * b.T;
  const int64_t nc = chunk_upper_bound(Ttot, b.N);
  const float scale = b.scale > 0.f ? b.scale : 1.f / sqrtf(static_cast<float>(b.K));
  if ((e = cudaFuncSetAttribute(bwd_dvlocal_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kDvlSmem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(bwd_state_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kStateSmem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(bwd_dqkw_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kDqkwSmem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(bwd_wy_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kWySmem))) != cudaSuccess) return e;
  if (nc > 0 && tcb) {
    if ((e = tc::launch_bwd_dvlocal_tc(b, tw, w.dvn, s)) != cudaSuccess) return e;
  } else if (nc > 0) {
    note_launch();
    bwd_dvlocal_kernel<T><<<dim3(static_cast<unsigned>(nc), b.HV), kT, kDvlSmem, s>>>(b, w, scale);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (tcb) {
    if ((e = tc::launch_bwd_state_tc(b, tw, w.dvn, reinterpret_cast<uint8_t*>(base + ws.dvimg),
                                     reinterpret_cast<uint8_t*>(base + ws.dhimg), s)) != cudaSuccess)
      return e;
  } else {
    note_launch();
    bwd_state_kernel<T><<<dim3(static_cast<unsigned>(b.N), b.HV, (b.V + kVS - 1) / kVS), kT, kStateSmem, s>>>(
        b, w, scale);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (nc > 0) {
    if (tcb) {
      const uint8_t* dvimg = reinterpret_cast<const uint8_t*>(base + ws.dvimg);
      uint8_t* dwimg = reinterpret_cast<uint8_t*>(base + ws.dwimg);
      tc::DqkwOut d{dvimg, w.gc, reinterpret_cast<const uint8_t*>(base + ws.himg),
                    reinterpret_cast<const uint8_t*>(base + ws.dhimg), reinterpret_cast<const uint8_t*>(base + ws.vnimg),
                    w.dqh, w.dkh, dwimg, w.dG};
      if ((e = tc::launch_bwd_dqkw_tc(b, tw, d, s)) != cudaSuccess) return e;
      if ((e = tc::launch_bwd_wy_tc(b, tw, tc::WyOut{dvimg, w.gc, dwimg, w.dkh, w.dG}, s)) != cudaSuccess) return e;
    } else {
      note_launch(2);
      bwd_dqkw_kernel<T><<<dim3(static_cast<unsigned>(nc), b.HV), kT, kDqkwSmem, s>>>(b, w, scale);
      bwd_wy_kernel<T><<<dim3(static_cast<unsigned>(nc), b.HV), kT, kWySmem, s>>>(b, w);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  }
  const int64_t rows = Ttot * b.H;
  if (rows > 0) {
    note_launch(2);
    bwd_qk_kernel<T><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(b, w.dqh, w.dkh, rows);
    const int64_t ng = nc * b.HV;
    bwd_dg_kernel<<<static_cast<unsigned>((ng + 255) / 256), 256, 0, s>>>(b, w.coff, w.dG);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

BwdWorkspace plan_bwd_workspace(const gdn_chunk_bwd_args& b) {
  auto al = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  BwdWorkspace w{};
  const int64_t Ttot = b.B * b.T;
  const int64_t nc = chunk_upper_bound(Ttot, b.N);
  const bool tcb = bwd_tc_applies(b);
  if (tcb) {  // the tensor-core path keeps only G of the forward's intermediates
    ChunkWorkspace f{};
    size_t o = 0;
    f.err = o; o += al(16);
    f.chunk_offsets = o; o += al(sizeof(int64_t) * (b.N + 1));
    f.gc = o; o += al(sizeof(float) * Ttot * b.HV);
    f.qn = f.kn = f.w = f.u = f.vnew = f.hs = o;
    f.total = o;
    w.fwd = f;
  } else {
    w.fwd = plan_generic_workspace(forward_args(b));
  }
  size_t o = w.fwd.total;
  w.dvn = o; o += al(sizeof(float) * Ttot * b.HV * b.V);
  w.dhn = o; o += tcb ? 0 : al(sizeof(float) * nc * b.HV * b.K * b.V);  // the tensor-core path keeps dh' as images
  w.dqh = o; o += al(sizeof(float) * Ttot * b.HV * b.K);
  w.dkh = o; o += al(sizeof(float) * Ttot * b.HV * b.K);
  w.dw = o; o += tcb ? 0 : al(sizeof(float) * Ttot * b.HV * b.K);  // the tensor-core path keeps dW as images
  w.dG = o; o += al(sizeof(float) * Ttot * b.HV);
  w.tc = o;
  w.himg = w.dhimg = w.vnimg = w.dvimg = w.dwimg = o;
  if (tcb) {
    gdn_chunk_args fa = forward_args(b);
    fa.force_generic = 0;
    o += al(tc_workspace_bytes(fa) + 1024);  // the tensor-core layout aligns its regions to 1 KiB
    const size_t imgs = static_cast<size_t>(nc) * b.HV;
    w.himg = o; o += al(imgs * tc::kStateImg);
    w.dhimg = o; o += al(imgs * tc::kStateImg);
    w.vnimg = o; o += al(imgs * tc::kVnImg);
    w.dvimg = o; o += al(imgs * tc::kVnImg);
    w.dwimg = o; o += al(imgs * tc::kVnImg);
  }
  w.total = o;
  return w;
}

cudaError_t launch_chunk_bwd(const gdn_chunk_bwd_args& b, const BwdWorkspace& ws, cudaStream_t s) {
  switch (b.qkv_dtype) {
    case GDN_F32: return run_bwd<float>(b, ws, s);
    case GDN_BF16: return run_bwd<__nv_bfloat16>(b, ws, s);
    case GDN_F16: return run_bwd<__half>(b, ws, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
