// Generic chunked gated delta-rule forward: fp32 SIMT kernels.
//
// This is the full-precision path (fp32 inputs, any K, V <= 128).  It runs
// the reference's six stages (triton/fla/chunk.py:10-74) as four kernels with
// fp32 intermediates in the caller's workspace:
//   chunk_prep_kernel   q/k -> f32, optional L2 norm (fused_recurrent_fn.py:110-112 formula)
//   chunk_wy_kernel     cumsum of g (cumsum.py:20-77), A = beta exp(G_i-G_j) k_i.k_j
//                       (chunk_scaled_dot_kkt.py:25-100), (I+A)^-1 by forward
//                       substitution (solve_tril.py:491-537), w, u (wy_fast.py:18-119)
//   chunk_state_kernel  inter-chunk recurrence (chunk_delta_h.py:28-197)
//   chunk_out_kernel    output (chunk_o.py:30-170)
// The bf16/fp16 Qwen3-Next shapes take the tcgen05 path in gdn_chunk_tc.cu.

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "tile_gemm.cuh"
#include "solve_tril.cuh"

namespace gdn {

__global__ void chunk_plan_kernel(const void* cu, int cu_dtype, int64_t N, int64_t T,
                                  int64_t* off, int chunk, int* err, int* zero, int64_t nzero) {
  __shared__ int64_t warp_tot[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) { carry = 0; off[0] = 0; }
  if (err && threadIdx.x < 4) err[threadIdx.x] = 0;  // the call's device error word starts clear
  for (int64_t i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < N; base += blockDim.x) {
    const int64_t n = base + threadIdx.x;
    int64_t cnt = 0;
    if (n < N) {
      int64_t bos, eos;
      seq_bounds(cu, cu_dtype, n, T, bos, eos);
      cnt = eos > bos ? (eos - bos + chunk - 1) / chunk : 0;
    }
    int64_t x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int64_t t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int64_t y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      warp_tot[lane] = t;
    }
    __syncthreads();
    const int64_t incl = x + (warp > 0 ? warp_tot[warp - 1] : 0) + carry;
    if (n < N) off[n + 1] = incl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
}

cudaError_t launch_chunk_plan(const void* cu, int cu_dtype, int64_t N, int64_t T,
                              int64_t* chunk_offsets, cudaStream_t s, int chunk, int* err, int* zero,
                              int64_t nzero) {
  chunk_plan_kernel<<<1, 1024, 0, s>>>(cu, cu_dtype, N, T, chunk_offsets, chunk, err, zero, nzero);
  return cudaGetLastError();
}

template <typename T>
__global__ void chunk_prep_kernel(const T* __restrict__ x, float* __restrict__ y,
                                  int64_t rows, int K, int l2) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float ss = 0.f;
  for (int i = lane; i < K; i += 32) {
    const float v = to_f<T>(x[row * K + i]);
    ss += v * v;
  }
  ss = group_sum<32>(ss);
  const float r = l2 ? 1.f / sqrtf(ss + 1e-6f) : 1.f;
  for (int i = lane; i < K; i += 32) y[row * K + i] = to_f<T>(x[row * K + i]) * r;
}

struct GenericPtrs {
  const int64_t* coff;
  float* gc;
  const float* qn;
  const float* kn;
  float* w;
  float* u;
  float* vnew;
  float* hs;
};

constexpr int kLD = kRowK;  // row stride of 64 x K fp32 tiles (row-major / k-contiguous reads)

// Per (chunk, v-head): G = chunk-local cumsum of g, A = tril_strict(diag(beta)
// exp(G_i - G_j) K K^T), T = (I + A)^-1, W = T diag(beta exp(G)) K,
// U = T diag(beta) V.
template <typename T>
__global__ void __launch_bounds__(kGemmThreads)
chunk_wy_kernel(const gdn_chunk_args p, const GenericPtrs w) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* Tm = sm;                  // [64][kTS] (16-byte aligned)
  float* Zs = Tm + 64 * kTS;       // kTrilScratch floats of solve scratch (16-byte aligned)
  float* A = Zs + kTrilScratch;    // [64][65]
  float* ks = A + 64 * 65;         // [64][kLD]
  float* vs = ks + 64 * kLD;       // [64][kLD]
  float* gcs = vs + 64 * kLD;      // [64]
  float* bs = gcs + 64;            // [64]
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int tid = threadIdx.x;
  const int64_t rowK = static_cast<int64_t>(p.HV) * K, rowV = static_cast<int64_t>(p.HV) * V;
  const T* vb = static_cast<const T*>(p.v);
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      ks[i * kLD + kk] = i < L ? w.kn[((s + i) * p.H + h) * K + kk] : 0.f;
    }
  }
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      vs[i * kLD + vv] = i < L ? to_f<T>(vb[(s + i) * rowV + static_cast<int64_t>(hv) * V + vv]) : 0.f;
    }
  }
  if (tid < 32) {  // chunk-local cumsum of g: warp scan over 2 x 32 values
    float x0 = tid < L ? p.g[(s + tid) * p.HV + hv] : 0.f;
    float x1 = tid + 32 < L ? p.g[(s + tid + 32) * p.HV + hv] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_up_sync(0xffffffffu, x0, o), y1 = __shfl_up_sync(0xffffffffu, x1, o);
      if (tid >= o) {
        x0 += y0;
        x1 += y1;
      }
    }
    x1 += __shfl_sync(0xffffffffu, x0, 31);
    gcs[tid] = x0;
    gcs[tid + 32] = x1;
  }
  if (tid < 64) bs[tid] = tid < L ? p.beta[(s + tid) * p.HV + hv] : 0.f;
  gemm_smem<false, kSplit<T>>(A, 65, 64, 64, K, ks, kLD, 1, ks, 1, kLD);  // K K^T
  if (tid < L) w.gc[(s + tid) * p.HV + hv] = gcs[tid];
  for (int e = tid; e < 64 * 64; e += kGemmThreads) {
    const int i = e >> 6, j = e & 63;
    A[i * 65 + j] = (i < L && j < i) ? bs[i] * expf(gcs[i] - gcs[j]) * A[i * 65 + j] : 0.f;
  }
  __syncthreads();
  solve_tril64_nt<kGemmThreads>(A, Tm, Zs);  // (I + A)^-1; ends with a barrier
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {  // rows of K by beta exp(G)
    for (int kk = tid & 31; kk < K; kk += 32) {
      ks[i * kLD + kk] *= bs[i] * expf(gcs[i]);
    }
  }
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {  // rows of V by beta
    for (int vv = tid & 31; vv < V; vv += 32) {
      vs[i * kLD + vv] *= bs[i];
    }
  }
  gemm_smem<false, kSplit<T>>(w.w + s * rowK + static_cast<int64_t>(hv) * K, rowK, L, K, 64, Tm, kTS, 1, ks, kLD, 1);
  gemm_smem<false, kSplit<T>>(w.u + s * rowV + static_cast<int64_t>(hv) * V, rowV, L, V, 64, Tm, kTS, 1, vs, kLD, 1);
}

constexpr int kStateCols = 32;
constexpr int kStateStage = 64 * kRowK + 64 * kRowN + 64 * kRow32 + 64;  // wc, kc, u slice, G

// Inter-chunk recurrence for one (sequence, v-head, 32-column slice of V):
// per chunk v_new = U - W h, h <- exp(G_last) h + K^T diag(exp(G_last - G)) v_new.
// The next chunk's W, K, U and G are copied in (cp.async) while the current
// chunk computes.
__global__ void __launch_bounds__(kGemmThreads, 1)
chunk_state_kernel(const gdn_chunk_args p, const GenericPtrs w) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* hsm = sm;                          // [128][kRow32] state slice
  float* stage0 = hsm + 128 * kRow32;       // 2 stages of kStateStage floats
  const int64_t n = blockIdx.x;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  const int v0 = blockIdx.z * kStateCols;
  const int vcols = V - v0 < kStateCols ? V - v0 : kStateCols;
  const int tid = threadIdx.x;
  const int64_t rowK = static_cast<int64_t>(p.HV) * K, rowV = static_cast<int64_t>(p.HV) * V;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  for (int e = tid; e < 128 * kStateCols; e += kGemmThreads) {
    const int kk = e / kStateCols, c = e % kStateCols, vv = v0 + c;
    float x = 0.f;
    if (p.initial_state && vv < V && kk < K)
      x = p.state_v_first ? p.initial_state[((n * p.HV + hv) * V + vv) * K + kk]
                          : p.initial_state[((n * p.HV + hv) * K + kk) * V + vv];
    hsm[kk * kRow32 + c] = x;
  }
  const int64_t nchunks = eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0;
  auto issue = [&](int64_t lc) {
    float* wc = stage0 + (lc & 1) * kStateStage;
    float* kc = wc + 64 * kRowK;
    float* us = kc + 64 * kRowN;
    float* gs = us + 64 * kRow32;
    const int64_t s = bos + lc * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    tile_async(wc, kRowK, w.w + s * rowK + static_cast<int64_t>(hv) * K, rowK, L, 64, K, K);
    tile_async(kc, kRowN, w.kn + (s * p.H + h) * K, static_cast<int64_t>(p.H) * K, L, 64, K, K);
    tile_async(us, kRow32, w.u + s * rowV + static_cast<int64_t>(hv) * V + v0, rowV, L, 64, vcols, kStateCols);
    if (tid < 64) cp_async4(gs + tid, tid < L ? w.gc + (s + tid) * p.HV + hv : w.gc, tid < L);
    cp_async_commit();
  };
  if (nchunks > 0) issue(0);
  for (int64_t lc = 0; lc < nchunks; ++lc) {
    const int64_t s = bos + lc * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    const int64_t cidx = w.coff[n] + lc;
    float* wc = stage0 + (lc & 1) * kStateStage;
    float* kc = wc + 64 * kRowK;
    float* us = kc + 64 * kRowN;
    float* gs = us + 64 * kRow32;
    if (lc + 1 < nchunks) {
      issue(lc + 1);  // the other stage was last read before the previous iteration's final barrier
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float* hg = w.hs + (cidx * p.HV + hv) * static_cast<int64_t>(K) * V;
    for (int e = tid; e < K * kStateCols; e += kGemmThreads) {
      const int kk = e / kStateCols, c = e % kStateCols;
      if (c < vcols) hg[kk * V + v0 + c] = hsm[kk * kRow32 + c];
    }
    gemm_smem<true>(us, kRow32, 64, kStateCols, K, wc, kRowK, 1, hsm, kRow32, 1, -1.f);  // U - W h
    const float glast = gs[L - 1], eg = expf(glast);
    for (int e = tid; e < 64 * kStateCols; e += kGemmThreads) {
      const int i = e / kStateCols, c = e % kStateCols;
      const float x = us[i * kRow32 + c];
      if (i < L && c < vcols) w.vnew[(s + i) * rowV + static_cast<int64_t>(hv) * V + v0 + c] = x;
      us[i * kRow32 + c] = i < L ? x * expf(glast - gs[i]) : 0.f;
    }
    for (int e = tid; e < K * kStateCols; e += kGemmThreads) hsm[(e / kStateCols) * kRow32 + e % kStateCols] *= eg;
    gemm_smem<true>(hsm, kRow32, min(K, 64), kStateCols, 64, kc, 1, kRowN, us, kRow32, 1);
    if (K > 64)
      gemm_smem<true>(hsm + 64 * kRow32, kRow32, K - 64, kStateCols, 64, kc + 64, 1, kRowN, us, kRow32, 1);
  }
  __syncthreads();
  if (p.final_state) {
    for (int e = tid; e < K * kStateCols; e += kGemmThreads) {
      const int kk = e / kStateCols, c = e % kStateCols, vv = v0 + c;
      if (c >= vcols) continue;
      if (p.state_v_first) p.final_state[((n * p.HV + hv) * V + vv) * K + kk] = hsm[kk * kRow32 + c];
      else p.final_state[((n * p.HV + hv) * K + kk) * V + vv] = hsm[kk * kRow32 + c];
    }
  }
}

// Output of one (chunk, v-head): o = scale (diag(exp(G)) Q h + (M * D * Q K^T) v_new).
template <typename T>
__global__ void __launch_bounds__(kGemmThreads)
chunk_out_kernel(const gdn_chunk_args p, const GenericPtrs w, float scale) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* qc = sm;                // [64][kLD]
  float* kc = qc + 64 * kLD;     // [64][kLD]
  float* oc = kc + 64 * kLD;     // [64][kLD]
  float* att = oc + 64 * kLD;    // [64][65]
  float* gcs = att + 64 * 65;    // [64]
  float* st = gcs + 64;          // staging
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t cidx = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t rowV = static_cast<int64_t>(p.HV) * V;
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int kk = tid & 31; kk < K; kk += 32) {
      qc[i * kLD + kk] = i < L ? w.qn[((s + i) * p.H + h) * K + kk] : 0.f;
      kc[i * kLD + kk] = i < L ? w.kn[((s + i) * p.H + h) * K + kk] : 0.f;
    }
  }
  if (tid < 64) gcs[tid] = tid < L ? w.gc[(s + tid) * p.HV + hv] : 0.f;
  gemm_smem<false, kSplit<T>>(att, 65, 64, 64, K, qc, kLD, 1, kc, 1, kLD);  // Q K^T
  for (int e = tid; e < 64 * 64; e += kGemmThreads) {
    const int i = e >> 6, j = e & 63;
    att[i * 65 + j] = (i < L && j <= i) ? att[i * 65 + j] * expf(gcs[i] - gcs[j]) : 0.f;
  }
  const float* hc = w.hs + (cidx * p.HV + hv) * static_cast<int64_t>(K) * V;
  gemm_staged<false, kSplit<T>>(oc, kLD, 64, V, K, qc, kLD, 1, 64, hc, V, 1, V, 1.f, st);  // Q h
  for (int i = tid >> 5; i < 64; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      oc[i * kLD + vv] *= expf(gcs[i]);
    }
  }
  const float* vn = w.vnew + s * rowV + static_cast<int64_t>(hv) * V;
  gemm_staged<true, kSplit<T>>(oc, kLD, 64, V, L, att, 65, 1, 64, vn, rowV, 1, V, 1.f, st);  // + P v_new
  T* ob = static_cast<T*>(p.o) + s * rowV + static_cast<int64_t>(hv) * V;
  for (int i = tid >> 5; i < L; i += kGemmThreads / 32) {
    for (int vv = tid & 31; vv < V; vv += 32) {
      ob[i * rowV + vv] = from_f<T>(scale * oc[i * kLD + vv]);
    }
  }
}

ChunkWorkspace plan_generic_workspace(const gdn_chunk_args& a) {
  auto al = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  const int64_t Ttot = a.B * a.T;
  const int64_t nc = chunk_upper_bound(Ttot, a.N);
  ChunkWorkspace w{};
  size_t o = 0;
  w.err = o; o += al(16);
  w.chunk_offsets = o; o += al(sizeof(int64_t) * (a.N + 1));
  w.gc = o; o += al(sizeof(float) * Ttot * a.HV);
  w.qn = o; o += al(sizeof(float) * Ttot * a.H * a.K);
  w.kn = o; o += al(sizeof(float) * Ttot * a.H * a.K);
  w.w = o; o += al(sizeof(float) * Ttot * a.HV * a.K);
  w.u = o; o += al(sizeof(float) * Ttot * a.HV * a.V);
  w.vnew = o; o += al(sizeof(float) * Ttot * a.HV * a.V);
  w.hs = o; o += al(sizeof(float) * nc * a.HV * a.K * a.V);
  w.total = o;
  return w;
}

template <typename T>
static cudaError_t run_generic(const gdn_chunk_args& a, const ChunkWorkspace& ws, cudaStream_t s,
                               bool with_output) {
  char* base = static_cast<char*>(a.workspace);
  GenericPtrs w;
  w.coff = reinterpret_cast<const int64_t*>(base + ws.chunk_offsets);
  w.gc = reinterpret_cast<float*>(base + ws.gc);
  w.qn = reinterpret_cast<const float*>(base + ws.qn);
  w.kn = reinterpret_cast<const float*>(base + ws.kn);
  w.w = reinterpret_cast<float*>(base + ws.w);
  w.u = reinterpret_cast<float*>(base + ws.u);
  w.vnew = reinterpret_cast<float*>(base + ws.vnew);
  w.hs = reinterpret_cast<float*>(base + ws.hs);
  const int64_t Ttot = a.B * a.T;
  const int64_t nc = chunk_upper_bound(Ttot, a.N);
  LaunchHooks hk(a.stage_events, a.n_stage_events);
  hk.pre(s);
  cudaError_t e = launch_chunk_plan(a.cu_seqlens, a.cu_dtype, a.N, a.T,
                                    reinterpret_cast<int64_t*>(base + ws.chunk_offsets), s, 64,
                                    reinterpret_cast<int*>(base + ws.err));
  if (e != cudaSuccess) return e;
  const int64_t rows = Ttot * a.H;
  if (rows > 0) {
    const unsigned pb = static_cast<unsigned>((rows + 7) / 8);
    hk.pre(s);
    chunk_prep_kernel<T><<<pb, 256, 0, s>>>(static_cast<const T*>(a.q), const_cast<float*>(w.qn),
                                            rows, a.K, a.use_qk_l2norm);
    hk.pre(s);
    chunk_prep_kernel<T><<<pb, 256, 0, s>>>(static_cast<const T*>(a.k), const_cast<float*>(w.kn),
                                            rows, a.K, a.use_qk_l2norm);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const float scale = a.scale > 0.f ? a.scale : 1.f / sqrtf(static_cast<float>(a.K));
  const size_t wy_smem = sizeof(float) * (64 * kTS + kTrilScratch + 64 * 65 + 2 * 64 * kLD + 2 * 64);
  const size_t st_smem = sizeof(float) * (128 * kRow32 + 2 * kStateStage);
  const size_t out_smem = sizeof(float) * (3 * 64 * kLD + 64 * 65 + 64 + kGemmStage);
  if ((e = cudaFuncSetAttribute(chunk_wy_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(wy_smem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(st_smem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(chunk_out_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(out_smem))) != cudaSuccess) return e;
  if (nc > 0) {
    hk.pre(s);
    chunk_wy_kernel<T><<<dim3(static_cast<unsigned>(nc), a.HV), kGemmThreads, wy_smem, s>>>(a, w);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  hk.pre(s);
  chunk_state_kernel<<<dim3(static_cast<unsigned>(a.N), a.HV, (a.V + kStateCols - 1) / kStateCols),
                       kGemmThreads, st_smem, s>>>(a, w);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (nc > 0 && with_output) {
    hk.pre(s);
    chunk_out_kernel<T><<<dim3(static_cast<unsigned>(nc), a.HV), kGemmThreads, out_smem, s>>>(a, w, scale);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  hk.end(s);
  return cudaSuccess;
}

cudaError_t launch_chunk_generic(const gdn_chunk_args& a, const ChunkWorkspace& ws, cudaStream_t s) {
  switch (a.qkv_dtype) {
    case GDN_F32: return run_generic<float>(a, ws, s, true);
    case GDN_BF16: return run_generic<__nv_bfloat16>(a, ws, s, true);
    case GDN_F16: return run_generic<__half>(a, ws, s, true);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_chunk_generic_recompute(const gdn_chunk_args& a, const ChunkWorkspace& ws, cudaStream_t s) {
  switch (a.qkv_dtype) {
    case GDN_F32: return run_generic<float>(a, ws, s, false);
    case GDN_BF16: return run_generic<__nv_bfloat16>(a, ws, s, false);
    case GDN_F16: return run_generic<__half>(a, ws, s, false);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
