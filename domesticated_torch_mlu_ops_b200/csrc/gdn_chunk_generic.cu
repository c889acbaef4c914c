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
#include "solve_tril.cuh"

namespace gdn {

__global__ void chunk_plan_kernel(const void* cu, int cu_dtype, int64_t N, int64_t T,
                                  int64_t* off, int chunk) {
  __shared__ int64_t warp_tot[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) { carry = 0; off[0] = 0; }
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
                              int64_t* chunk_offsets, cudaStream_t s, int chunk) {
  chunk_plan_kernel<<<1, 1024, 0, s>>>(cu, cu_dtype, N, T, chunk_offsets, chunk);
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

template <typename T>
__global__ void __launch_bounds__(256)
chunk_wy_kernel(const gdn_chunk_args p, const GenericPtrs w) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* ks = sm;                 // [64][K]
  float* vs = ks + 64 * K;        // [64][V]
  float* A = vs + 64 * V;         // [64][65]
  float* Tm = A + 64 * 68;        // [64][kTS] (A rows use 65, padded to 68)
  float* gcs = Tm + 64 * kTS;     // [64]
  float* bs = gcs + 64;           // [64]
  float* cw = bs + 64;            // [64] beta * exp(G)
  float* Zs = cw + 64;            // kTrilScratch floats of solve scratch
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int tid = threadIdx.x;
  const T* vb = static_cast<const T*>(p.v);
  for (int e = tid; e < 64 * K; e += blockDim.x) {
    const int i = e / K, kk = e % K;
    ks[e] = i < L ? w.kn[((s + i) * p.H + h) * K + kk] : 0.f;
  }
  for (int e = tid; e < 64 * V; e += blockDim.x) {
    const int i = e / V, vv = e % V;
    vs[e] = i < L ? to_f<T>(vb[((s + i) * p.HV + hv) * V + vv]) : 0.f;
  }
  if (tid < 64) bs[tid] = tid < L ? p.beta[(s + tid) * p.HV + hv] : 0.f;
  if (tid == 0) {
    float acc = 0.f;
    for (int i = 0; i < 64; ++i) {
      if (i < L) acc += p.g[(s + i) * p.HV + hv];
      gcs[i] = acc;
    }
  }
  __syncthreads();
  if (tid < L) {
    w.gc[(s + tid) * p.HV + hv] = gcs[tid];
    cw[tid] = bs[tid] * expf(gcs[tid]);
  } else if (tid < 64) {
    cw[tid] = 0.f;
  }
  for (int e = tid; e < 64 * 64; e += blockDim.x) {
    const int i = e >> 6, j = e & 63;
    float a = 0.f;
    if (i < L && j < i) {
      const float* ki = ks + i * K;
      const float* kj = ks + j * K;
      for (int kk = 0; kk < K; ++kk) a += ki[kk] * kj[kk];
      a *= bs[i] * expf(gcs[i] - gcs[j]);
    }
    A[i * 65 + j] = a;
  }
  __syncthreads();
  solve_tril64_nt<256>(A, Tm, Zs);  // (I + A)^-1; ends with a barrier
  for (int e = tid; e < L * K; e += blockDim.x) {
    const int i = e / K, kk = e % K;
    float acc = 0.f;
    for (int j = 0; j <= i; ++j) acc += Tm[i * kTS + j] * cw[j] * ks[j * K + kk];
    w.w[((s + i) * p.HV + hv) * K + kk] = acc;
  }
  for (int e = tid; e < L * V; e += blockDim.x) {
    const int i = e / V, vv = e % V;
    float acc = 0.f;
    for (int j = 0; j <= i; ++j) acc += Tm[i * kTS + j] * bs[j] * vs[j * V + vv];
    w.u[((s + i) * p.HV + hv) * V + vv] = acc;
  }
}

constexpr int kStateCols = 32;

__global__ void __launch_bounds__(256)
chunk_state_kernel(const gdn_chunk_args p, const GenericPtrs w) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* hsm = sm;                    // [K][32]
  float* vn = hsm + K * kStateCols;   // [64][32]
  float* wc = vn + 64 * kStateCols;   // [64][K]
  float* kc = wc + 64 * K;            // [64][K]
  float* gcs = kc + 64 * K;           // [64]
  const int64_t n = blockIdx.x;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  const int v0 = blockIdx.z * kStateCols;
  const int tid = threadIdx.x;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  for (int e = tid; e < K * kStateCols; e += blockDim.x) {
    const int kk = e / kStateCols, vv = v0 + e % kStateCols;
    float x = 0.f;
    if (p.initial_state && vv < V)
      x = p.state_v_first ? p.initial_state[((n * p.HV + hv) * V + vv) * K + kk]
                          : p.initial_state[((n * p.HV + hv) * K + kk) * V + vv];
    hsm[e] = x;
  }
  __syncthreads();
  const int64_t nchunks = eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0;
  for (int64_t lc = 0; lc < nchunks; ++lc) {
    const int64_t s = bos + lc * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    const int64_t cidx = w.coff[n] + lc;
    for (int e = tid; e < K * kStateCols; e += blockDim.x) {
      const int kk = e / kStateCols, vv = v0 + e % kStateCols;
      if (vv < V) w.hs[((cidx * p.HV + hv) * K + kk) * V + vv] = hsm[e];
    }
    for (int e = tid; e < 64 * K; e += blockDim.x) {
      const int i = e / K, kk = e % K;
      wc[e] = i < L ? w.w[((s + i) * p.HV + hv) * K + kk] : 0.f;
      kc[e] = i < L ? w.kn[((s + i) * p.H + h) * K + kk] : 0.f;
    }
    if (tid < 64) gcs[tid] = tid < L ? w.gc[(s + tid) * p.HV + hv] : 0.f;
    __syncthreads();
    for (int e = tid; e < 64 * kStateCols; e += blockDim.x) {
      const int i = e / kStateCols, c = e % kStateCols, vv = v0 + c;
      float x = 0.f;
      if (i < L && vv < V) {
        float acc = 0.f;
        for (int kk = 0; kk < K; ++kk) acc += wc[i * K + kk] * hsm[kk * kStateCols + c];
        x = w.u[((s + i) * p.HV + hv) * V + vv] - acc;
        w.vnew[((s + i) * p.HV + hv) * V + vv] = x;
      }
      vn[e] = x;
    }
    __syncthreads();
    const float glast = gcs[L - 1];
    const float eg = expf(glast);
    for (int e = tid; e < K * kStateCols; e += blockDim.x) {
      const int kk = e / kStateCols, c = e % kStateCols;
      float acc = 0.f;
      for (int i = 0; i < L; ++i) acc += kc[i * K + kk] * expf(glast - gcs[i]) * vn[i * kStateCols + c];
      hsm[e] = eg * hsm[e] + acc;
    }
    __syncthreads();
  }
  if (p.final_state) {
    for (int e = tid; e < K * kStateCols; e += blockDim.x) {
      const int kk = e / kStateCols, vv = v0 + e % kStateCols;
      if (vv >= V) continue;
      if (p.state_v_first) p.final_state[((n * p.HV + hv) * V + vv) * K + kk] = hsm[e];
      else p.final_state[((n * p.HV + hv) * K + kk) * V + vv] = hsm[e];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
chunk_out_kernel(const gdn_chunk_args p, const GenericPtrs w, float scale) {
  extern __shared__ float sm[];
  const int K = p.K, V = p.V;
  float* qc = sm;               // [64][K]
  float* kc = qc + 64 * K;      // [64][K]
  float* att = kc + 64 * K;     // [64][65]
  float* gcs = att + 64 * 65;   // [64]
  int64_t n, lc;
  if (!locate_chunk(w.coff, p.N, blockIdx.x, n, lc)) return;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t cidx = blockIdx.x;
  const int tid = threadIdx.x;
  for (int e = tid; e < 64 * K; e += blockDim.x) {
    const int i = e / K, kk = e % K;
    qc[e] = i < L ? w.qn[((s + i) * p.H + h) * K + kk] : 0.f;
    kc[e] = i < L ? w.kn[((s + i) * p.H + h) * K + kk] : 0.f;
  }
  if (tid < 64) gcs[tid] = tid < L ? w.gc[(s + tid) * p.HV + hv] : 0.f;
  __syncthreads();
  for (int e = tid; e < 64 * 64; e += blockDim.x) {
    const int i = e >> 6, j = e & 63;
    float a = 0.f;
    if (i < L && j <= i) {
      for (int kk = 0; kk < K; ++kk) a += qc[i * K + kk] * kc[j * K + kk];
      a *= expf(gcs[i] - gcs[j]);
    }
    att[i * 65 + j] = a;
  }
  __syncthreads();
  const float* hc = w.hs + cidx * p.HV * K * V + static_cast<int64_t>(hv) * K * V;
  T* ob = static_cast<T*>(p.o);
  for (int e = tid; e < L * V; e += blockDim.x) {
    const int i = e / V, vv = e % V;
    float inter = 0.f;
    for (int kk = 0; kk < K; ++kk) inter += qc[i * K + kk] * hc[kk * V + vv];
    float intra = 0.f;
    for (int j = 0; j <= i; ++j) intra += att[i * 65 + j] * w.vnew[((s + j) * p.HV + hv) * V + vv];
    ob[((s + i) * p.HV + hv) * V + vv] = from_f<T>(scale * (expf(gcs[i]) * inter + intra));
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
                                    reinterpret_cast<int64_t*>(base + ws.chunk_offsets), s);
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
  const size_t wy_smem = sizeof(float) * (64 * a.K + 64 * a.V + 2 * 64 * 68 + 3 * 64 + kTrilScratch);
  const size_t st_smem = sizeof(float) * (a.K * kStateCols + 64 * kStateCols + 2 * 64 * a.K + 64);
  const size_t out_smem = sizeof(float) * (2 * 64 * a.K + 64 * 65 + 64);
  if ((e = cudaFuncSetAttribute(chunk_wy_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(wy_smem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(st_smem))) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(chunk_out_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(out_smem))) != cudaSuccess) return e;
  if (nc > 0) {
    hk.pre(s);
    chunk_wy_kernel<T><<<dim3(static_cast<unsigned>(nc), a.HV), 256, wy_smem, s>>>(a, w);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  hk.pre(s);
  chunk_state_kernel<<<dim3(static_cast<unsigned>(a.N), a.HV, (a.V + kStateCols - 1) / kStateCols),
                       256, st_smem, s>>>(a, w);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (nc > 0 && with_output) {
    hk.pre(s);
    chunk_out_kernel<T><<<dim3(static_cast<unsigned>(nc), a.HV), 256, out_smem, s>>>(a, w, scale);
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
