// Recurrent (token-by-token) gated delta-rule kernels.
//
// recurrent_vfirst_kernel: the slot-indexed decode of
//   fused_recurrent_gated_delta_rule_fn (triton/fla/fused_recurrent_fn.py:15-159).
//   The state is V-first ([slot][HV][V][K] f32).  For one token every state
//   row v is independent given (k, q): with S' = e^g S,
//     s_k = S_v . k,  s_q = S_v . q
//     v'  = beta (v_v - e^g s_k)
//     S_v <- e^g S_v + v' k,   o_v = e^g s_q + v' (k . q)
//   so each row is read once and written once.  With per-key decays gk (the
//   IS_KDA branch, fused_recurrent_fn.py:115-120) s_k and s_q use e^gk * k
//   and e^gk * q and the row decays by e^gk.  K/4 lanes share one row,
//   each holding a 128-bit segment, and the two dot products are reduced
//   together; the state is streamed with no-allocate loads and evict-first
//   stores.  This kernel is HBM-bound: 2 * HV * V * K * 4 bytes per sequence.
//   With K = 128 and aligned buffers the persistent streaming kernel of
//   gdn_decode_stream.cu is used instead.
//
// recurrent_kfirst_kernel: the plain recurrence of
//   fused_recurrent_gated_delta_rule (triton/fla/fused_recurrent.py:15-131)
//   with a K-first [N][HV][K][V] state and optional gk / gv decays.  One CTA
//   per (sequence, v-head) keeps the state in shared memory; thread v owns
//   column v.

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

template <typename T, int TPR, int RW, int kThreads>
__global__ void __launch_bounds__(kThreads)
recurrent_vfirst_kernel(const gdn_recurrent_args p) {
  constexpr int kWarps = kThreads / 32;
  constexpr int RPP = 32 / TPR;                  // rows per warp per slot
  constexpr int kRowsPerCta = kWarps * RPP * RW;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / TPR, seg = lane % TPR;
  const int64_t nh = blockIdx.x;
  const int64_t n = nh / p.HV;
  const int hv = static_cast<int>(nh % p.HV);
  const int h = hv / (p.HV / p.H);
  const int K = p.K, V = p.V;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  if (eos <= bos) return;  // no tokens (fused_recurrent_fn.py:62-64)

  int rows[RW];
#pragma unroll
  for (int j = 0; j < RW; ++j)
    rows[j] = blockIdx.y * kRowsPerCta + j * (kWarps * RPP) + warp * RPP + sub;

  const T* vptr = static_cast<const T*>(p.v);
  T* optr = static_cast<T*>(p.o);

  float4 S[RW];
#pragma unroll
  for (int j = 0; j < RW; ++j) S[j] = make_float4(0.f, 0.f, 0.f, 0.f);

  if (p.initial_state) {
    int64_t srow;
    if (p.ssm_state_indices) {
      int64_t i0 = 0;
      if (p.num_accepted_tokens) i0 = load_index(p.num_accepted_tokens, p.nacc_dtype, n) - 1;
      srow = load_index(p.ssm_state_indices, p.idx_dtype,
                        n * p.stride_indices_seq + i0 * p.stride_indices_tok);
      if (p.num_slots > 0 && srow >= p.num_slots) {  // past the declared slots: skipped like PAD
        if (threadIdx.x == 0 && blockIdx.y == 0)
          record_device_error(p.err, kErrSlotRange, kSiteSlotInitial, static_cast<int>(n), static_cast<int>(srow));
        srow = -1;
      }
      if (srow < 0) {  // PAD slot: skip the sequence, clear its outputs
        for (int64_t t = bos; t < eos; ++t)
#pragma unroll
          for (int j = 0; j < RW; ++j)
            if (seg == 0 && rows[j] < V) optr[(t * p.HV + hv) * V + rows[j]] = from_f<T>(0.f);
        return;
      }
    } else {
      srow = bos;  // reference indexes the state by bos (fused_recurrent_fn.py:101-102)
    }
    const float* base = p.initial_state + srow * p.stride_init_state_token +
                        static_cast<int64_t>(hv) * V * K + seg * 4;
#pragma unroll
    for (int j = 0; j < RW; ++j)
      if (rows[j] < V) S[j] = ld_stream(base + static_cast<int64_t>(rows[j]) * K);
  }

  const T* qb = static_cast<const T*>(p.q);
  const T* kb = static_cast<const T*>(p.k);
  for (int64_t t = bos; t < eos; ++t) {
    const int64_t qk_off = (t * p.H + h) * K + seg * 4;
    float4 q = load4<T>(qb + qk_off);
    float4 k = load4<T>(kb + qk_off);
    if (p.use_qk_l2norm) {
      float sq = group_sum<TPR>(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
      float sk = group_sum<TPR>(k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w);
      float rq = 1.f / sqrtf(sq + 1e-6f), rk = 1.f / sqrtf(sk + 1e-6f);
      q.x *= rq; q.y *= rq; q.z *= rq; q.w *= rq;
      k.x *= rk; k.y *= rk; k.z *= rk; k.w *= rk;
    }
    const float sc = p.scale;
    q.x *= sc; q.y *= sc; q.z *= sc; q.w *= sc;
    const float kq = group_sum<TPR>(k.x * q.x + k.y * q.y + k.z * q.z + k.w * q.w);
    const float eg = p.g ? expf(p.g[t * p.HV + hv]) : 1.f;
    float4 ek = make_float4(1.f, 1.f, 1.f, 1.f), kd = k, qd = q;
    if (p.gk) {  // per-key decay
      const float* gkr = p.gk + (t * p.HV + hv) * K + seg * 4;
      ek = make_float4(expf(gkr[0]), expf(gkr[1]), expf(gkr[2]), expf(gkr[3]));
      kd = make_float4(ek.x * k.x, ek.y * k.y, ek.z * k.z, ek.w * k.w);
      qd = make_float4(ek.x * q.x, ek.y * q.y, ek.z * q.z, ek.w * q.w);
    }
    const float beta_h = p.beta_per_v ? 0.f : p.beta[t * p.HV + hv];
#pragma unroll
    for (int j = 0; j < RW; ++j) {
      float sk = S[j].x * kd.x + S[j].y * kd.y + S[j].z * kd.z + S[j].w * kd.w;
      float sq = S[j].x * qd.x + S[j].y * qd.y + S[j].z * qd.z + S[j].w * qd.w;
      sk = group_sum<TPR>(sk);
      sq = group_sum<TPR>(sq);
      const int r = rows[j];
      const bool ok = r < V;
      const float vr = ok ? to_f<T>(vptr[(t * p.HV + hv) * V + r]) : 0.f;
      const float br = p.beta_per_v ? (ok ? p.beta[(t * p.HV + hv) * V + r] : 0.f) : beta_h;
      const float vp = br * (vr - eg * sk);
      S[j].x = eg * ek.x * S[j].x + vp * k.x;
      S[j].y = eg * ek.y * S[j].y + vp * k.y;
      S[j].z = eg * ek.z * S[j].z + vp * k.z;
      S[j].w = eg * ek.w * S[j].w + vp * k.w;
      if (ok && seg == 0) optr[(t * p.HV + hv) * V + r] = from_f<T>(eg * sq + vp * kq);
    }
    if (p.final_state) {
      int64_t frow;
      if (p.inplace_final_state) {
        frow = load_index(p.ssm_state_indices, p.idx_dtype,
                          n * p.stride_indices_seq + (t - bos) * p.stride_indices_tok);
        if (p.num_slots > 0 && frow >= p.num_slots) {
          if (threadIdx.x == 0 && blockIdx.y == 0)
            record_device_error(p.err, kErrSlotRange, kSiteSlotFinal, static_cast<int>(n), static_cast<int>(frow));
          frow = -1;
        }
      } else {
        frow = t;
      }
      if (frow >= 0) {
        float* base = p.final_state + frow * p.stride_final_state_token +
                      static_cast<int64_t>(hv) * V * K + seg * 4;
#pragma unroll
        for (int j = 0; j < RW; ++j)
          if (rows[j] < V) st_stream(base + static_cast<int64_t>(rows[j]) * K, S[j]);
      }
    }
  }
}

template <typename T>
__global__ void recurrent_kfirst_kernel(const gdn_recurrent_plain_args p) {
  extern __shared__ float smem[];
  const int K = p.K, V = p.V;
  float* S = smem;             // [K][V]
  float* qs = S + K * V;       // [K]  scale * q (normalised), times exp(gk)
  float* ks = qs + K;          // [K]  k (normalised), times exp(gk)
  float* kraw = ks + K;        // [K]  k (normalised)
  float* qraw = kraw + K;      // [K]
  float* gks = qraw + K;       // [K]  exp(gk)
  float* red = gks + K;        // [4]
  const int64_t nh = blockIdx.x;
  const int64_t n = nh / p.HV;
  const int hv = static_cast<int>(nh % p.HV);
  const int h = hv / (p.HV / p.H);
  const int tid = threadIdx.x;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const float scale = p.scale > 0.f ? p.scale : rsqrtf(static_cast<float>(K));

  for (int i = tid; i < K * V; i += blockDim.x)
    S[i] = p.initial_state ? p.initial_state[nh * K * V + i] : 0.f;
  __syncthreads();

  const T* qb = static_cast<const T*>(p.q);
  const T* kb = static_cast<const T*>(p.k);
  const T* vb = static_cast<const T*>(p.v);
  T* ob = static_cast<T*>(p.o);
  for (int64_t t = bos; t < eos; ++t) {
    for (int i = tid; i < K; i += blockDim.x) {
      qraw[i] = to_f<T>(qb[(t * p.H + h) * K + i]);
      kraw[i] = to_f<T>(kb[(t * p.H + h) * K + i]);
      gks[i] = p.gk ? expf(p.gk[(t * p.HV + hv) * K + i]) : 1.f;
    }
    __syncthreads();
    if (tid == 0) {
      float sq = 0.f, sk = 0.f;
      for (int i = 0; i < K; ++i) { sq += qraw[i] * qraw[i]; sk += kraw[i] * kraw[i]; }
      red[0] = p.use_qk_l2norm ? 1.f / sqrtf(sq + 1e-6f) : 1.f;
      red[1] = p.use_qk_l2norm ? 1.f / sqrtf(sk + 1e-6f) : 1.f;
    }
    __syncthreads();
    for (int i = tid; i < K; i += blockDim.x) {
      const float qv = qraw[i] * red[0] * scale, kv = kraw[i] * red[1];
      qraw[i] = qv;
      kraw[i] = kv;
      qs[i] = qv * gks[i];
      ks[i] = kv * gks[i];
    }
    __syncthreads();
    if (tid < V) {
      const int vv = tid;
      float sk = 0.f, sq = 0.f, kq = 0.f;
      for (int i = 0; i < K; ++i) {
        const float s = S[i * V + vv];
        sk += s * ks[i];
        sq += s * qs[i];
        kq += kraw[i] * qraw[i];
      }
      float eg = p.g ? expf(p.g[t * p.HV + hv]) : 1.f;
      if (p.gv) eg *= expf(p.gv[(t * p.HV + hv) * V + vv]);
      const float br = p.beta_per_v ? p.beta[(t * p.HV + hv) * V + vv] : p.beta[t * p.HV + hv];
      const float vr = to_f<T>(vb[(t * p.HV + hv) * V + vv]);
      const float vp = br * (vr - eg * sk);
      for (int i = 0; i < K; ++i) S[i * V + vv] = eg * gks[i] * S[i * V + vv] + kraw[i] * vp;
      ob[(t * p.HV + hv) * V + vv] = from_f<T>(eg * sq + vp * kq);
    }
    __syncthreads();
  }
  if (p.final_state)
    for (int i = tid; i < K * V; i += blockDim.x) p.final_state[nh * K * V + i] = S[i];
}

// ---- launchers ---------------------------------------------------------------

template <typename T, int TPR, int RW, int kThreads = 128>
static cudaError_t launch_vfirst_t(const gdn_recurrent_args& a, cudaStream_t s) {
  constexpr int kRowsPerCta = (kThreads / 32) * (32 / TPR) * RW;
  dim3 grid(static_cast<unsigned>(a.N * a.HV), (a.V + kRowsPerCta - 1) / kRowsPerCta);
  note_launch();
  recurrent_vfirst_kernel<T, TPR, RW, kThreads><<<grid, kThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_vfirst_k(const gdn_recurrent_args& a, cudaStream_t s) {
  switch (a.K / 4) {
    case 32: return launch_vfirst_t<T, 32, 4>(a, s);
    case 16: return launch_vfirst_t<T, 16, 2>(a, s);
    case 8: return launch_vfirst_t<T, 8, 1>(a, s);
    case 4: return launch_vfirst_t<T, 4, 1>(a, s);
    case 2: return launch_vfirst_t<T, 2, 1>(a, s);
    case 1: return launch_vfirst_t<T, 1, 1>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_recurrent_vfirst(const gdn_recurrent_args& a, cudaStream_t s) {
  if (decode_stream_applies(a)) return launch_decode_stream(a, s);
  switch (a.qkv_dtype) {
    case GDN_F32: return launch_vfirst_k<float>(a, s);
    case GDN_BF16: return launch_vfirst_k<__nv_bfloat16>(a, s);
    case GDN_F16: return launch_vfirst_k<__half>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_kfirst_t(const gdn_recurrent_plain_args& a, cudaStream_t s) {
  const size_t smem = (static_cast<size_t>(a.K) * a.V + 5 * a.K + 4) * sizeof(float);
  auto kern = recurrent_kfirst_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int threads = ((a.V + 31) / 32) * 32;
  note_launch();
  kern<<<static_cast<unsigned>(a.N * a.HV), threads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_recurrent_kfirst(const gdn_recurrent_plain_args& a, cudaStream_t s) {
  switch (a.qkv_dtype) {
    case GDN_F32: return launch_kfirst_t<float>(a, s);
    case GDN_BF16: return launch_kfirst_t<__nv_bfloat16>(a, s);
    case GDN_F16: return launch_kfirst_t<__half>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
