// Streaming slot-cache decode: the fused_recurrent_gated_delta_rule_fn
// recurrence (triton/fla/fused_recurrent_fn.py:15-159) for K = 128, written
// as a persistent pipeline so that HBM never waits on a CTA's serial
// index -> state -> compute -> store chain.
//
// One CTA per SM loops over (sequence, v-head) items (rows of a V-first
// state are independent, so the item is a block of up to kRows state rows;
// with V <= 128 that is the whole V x 128 fp32 state, 64 KiB).  The 32 lanes
// of a producer warp look up 32 items at once (state slot from
// ssm_state_indices, PAD = -1, num_accepted_tokens; first gate and beta),
// and lane 0 issues 1-D bulk copies of each state block and of the first
// token's q, k, v rows into one of three shared-memory stages.  Eight
// consumer warps update the block in place (eight lanes per row, each owning
// four 16-byte segments, so one 3-step shuffle reduction serves four rows)
// and write it back with a bulk store.  The stage of a stored block is
// released only when the next item ends (its store has read it by then), so
// the consumers never wait on a store.  Measured alternatives: 64-row blocks
// in six stages ran 30 % slower (the per-item barriers and store waits
// double), and releasing each stage after its own store 17 % slower.
// Per token:
//   S <- e^g S;  v' = beta (v - S k);  S <- S + v' k^T;  o = S q
// computed as s_k = S_v.k, s_q = S_v.q, v' = beta (v - e^g s_k),
// S_v <- e^g S_v + v' k, o_v = e^g s_q + v' (k.q).  With per-key decays gk
// (the IS_KDA branch, fused_recurrent_fn.py:115-120) the dot products use
// e^gk * k and e^gk * q and the state decays by e^gk per column.
//
// Failures are recorded in the caller's error word (p.err) instead of
// faulting: a bounded stage wait that gives up, or (with p.num_slots) a
// state index past the declared slot count, whose sequence is then skipped
// like a PAD slot.

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "umma.cuh"

namespace gdn {

namespace {

constexpr int kDK = 128;           // key dim handled by this kernel
constexpr int kConsumers = 256;    // 8 consumer warps
constexpr int kThreads = kConsumers + 32;
constexpr int kRows = 128;         // state rows (V) per item: the whole state for V <= 128
constexpr int kStages = 3;         // state blocks per SM (192 KiB)

struct ItemMeta {
  int64_t n, bos, eos, src_row;
  int hv, pad, r0, nr;  // v-head, PAD flag, first state row and row count of the block
  float g0, beta0;  // first token's gate and (head-wise) beta
};

struct StreamSmem {
  static constexpr int kTile = kDK * kRows * 4;      // kRows rows of 128 fp32
  static constexpr int kRow = kDK * 4;               // one q/k/v row, up to fp32 x 128
  static constexpr int kBuf = 0;                     // kStages state tiles
  static constexpr int kQ = kStages * kTile;         // q rows
  static constexpr int kK = kQ + kStages * kRow;     // k rows
  static constexpr int kV = kK + kStages * kRow;     // v rows
  static constexpr int kMeta = kV + kStages * kRow;  // ItemMeta per stage
  static constexpr int kBar = kMeta + kStages * 64;  // full[kStages], empty[kStages]
  static constexpr int kBytes = kBar + 2 * kStages * 8;
};

template <typename T, bool KDA>
__global__ void __launch_bounds__(kThreads, 1)
decode_stream_kernel(const gdn_recurrent_args p, int64_t items) {
  extern __shared__ __align__(128) uint8_t sm[];
  float* tiles = reinterpret_cast<float*>(sm + StreamSmem::kBuf);
  ItemMeta* meta = reinterpret_cast<ItemMeta*>(sm + StreamSmem::kMeta);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + StreamSmem::kBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int V = p.V, HV = p.HV;
  const int es = static_cast<int>(sizeof(T));
  const int nblk = (V + kRows - 1) / kRows;  // blocks per (sequence, v-head)

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      umma::mbar_init(bars + i, 1);            // full: producer arrival + copy bytes
      umma::mbar_init(bars + kStages + i, 1);  // empty: one consumer arrival
    }
    umma::mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumers / 32) {
    // ---------------- producer warp ----------------
    // The 32 lanes look up the next 32 items of this CTA at once (sequence
    // bounds, state slot, first gate and beta: dependent global loads), so
    // that their latency is paid once per 32 items; lane 0 then takes each
    // item's record by shuffles and issues its copies as stages free up.
    const int64_t hb = static_cast<int64_t>(HV) * nblk;
    bool live = true;
    int64_t j = 0;
    for (int64_t base = blockIdx.x; live && base < items; base += 32 * static_cast<int64_t>(gridDim.x)) {
      ItemMeta m{};
      const int64_t item = base + static_cast<int64_t>(lane) * gridDim.x;
      if (item < items) {
        m.n = item / hb;
        const int rem = static_cast<int>(item % hb);
        m.hv = rem / nblk;
        m.r0 = (rem % nblk) * kRows;
        m.nr = min(kRows, V - m.r0);
        seq_bounds(p.cu_seqlens, p.cu_dtype, m.n, p.T, m.bos, m.eos);
        m.src_row = m.bos;
        if (p.initial_state && p.ssm_state_indices) {
          int64_t i0 = 0;
          if (p.num_accepted_tokens) i0 = load_index(p.num_accepted_tokens, p.nacc_dtype, m.n) - 1;
          m.src_row = load_index(p.ssm_state_indices, p.idx_dtype,
                                 m.n * p.stride_indices_seq + i0 * p.stride_indices_tok);
          m.pad = m.src_row < 0;
          if (p.num_slots > 0 && m.src_row >= p.num_slots) {  // skipped like PAD, and reported
            record_device_error(p.err, kErrSlotRange, kSiteSlotInitial, static_cast<int>(m.n),
                                static_cast<int>(m.src_row));
            m.pad = 1;
          }
        }
        m.g0 = (m.eos > m.bos && p.g) ? p.g[m.bos * HV + m.hv] : 0.f;
        m.beta0 = (m.eos > m.bos && !p.beta_per_v) ? p.beta[m.bos * HV + m.hv] : 0.f;
      }
      const int64_t left = (items - base + gridDim.x - 1) / gridDim.x;
      const int cnt = left < 32 ? static_cast<int>(left) : 32;
      for (int l = 0; l < cnt; ++l, ++j) {
        ItemMeta x;
        x.n = __shfl_sync(0xffffffffu, m.n, l);
        x.bos = __shfl_sync(0xffffffffu, m.bos, l);
        x.eos = __shfl_sync(0xffffffffu, m.eos, l);
        x.src_row = __shfl_sync(0xffffffffu, m.src_row, l);
        x.hv = __shfl_sync(0xffffffffu, m.hv, l);
        x.pad = __shfl_sync(0xffffffffu, m.pad, l);
        x.r0 = __shfl_sync(0xffffffffu, m.r0, l);
        x.nr = __shfl_sync(0xffffffffu, m.nr, l);
        x.g0 = __shfl_sync(0xffffffffu, m.g0, l);
        x.beta0 = __shfl_sync(0xffffffffu, m.beta0, l);
        const int st = static_cast<int>(j % kStages);
        const uint32_t ph = static_cast<uint32_t>((j / kStages) & 1);
        bool ok = true;
        if (lane == 0 && j >= kStages) ok = umma::mbar_wait(umma::smem_u32(bars + kStages + st), ph ^ 1u);
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          if (lane == 0) record_device_error(p.err, kErrWaitTimeout, kSiteDecodeRelease, linear_block_id(), tid);
          live = false;
          break;
        }
        if (lane == 0) {
          meta[st] = x;
          const bool work = !x.pad && x.eos > x.bos;
          const uint32_t tile_bytes = static_cast<uint32_t>(x.nr * kDK * 4);
          uint32_t bytes = 0;
          if (work) bytes = (p.initial_state ? tile_bytes : 0u) + static_cast<uint32_t>((2 * kDK + x.nr) * es);
          const uint32_t full = umma::smem_u32(bars + st);
          umma::mbar_arrive_expect_tx(full, bytes);
          if (work) {
            const int h = x.hv / (HV / p.H);
            if (p.initial_state)
              umma::bulk_g2s(sm + StreamSmem::kBuf + st * StreamSmem::kTile,
                             p.initial_state + x.src_row * p.stride_init_state_token +
                                 (static_cast<int64_t>(x.hv) * V + x.r0) * kDK,
                             tile_bytes, full);
            const T* q = static_cast<const T*>(p.q) + (x.bos * p.H + h) * kDK;
            const T* k = static_cast<const T*>(p.k) + (x.bos * p.H + h) * kDK;
            const T* v = static_cast<const T*>(p.v) + (x.bos * HV + x.hv) * V + x.r0;
            umma::bulk_g2s(sm + StreamSmem::kQ + st * StreamSmem::kRow, q, kDK * es, full);
            umma::bulk_g2s(sm + StreamSmem::kK + st * StreamSmem::kRow, k, kDK * es, full);
            umma::bulk_g2s(sm + StreamSmem::kV + st * StreamSmem::kRow, v, x.nr * es, full);
          }
        }
        __syncwarp();
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  T* optr = static_cast<T*>(p.o);
  int pend = -1;  // (tid 0) stage whose state store may still be reading it
  int64_t j = 0;
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x, ++j) {
    const int st = static_cast<int>(j % kStages);
    const uint32_t ph = static_cast<uint32_t>((j / kStages) & 1);
    const bool ok = umma::mbar_wait(umma::smem_u32(bars + st), ph);
    if (!ok && tid == 0) record_device_error(p.err, kErrWaitTimeout, kSiteDecodeLoad, linear_block_id(), tid);
    if (umma::named_sync_or(1, kConsumers, !ok)) break;  // every consumer leaves together
    const ItemMeta m = meta[st];
    float* S = tiles + st * (StreamSmem::kTile / 4);
    const int R = m.nr;  // rows of this block; row r is state row m.r0 + r
    bool stored = false;
    if (m.pad) {  // PAD slot: skip the sequence, clear its outputs
      for (int64_t t = m.bos; t < m.eos; ++t)
        for (int r = tid; r < R; r += kConsumers) optr[(t * HV + m.hv) * V + m.r0 + r] = from_f<T>(0.f);
    } else if (m.eos > m.bos) {
      if (!p.initial_state) {
        for (int e = tid; e < R * kDK / 4; e += kConsumers)
          reinterpret_cast<float4*>(S)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        umma::named_sync(1, kConsumers);
      }
      const int h = m.hv / (HV / p.H);
      const int sub = lane >> 3, li = lane & 7;  // 8 lanes per row; lane li owns float4s li + 8 j
      for (int64_t t = m.bos; t < m.eos; ++t) {
        float4 q[4], k[4], ek[4], kd[4], qd[4];
        const T* vrow;
        const T* qsrc;
        const T* ksrc;
        if (t == m.bos) {
          qsrc = reinterpret_cast<const T*>(sm + StreamSmem::kQ + st * StreamSmem::kRow);
          ksrc = reinterpret_cast<const T*>(sm + StreamSmem::kK + st * StreamSmem::kRow);
          vrow = reinterpret_cast<const T*>(sm + StreamSmem::kV + st * StreamSmem::kRow);
        } else {
          qsrc = static_cast<const T*>(p.q) + (t * p.H + h) * kDK;
          ksrc = static_cast<const T*>(p.k) + (t * p.H + h) * kDK;
          vrow = static_cast<const T*>(p.v) + (t * HV + m.hv) * V + m.r0;
        }
        float qq = 0.f, kk = 0.f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          q[jj] = load4<T>(qsrc + (li + 8 * jj) * 4);
          k[jj] = load4<T>(ksrc + (li + 8 * jj) * 4);
          qq += q[jj].x * q[jj].x + q[jj].y * q[jj].y + q[jj].z * q[jj].z + q[jj].w * q[jj].w;
          kk += k[jj].x * k[jj].x + k[jj].y * k[jj].y + k[jj].z * k[jj].z + k[jj].w * k[jj].w;
        }
        const float rq = p.use_qk_l2norm ? 1.f / sqrtf(group_sum<8>(qq) + 1e-6f) : 1.f;
        const float rk = p.use_qk_l2norm ? 1.f / sqrtf(group_sum<8>(kk) + 1e-6f) : 1.f;
        float kq = 0.f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float a = rq * p.scale;
          q[jj].x *= a; q[jj].y *= a; q[jj].z *= a; q[jj].w *= a;
          k[jj].x *= rk; k[jj].y *= rk; k[jj].z *= rk; k[jj].w *= rk;
          kq += k[jj].x * q[jj].x + k[jj].y * q[jj].y + k[jj].z * q[jj].z + k[jj].w * q[jj].w;
        }
        kq = group_sum<8>(kq);
        if constexpr (KDA) {  // per-key decay: dot products against e^gk * k, e^gk * q
          const float* gkr = p.gk + (t * HV + m.hv) * kDK;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float4 x = *reinterpret_cast<const float4*>(gkr + (li + 8 * jj) * 4);
            ek[jj] = make_float4(expf(x.x), expf(x.y), expf(x.z), expf(x.w));
            kd[jj] = make_float4(ek[jj].x * k[jj].x, ek[jj].y * k[jj].y, ek[jj].z * k[jj].z, ek[jj].w * k[jj].w);
            qd[jj] = make_float4(ek[jj].x * q[jj].x, ek[jj].y * q[jj].y, ek[jj].z * q[jj].z, ek[jj].w * q[jj].w);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) { kd[jj] = k[jj]; qd[jj] = q[jj]; }
        }
        // destination row of this token's state, loaded before the math so that its latency overlaps
        int64_t frow = !p.final_state ? -1
                       : p.inplace_final_state
                           ? load_index(p.ssm_state_indices, p.idx_dtype,
                                        m.n * p.stride_indices_seq + (t - m.bos) * p.stride_indices_tok)
                           : t;
        if (p.inplace_final_state && p.num_slots > 0 && frow >= p.num_slots) {
          if (tid == 0)
            record_device_error(p.err, kErrSlotRange, kSiteSlotFinal, static_cast<int>(m.n), static_cast<int>(frow));
          frow = -1;
        }
        const float eg = !p.g ? 1.f : expf(t == m.bos ? m.g0 : p.g[t * HV + m.hv]);
        const float beta_h = p.beta_per_v ? 0.f : (t == m.bos ? m.beta0 : p.beta[t * HV + m.hv]);
        // a warp covers 4 rows per pass; two passes (8 rows) are reduced together
        for (int r0 = warp * 4; r0 < R; r0 += 8 * (kConsumers / 32)) {
          float4 sv[2][4];
          float red[4];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int r = r0 + u * 4 * (kConsumers / 32) + sub;
            float dk = 0.f, dq = 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              sv[u][jj] = r < R ? reinterpret_cast<const float4*>(S + r * kDK)[li + 8 * jj]
                                : make_float4(0.f, 0.f, 0.f, 0.f);
              dk += sv[u][jj].x * kd[jj].x + sv[u][jj].y * kd[jj].y + sv[u][jj].z * kd[jj].z + sv[u][jj].w * kd[jj].w;
              dq += sv[u][jj].x * qd[jj].x + sv[u][jj].y * qd[jj].y + sv[u][jj].z * qd[jj].z + sv[u][jj].w * qd[jj].w;
            }
            red[2 * u] = dk;
            red[2 * u + 1] = dq;
          }
#pragma unroll
          for (int o = 4; o > 0; o >>= 1)
#pragma unroll
            for (int e = 0; e < 4; ++e) red[e] += __shfl_xor_sync(0xffffffffu, red[e], o);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int r = r0 + u * 4 * (kConsumers / 32) + sub;
            if (r >= R) continue;
            const float br = p.beta_per_v ? p.beta[(t * HV + m.hv) * V + m.r0 + r] : beta_h;
            const float vp = br * (to_f<T>(vrow[r]) - eg * red[2 * u]);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              float4 s4 = sv[u][jj];
              if constexpr (KDA) { s4.x *= ek[jj].x; s4.y *= ek[jj].y; s4.z *= ek[jj].z; s4.w *= ek[jj].w; }
              s4.x = eg * s4.x + vp * k[jj].x;
              s4.y = eg * s4.y + vp * k[jj].y;
              s4.z = eg * s4.z + vp * k[jj].z;
              s4.w = eg * s4.w + vp * k[jj].w;
              reinterpret_cast<float4*>(S + r * kDK)[li + 8 * jj] = s4;
            }
            if (li == 0) optr[(t * HV + m.hv) * V + m.r0 + r] = from_f<T>(eg * red[2 * u + 1] + vp * kq);
          }
        }
        if (p.final_state) {
          umma::fence_proxy_async();
          umma::named_sync(1, kConsumers);
          if (tid == 0 && frow >= 0) {
            umma::bulk_s2g(p.final_state + frow * p.stride_final_state_token +
                               (static_cast<int64_t>(m.hv) * V + m.r0) * kDK,
                           S, static_cast<uint32_t>(R * kDK * 4));
            umma::bulk_commit();
            stored = true;
          }
          if (t + 1 < m.eos) {  // the next token rewrites the tile: let the store read it first
            if (tid == 0 && stored) umma::bulk_wait_read_all();
            umma::named_sync(1, kConsumers);
          }
        }
      }
    }
    umma::named_sync(1, kConsumers);  // every consumer is done with stage st
    if (tid == 0) {
      // A stage whose block is being stored stays held until the next item
      // ends, so the consumers never wait for a store to read shared memory;
      // the previous item's stage is released once its (older) store has.
      if (stored) {
        umma::bulk_wait_read_all_but_one();
        if (pend >= 0) umma::mbar_arrive(umma::smem_u32(bars + kStages + pend));
        pend = st;
      } else {
        if (pend >= 0) {
          umma::bulk_wait_read_all();
          umma::mbar_arrive(umma::smem_u32(bars + kStages + pend));
        }
        umma::mbar_arrive(umma::smem_u32(bars + kStages + st));
        pend = -1;
      }
    }
  }
  if (tid == 0) umma::bulk_wait_all();
}

template <typename T, bool KDA>
cudaError_t launch_stream_kda(const gdn_recurrent_args& a, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  auto kern = decode_stream_kernel<T, KDA>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                StreamSmem::kBytes)) != cudaSuccess)
    return e;
  const int64_t items = a.N * a.HV * ((a.V + kRows - 1) / kRows);
  const unsigned grid = static_cast<unsigned>(items < sms ? items : sms);
  note_launch();
  kern<<<grid, kThreads, StreamSmem::kBytes, s>>>(a, items);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_stream_t(const gdn_recurrent_args& a, cudaStream_t s) {
  return a.gk ? launch_stream_kda<T, true>(a, s) : launch_stream_kda<T, false>(a, s);
}

}  // namespace

// The streaming kernel needs 16-byte aligned rows for its bulk copies.
bool decode_stream_applies(const gdn_recurrent_args& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int es = a.qkv_dtype == GDN_F32 ? 4 : 2;
  return a.K == kDK && a.V <= 128 && (a.V * es) % 16 == 0 && al(a.q) && al(a.k) && al(a.v) && al(a.gk) &&
         (!a.initial_state || (al(a.initial_state) && a.stride_init_state_token % 4 == 0)) &&
         (!a.final_state || (al(a.final_state) && a.stride_final_state_token % 4 == 0));
}

cudaError_t launch_decode_stream(const gdn_recurrent_args& a, cudaStream_t s) {
  switch (a.qkv_dtype) {
    case GDN_F32: return launch_stream_t<float>(a, s);
    case GDN_BF16: return launch_stream_t<__nv_bfloat16>(a, s);
    case GDN_F16: return launch_stream_t<__half>(a, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
