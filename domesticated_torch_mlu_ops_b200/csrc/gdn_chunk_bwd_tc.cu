// Tensor-core (tcgen05) state-gradient recurrence of the GDN backward for
// bf16/fp16 inputs with K = V = 128: chunk_gated_delta_rule_bwd_dhu
// (triton/fla/chunk_delta_h.py:273-581, called from chunk.py:76-186).
//
// Per (sequence, v-head, 32-column V-slice), over the chunks in reverse,
// with dh' the gradient of the state after the chunk (fp32, registers):
//   X   = [K; Q] dh~                         (tcgen05, M = 128; rows 0..63 used)
//   dv  = dv_local + diag(b) X               (b_i = exp(G_L - G_i) r_k,i; rows past the end: 0)
//   dH  = Q^T diag(a) dO + W^T (-dv)         (tcgen05, M = 128, two products in one accumulator)
//   dh  = gamma dh' + dH
// where dh~ is dh' rounded to the input dtype, a_i = scale exp(G_i) r_q,i and
// gamma = exp(G_L): the row scales the forward WY kernel writes, whose W
// images (L2 norm and gates folded in) this kernel reads.  q, k, dO and
// dv_local come in by TMA.  Every chunk stores dv and dh' as bf16 operand
// images for the remaining backward kernels; dh at the first chunk is dh0.  The bf16 roundings are the
// reference's: dh and dv are cast to the input dtype before their products.
//
// Warp roles as in the forward state kernel: warp 0 issues the MMAs, warps
// 0,1,4,5 form dv (rows 0..63), warps 2,3,6,7 build the diag(a) dO image
// while the first product runs, all eight update dh, and a ninth warp
// streams the chunks ahead into three stages.  Every wait is bounded; on a
// timeout the kernel records an error, drains its copies and MMAs (bounded)
// and exits.

#include <cuda.h>

#include <type_traits>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_chunk_tc.cuh"
#include "solve_tril.cuh"
#include "umma.cuh"

namespace gdn {
namespace tc {

namespace {

struct BwdSt {
  static constexpr int VS = 32;
  // stage: K a0 | Q a0 | K a1 | Q a1 | W a0 | W a1 | dO [64][VS] | dv_local [64][VS] fp32 | scalars
  static constexpr int kKQ = 0;
  static constexpr int kW = 4 * kAtom;
  static constexpr int kDO = kW + 2 * kAtom;
  static constexpr int kDvl = kDO + 64 * VS * 2;
  static constexpr int kSc = kDvl + 64 * VS * 4;
  static constexpr int kStage = ((kSc + kScal * 4 + 1023) / 1024) * 1024;
  static constexpr uint32_t kTx = 6 * kAtom + 64 * VS * 2 + 64 * VS * 4 + kScal * 4;
  static constexpr int kStages = 3;
  static constexpr int kH = kStages * kStage;       // dh~ image 128 x VS
  static constexpr int kDo = kH + D * VS * 2;       // diag(a) dO image 64 x VS
  static constexpr int kMdv = kDo + 64 * VS * 2;    // -dv image 64 x VS
  static constexpr int kBar = kMdv + 64 * VS * 2;   // full[kStages], mma1, mma2
  static constexpr int kTmem = kBar + (kStages + 2) * 8;
  static constexpr int kBytes = kTmem + 8 + 1024;
  static constexpr int kAcc = 0, kDH = VS, kCols = 64;  // TMEM columns
  static_assert(kDO % 128 == 0 && kDvl % 128 == 0, "TMA destinations");
  static_assert(kBytes <= 227 * 1024, "shared memory");
};

struct BwdOut {
  uint8_t* dv_img;  // [chunks][HV] bf16 images of dv (bwd_img_off, 64 rows)
  uint8_t* dh_img;  // [chunks][HV] bf16 images of dh' (bwd_img_off, 128 rows)
};

template <typename T>
__global__ void __launch_bounds__(kSt3Threads, 1)
tc_bwd_state_kernel(const gdn_chunk_bwd_args p, const Work w, const BwdOut o,
                    const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tdo, const __grid_constant__ CUtensorMap tdv) {
  using S = BwdSt;
  constexpr int VS = S::VS;
  constexpr int RSV = (VS / 8) * 128;
  constexpr int CW = VS / 2;  // columns per thread
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* himg = sm + S::kH;
  uint8_t* doimg = sm + S::kDo;
  uint8_t* mdvimg = sm + S::kMdv;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::kTmem);
  const uint32_t bar_mma1 = umma::smem_u32(bars + S::kStages), bar_mma2 = umma::smem_u32(bars + S::kStages + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool producer = warp == 8;
  const int quad = warp & 3, colh = (warp >> 2) & 1;
  const int row = quad * 32 + lane;
  constexpr int kSlices = D / VS;  // block = (sequence * HV + v-head) * slices + slice
  const int64_t chain = blockIdx.x / kSlices;
  const int64_t n = chain / p.HV;
  const int hv = static_cast<int>(chain - n * p.HV), h = hv / (p.HV / p.H);
  const int v0 = static_cast<int>(blockIdx.x % kSlices) * VS;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int nch = static_cast<int>(eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0);
  const int64_t c0 = w.coff[n];
  // iteration j works on chunk nch - 1 - j
  auto stage = [&](int j) { return sm + (j % S::kStages) * S::kStage; };
  auto full = [&](int j) { return umma::smem_u32(bars + j % S::kStages); };
  const long long wlim = 2000000000LL;
  int fetched[S::kStages];
#pragma unroll
  for (int i = 0; i < S::kStages; ++i) fetched[i] = -1;

  auto fetch = [&](int j) {  // one thread
    fetched[j % S::kStages] = j;
    const int c = nch - 1 - j;
    uint8_t* b = stage(j);
    const uint32_t bar = full(j);
    const int s = static_cast<int>(bos + static_cast<int64_t>(c) * kChunk);
    const int64_t hc = static_cast<int64_t>(hv) * w.ncu + c0 + c;
    const uint8_t* wsrc = w.wimg + hc * kImg64x128;
    umma::mbar_arrive_expect_tx(bar, S::kTx);
    umma::tma_load_3d(b + S::kKQ, &tk, 0, h, s, bar);
    umma::tma_load_3d(b + S::kKQ + kAtom, &tq, 0, h, s, bar);
    umma::tma_load_3d(b + S::kKQ + 2 * kAtom, &tk, 64, h, s, bar);
    umma::tma_load_3d(b + S::kKQ + 3 * kAtom, &tq, 64, h, s, bar);
    umma::bulk_g2s(b + S::kW, wsrc, kAtom, bar);
    umma::bulk_g2s(b + S::kW + kAtom, wsrc + kAtom, kAtom, bar);
    umma::tma_load_3d(b + S::kDO, &tdo, v0, hv, s, bar);
    umma::tma_load_3d(b + S::kDvl, &tdv, v0, hv, s, bar);
    umma::bulk_g2s(b + S::kSc, w.scal + hc * kScal, kScal * 4, bar);
  };

  if (tid == 256) {
    for (int i = 0; i < S::kStages + 2; ++i) umma::mbar_init(bars + i, 1);
    umma::mbar_fence_init();
    for (int j = 0; j < S::kStages - 1 && j < nch; ++j) fetch(j);
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, S::kCols);
    umma::fence_before_sync();
  }
  // dh' slice: thread `row` owns dh[row][v0 + colh*CW .. +CW] in fp32
  float hreg[CW];
  if (!producer) {
    const int64_t base = (n * p.HV + hv) * D * D;
#pragma unroll
    for (int jj = 0; jj < CW; ++jj) {
      const int col = v0 + colh * CW + jj;
      hreg[jj] = !p.dht ? 0.f
                 : p.state_v_first ? p.dht[base + static_cast<int64_t>(col) * D + row]
                                   : p.dht[base + static_cast<int64_t>(row) * D + col];
    }
#pragma unroll
    for (int j8 = 0; j8 < CW / 8; ++j8)
      *reinterpret_cast<uint4*>(himg + umma::img_off(row, colh * CW + j8 * 8, RSV)) = pack8<T>(hreg + j8 * 8);
  }
  umma::fence_proxy_async();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t t_acc = tmem + S::kAcc, t_dh = tmem + S::kDH;
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  const uint32_t id_x = umma::idesc_f16(128, VS, kBf16, false, true);   // A K-major, B MN-major
  const uint32_t id_dh = umma::idesc_f16(128, VS, kBf16, true, true);   // A MN-major (transposed tiles)
  const uint64_t d_h = umma::smem_desc(umma::smem_u32(himg), RSV, 128);
  const uint64_t d_do = umma::smem_desc(umma::smem_u32(doimg), RSV, 128);
  const uint64_t d_mdv = umma::smem_desc(umma::smem_u32(mdvimg), RSV, 128);
  const int64_t rowV = static_cast<int64_t>(p.HV) * D;

  bool ok = true, mine = true;
  uint32_t last_bar = 0, last_par = 0;
  if (producer && nch > 0) {
    mine = umma::mbar_wait(full(0), 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStLoad);
  }
  for (int j = 0; j < nch; ++j) {
    if (__syncthreads_or(!mine)) { ok = false; break; }
    umma::fence_after_sync();
    const int c = nch - 1 - j;
    const int64_t s = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    uint8_t* b = stage(j);
    const float* sc = reinterpret_cast<const float*>(b + S::kSc);
    if (warp == 0) {  // MMA1: X = [K; Q] dh~
      if (umma::elect_one()) {
        const uint64_t da = umma::smem_desc_sw128(umma::smem_u32(b + S::kKQ), 16, 1024);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          umma::mma_f16(t_acc, da + (((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4), d_h + ((ks * 2 * RSV) >> 4),
                        id_x, ks > 0);
        umma::mma_commit(bar_mma1);
      }
      __syncwarp();
      last_bar = bar_mma1;
      last_par = static_cast<uint32_t>(j & 1);
    }
    if (producer) {
      // iteration j + kStages - 1 goes where iteration j - 1 was: its products must be done
      if (j >= 1) {
        mine = umma::mbar_wait(bar_mma2, static_cast<uint32_t>((j - 1) & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStMma2);
      }
      if (mine && j + S::kStages - 1 < nch && lane == 0) fetch(j + S::kStages - 1);
      __syncwarp();
      if (mine && j + 1 < nch) {
        mine = umma::mbar_wait(full(j + 1), static_cast<uint32_t>(((j + 1) / S::kStages) & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStLoad);
      }
      continue;
    }
    if (quad >= 2) {  // diag(a) dO image (rows 0..63), off the chain
      const int i = row - 64;
      const float ai = sc[i];  // zero past the sequence end
      const T* dor = reinterpret_cast<const T*>(b + S::kDO) + i * VS + colh * CW;
#pragma unroll
      for (int j8 = 0; j8 < CW / 8; ++j8) {
        float x[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(dor + j8 * 8), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] *= ai;
        *reinterpret_cast<uint4*>(doimg + umma::img_off(i, colh * CW + j8 * 8, RSV)) = pack8<T>(x);
      }
    } else {  // dv (rows 0..63)
      const int i = row;
      const float bi = sc[64 + i];
      const float* dl = reinterpret_cast<const float*>(b + S::kDvl) + i * VS + colh * CW;
      float dv[CW];
#pragma unroll
      for (int j4 = 0; j4 < CW / 4; ++j4) {
        const float4 v4 = *reinterpret_cast<const float4*>(dl + j4 * 4);
        dv[j4 * 4] = v4.x;
        dv[j4 * 4 + 1] = v4.y;
        dv[j4 * 4 + 2] = v4.z;
        dv[j4 * 4 + 3] = v4.w;
      }
      mine = umma::mbar_wait(bar_mma1, static_cast<uint32_t>(j & 1), wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma1);
      umma::fence_after_sync();
      uint32_t rx[CW];
#pragma unroll
      for (int q = 0; q < CW / 16; ++q) umma::tmem_ld16_nw(t_acc + lane_base + colh * CW + q * 16, rx + q * 16);
      umma::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < CW / 16; ++q) umma::reg_fence16(rx + q * 16);
      const bool live = i < L;
#pragma unroll
      for (int e = 0; e < CW; ++e) dv[e] = live ? fmaf(bi, __uint_as_float(rx[e]), dv[e]) : 0.f;
#pragma unroll
      for (int j8 = 0; j8 < CW / 8; ++j8) {
        float m[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) m[e] = -dv[j8 * 8 + e];
        *reinterpret_cast<uint4*>(mdvimg + umma::img_off(i, colh * CW + j8 * 8, RSV)) = pack8<T>(m);
      }
      {  // every row, so that the image holds no stale values (rows past the end are zeros)
        uint8_t* dst = o.dv_img + ((c0 + c) * p.HV + hv) * static_cast<int64_t>(kVnImg);
#pragma unroll
        for (int j8 = 0; j8 < CW / 8; ++j8)
          *reinterpret_cast<uint4*>(dst + bwd_img_off(i, v0 + colh * CW + j8 * 8, 64)) = pack8<T>(dv + j8 * 8);
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    umma::named_sync(1, 256);  // both images are in place
    if (warp == 0) {  // MMA2: dH = Q^T diag(a) dO + W^T (-dv)
      umma::fence_after_sync();
      if (umma::elect_one()) {
        const uint64_t dq = umma::smem_desc_sw128(umma::smem_u32(b + S::kKQ + kAtom), 2 * kAtom, 1024);
#pragma unroll
        for (int ks = 0; ks < 64 / 16; ++ks)
          umma::mma_f16(t_dh, dq + ((ks * 2048) >> 4), d_do + ((ks * 2 * RSV) >> 4), id_dh, ks > 0);
        const uint64_t dw = umma::smem_desc_sw128(umma::smem_u32(b + S::kW), kAtom, 1024);
#pragma unroll
        for (int ks = 0; ks < 64 / 16; ++ks)
          umma::mma_f16(t_dh, dw + ((ks * 2048) >> 4), d_mdv + ((ks * 2 * RSV) >> 4), id_dh, true);
        umma::mma_commit(bar_mma2);
      }
      __syncwarp();
      last_bar = bar_mma2;
      last_par = static_cast<uint32_t>(j & 1);
    }
    // dh <- gamma dh' + dH (rows 0..127), its image for the next chunk, and dh' out
    if (mine) {
      mine = umma::mbar_wait(bar_mma2, static_cast<uint32_t>(j & 1), wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma2);
    }
    umma::fence_after_sync();
    if (mine) {
      float d[CW];
#pragma unroll
      for (int q = 0; q < CW / 16; ++q) umma::tmem_ld16(t_dh + lane_base + colh * CW + q * 16, d + q * 16);
      const float g = sc[128];
#pragma unroll
      for (int e = 0; e < CW; ++e) d[e] = fmaf(g, hreg[e], d[e]);
      if (j + 1 < nch) {
#pragma unroll
        for (int j8 = 0; j8 < CW / 8; ++j8)
          *reinterpret_cast<uint4*>(himg + umma::img_off(row, colh * CW + j8 * 8, RSV)) = pack8<T>(d + j8 * 8);
      }
      uint8_t* dst = o.dh_img + ((c0 + c) * p.HV + hv) * static_cast<int64_t>(kStateImg);
#pragma unroll
      for (int j8 = 0; j8 < CW / 8; ++j8)
        *reinterpret_cast<uint4*>(dst + bwd_img_off(row, v0 + colh * CW + j8 * 8, 128)) = pack8<T>(hreg + j8 * 8);
#pragma unroll
      for (int e = 0; e < CW; ++e) hreg[e] = d[e];
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
  }
  if (ok) ok = !__syncthreads_or(!mine);
  if (ok && !producer && p.dh0) {
    const int64_t base = (n * p.HV + hv) * D * D;
#pragma unroll
    for (int jj = 0; jj < CW; ++jj) {
      const int col = v0 + colh * CW + jj;
      if (p.state_v_first) p.dh0[base + static_cast<int64_t>(col) * D + row] = hreg[jj];
      else p.dh0[base + static_cast<int64_t>(row) * D + col] = hreg[jj];
    }
  }
  if (!ok) {  // drain (bounded) this CTA's copies and products before its memory is released
    const long long drain = 20000000LL;
    if (tid == 256)
      for (int x = 0; x < S::kStages; ++x)
        if (fetched[x] >= 0)
          umma::mbar_wait(full(fetched[x]), static_cast<uint32_t>((fetched[x] / S::kStages) & 1), drain);
    if (warp == 0 && last_bar) umma::mbar_wait(last_bar, last_par, drain);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, S::kCols);
}

// ---------------------------------------------------------------------------
// dq, dk, dW and dG per (chunk, v-head): chunk_bwd_dqkwg (chunk_o.py:233-778)
// ---------------------------------------------------------------------------
// With s = scale, Gam_i = exp(G_i), c_i = exp(G_L - G_i) and r_q, r_k the L2
// norm factors (q^ = diag(r_q) q, k^ = diag(r_k) k):
//   S   = [dO; v_new] v_new^T                     rows 0..63 used
//   dP  = s M * exp(G_i - G_j) * S                 (M: j <= i < L)
//   X_h = [s Gam dO; dv] h~^T                      rows 0..63: dq part, rows 64..127: -dW
//   X_q = [dP diag(r_k); 0] K                      dq = X_h + X_q (rows 0..63)
//   X_k = [diag(r_q) dP; 0]^T Q                    dk = X_k + diag(c) X_v (rows 0..63 / 64..127)
//   X_v = [dO; v_new] dh~'^T                       rows 64..127 used
//   dG_i = r_q,i q_i.dq_i - r_k,i k_i.dk_i, and on the last row also
//          gamma <dh~', h~> + sum_i r_k,i k_i.(diag(c) X_v)_i
// All products on tcgen05 (M = 128, accumulators in TMEM); q, k and dO come
// in by TMA, h~, dh~' and v_new as the bf16 images the state kernels wrote,
// dv as the bf16 image the state-gradient kernel wrote; dW leaves as a bf16
// image for the WY-form gradient kernel.  One CTA per (chunk, v-head), one per SM.

struct DqSm {
  static constexpr int kQ = 0;                  // Q a0 | Q a1
  static constexpr int kK = kQ + 2 * kAtom;     // K a0 | K a1
  static constexpr int kDV = kK + 2 * kAtom;    // dO a0 | v_new a0 | dO a1 | v_new a1
  static constexpr int kH = kDV + 4 * kAtom;    // h~ (two 128-row atoms)
  static constexpr int kDH = kH + kStateImg;    // dh~'
  static constexpr int kA1 = kDH + kStateImg;   // [s Gam dO; dv]; later diag(c) X_v rows (fp32 [64][128])
  static constexpr int kPk = kA1 + kStateImg;   // dP diag(r_k) atom | zero atom
  static constexpr int kPq = kPk + 2 * kAtom;   // diag(r_q) dP atom | zero atom
  static constexpr int kVec = kPq + 2 * kAtom;  // G, r_q, r_k, half-row dG [64] each; reduction [8]
  static constexpr int kBar = kVec + (4 * 64 + 8) * 4;
  static constexpr int kTmem = kBar + 4 * 8;    // mbarriers: loads, S, first products, second products
  static constexpr int kBytes = kTmem + 8 + 1024;
  static constexpr uint32_t kTx = 6 * kAtom + 2 * kVnImg + 2 * kStateImg;  // q, k, dO, v_new, dv, h, dh'
  static constexpr int kThreads = 256;
  // TMEM columns: X_h 0-127, S then X_q 128-255, X_v 256-383, X_k 384-511
  static constexpr uint32_t kXh = 0, kS = 128, kXq = 128, kXv = 256, kXk = 384;
  static_assert(kBytes <= 227 * 1024, "shared memory");
  static_assert(64 * 128 * 4 <= kStateImg, "the dK2 rows fit over the first product's A image");
};

__device__ __forceinline__ float dq_block_sum(float x, float* red) {
  x = group_sum<32>(x);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < DqSm::kThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

template <typename T>
__global__ void __launch_bounds__(DqSm::kThreads, 1)
tc_bwd_dqkw_kernel(const gdn_chunk_bwd_args p, const Work w, const DqkwOut o, float scale,
                   const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tdo) {
  using S = DqSm;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  float* Gs = reinterpret_cast<float*>(sm + S::kVec);
  float* rq = Gs + 64;
  float* rk = rq + 64;
  float* dgh = rk + 64;
  float* red = dgh + 64;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::kTmem);
  const uint32_t bar_ld = umma::smem_u32(bars), bar_s = umma::smem_u32(bars + 1), bar_a = umma::smem_u32(bars + 2),
                 bar_b = umma::smem_u32(bars + 3);
  int64_t n, lc;
  const int64_t cix = blockIdx.x / static_cast<unsigned>(p.HV);  // chunk-major, the v-heads of a chunk adjacent
  if (!locate_chunk(w.coff, p.N, cix, n, lc)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, colh = warp >> 2, row = quad * 32 + lane;
  const bool rows_lo = quad < 2;  // TMEM lanes 0..63
  const int hv = static_cast<int>(blockIdx.x - cix * p.HV), h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t img = cix * p.HV + hv;  // cix = the chunk's global index
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  const long long wlim = 2000000000LL;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) umma::mbar_init(bars + i, 1);
    umma::mbar_fence_init();
    umma::mbar_arrive_expect_tx(bar_ld, S::kTx);
    umma::tma_load_3d(sm + S::kQ, &tq, 0, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kQ + kAtom, &tq, 64, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kK, &tk, 0, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kK + kAtom, &tk, 64, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kDV, &tdo, 0, hv, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kDV + 2 * kAtom, &tdo, 64, hv, static_cast<int>(s), bar_ld);
    const uint8_t* vn = o.vn_img + img * kVnImg;
    umma::bulk_g2s(sm + S::kDV + kAtom, vn, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kDV + 3 * kAtom, vn + kAtom, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kH, o.hs_img + img * kStateImg, kStateImg, bar_ld);
    umma::bulk_g2s(sm + S::kDH, o.dh_img + img * kStateImg, kStateImg, bar_ld);
    // dv into rows 64..127 of the X_h operand (same swizzle phase as rows 0..63 of the image)
    const uint8_t* dv = o.dv_img + img * kVnImg;
    umma::bulk_g2s(sm + S::kA1 + 64 * 128, dv, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kA1 + kStateImg / 2 + 64 * 128, dv + kAtom, kAtom, bar_ld);
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, 512);
    umma::fence_before_sync();
  }
  for (int e = tid; e < kAtom / 16; e += S::kThreads) {
    reinterpret_cast<uint4*>(sm + S::kPk + kAtom)[e] = make_uint4(0u, 0u, 0u, 0u);
    reinterpret_cast<uint4*>(sm + S::kPq + kAtom)[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (tid < 64) Gs[tid] = tid < L ? o.gc[(s + tid) * p.HV + hv] * kLog2e : 0.f;  // G in the log2 domain
  const int di = tid >> 2;
  umma::fence_proxy_async();  // the zero atoms are tcgen05 operands
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  bool mine = umma::mbar_wait(bar_ld, 0, wlim);
  if (!mine) record_error(w.err, 1, kSiteStLoad);
  bool ok = !__syncthreads_or(!mine);  // uniform
  uint32_t last_bar = 0;

  if (ok) {
    {  // L2-norm factors of the q and k rows: two threads per row, one atom each
      const int r = tid >> 1, half = tid & 1, i = r & 63;
      const uint8_t* at = sm + (r < 64 ? S::kQ : S::kK) + half * kAtom + i * 128;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float x[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(at + c * 16), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      if (half == 0) (r < 64 ? rq : rk)[i] = p.use_qk_l2norm ? rsqrtf(ss + 1e-6f) : 1.f;
    }
    {  // A operand of X_h: rows 0..63 s Gam dO (same swizzle as the dO atoms); rows 64..127 hold dv
      const int i = di;
      const float f = i < L ? scale * exp2f(Gs[i]) : 0.f;
      const int atom = (tid & 3) >> 1;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pc = (tid & 1) * 4 + u;
        float x[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kDV + atom * 2 * kAtom + i * 128 + pc * 16), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] *= f;
        *reinterpret_cast<uint4*>(sm + S::kA1 + atom * (kStateImg / 2) + i * 128 + pc * 16) = pack8<T>(x);
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    auto adv = [](int ks) { return static_cast<uint64_t>(((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4); };
    if (warp == 0) {  // S, then X_h and X_v
      umma::fence_after_sync();
      if (umma::elect_one()) {
        const uint32_t id64 = umma::idesc_f16(128, 64, kBf16, false, false);
        const uint32_t id128 = umma::idesc_f16(128, 128, kBf16, false, false);
        const uint64_t d_dv = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDV), 16, 1024);
        const uint64_t d_vn = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDV + kAtom), 16, 1024);
        const uint64_t d_a1 = umma::smem_desc_sw128(umma::smem_u32(sm + S::kA1), 16, 1024);
        const uint64_t d_h = umma::smem_desc_sw128(umma::smem_u32(sm + S::kH), 16, 1024);
        const uint64_t d_dh = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDH), 16, 1024);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) umma::mma_f16(tmem + S::kS, d_dv + adv(ks), d_vn + adv(ks), id64, ks > 0);
        umma::mma_commit(bar_s);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) umma::mma_f16(tmem + S::kXh, d_a1 + adv(ks), d_h + adv(ks), id128, ks > 0);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) umma::mma_f16(tmem + S::kXv, d_dv + adv(ks), d_dh + adv(ks), id128, ks > 0);
        umma::mma_commit(bar_a);
      }
      __syncwarp();
      last_bar = bar_a;
    }
    if (rows_lo) {  // dP images from S (rows 0..63, 32 columns per thread)
      mine = umma::mbar_wait(bar_s, 0, wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma1);
      umma::fence_after_sync();
      if (mine) {
        float sv[32];
        umma::tmem_ld32(tmem + S::kS + lane_base + colh * 32, sv);
        const int i = row;
        const float gi = Gs[i], rqi = rq[i];
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float pk[8], pq[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = colh * 32 + q8 * 8 + e;
            const float v = (i < L && j <= i) ? scale * exp2f(gi - Gs[j]) * sv[q8 * 8 + e] : 0.f;
            pk[e] = v * rk[j];
            pq[e] = v * rqi;
          }
          const int j0 = colh * 32 + q8 * 8;
          const uint32_t off = i * 128 + ((((j0 >> 3) ^ (i & 7))) << 4);
          *reinterpret_cast<uint4*>(sm + S::kPk + off) = pack8<T>(pk);
          *reinterpret_cast<uint4*>(sm + S::kPq + off) = pack8<T>(pq);
        }
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    ok = !__syncthreads_or(!mine);
  }
  if (ok && warp == 0) {  // X_q and X_k
    umma::fence_after_sync();
    if (umma::elect_one()) {
      const uint32_t idq = umma::idesc_f16(128, 128, kBf16, false, true);
      const uint32_t idk = umma::idesc_f16(128, 128, kBf16, true, true);
      const uint64_t d_pk = umma::smem_desc_sw128(umma::smem_u32(sm + S::kPk), 16, 1024);
      const uint64_t d_pq = umma::smem_desc_sw128(umma::smem_u32(sm + S::kPq), kAtom, 1024);
      const uint64_t d_k = umma::smem_desc_sw128(umma::smem_u32(sm + S::kK), kAtom, 1024);
      const uint64_t d_q = umma::smem_desc_sw128(umma::smem_u32(sm + S::kQ), kAtom, 1024);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem + S::kXq, d_pk + ((ks * 32) >> 4), d_k + ((ks * 2048) >> 4), idq, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem + S::kXk, d_pq + ((ks * 2048) >> 4), d_q + ((ks * 2048) >> 4), idk, ks > 0);
      umma::mma_commit(bar_b);
    }
    __syncwarp();
    last_bar = bar_b;
  }
  float esum = 0.f, hp = 0.f;
  if (ok) {
    if (!rows_lo) {  // rows 64..127: dW (image), and diag(c) X_v into shared memory (over the consumed A image)
      mine = umma::mbar_wait(bar_a, 0, wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma2);
      umma::fence_after_sync();
      if (mine) {
        const int i = row - 64;
        const bool live = i < L;
        const float ci = live ? exp2f(Gs[L - 1] - Gs[i]) : 0.f;
        float4* dk2 = reinterpret_cast<float4*>(sm + S::kA1) + i * 32;
        uint8_t* dwimg = o.dw_img + img * kVnImg;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int c0 = colh * 64 + half * 32;
          float x[32];
          umma::tmem_ld32(tmem + S::kXh + lane_base + c0, x);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {  // every row (zeros past the end): dW = -dv h~^T
            float m[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) m[e] = -x[q8 * 8 + e];
            *reinterpret_cast<uint4*>(dwimg + bwd_img_off(i, c0 + q8 * 8, 64)) = pack8<T>(m);
          }
          umma::tmem_ld32(tmem + S::kXv + lane_base + c0, x);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            const int col = c0 + q8 * 8;
            float kv[8];
            unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kK + (col >> 6) * kAtom + i * 128 +
                                                       ((((col & 63) >> 3) ^ (i & 7)) << 4)), kv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              x[q8 * 8 + e] *= ci;
              esum = fmaf(kv[e], x[q8 * 8 + e], esum);
            }
          }
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            dk2[((c0 >> 2) + j4) ^ (i & 31)] = make_float4(x[j4 * 4], x[j4 * 4 + 1], x[j4 * 4 + 2], x[j4 * 4 + 3]);
        }
        esum *= rk[i];
      }
    }
    // <dh~', h~> over the two images (same layout)
    for (int e = tid; e < kStateImg / 16; e += S::kThreads) {
      float a[8], b[8];
      unpack8<T>(reinterpret_cast<const uint4*>(sm + S::kH)[e], a);
      unpack8<T>(reinterpret_cast<const uint4*>(sm + S::kDH)[e], b);
#pragma unroll
      for (int k = 0; k < 8; ++k) hp = fmaf(a[k], b[k], hp);
    }
    ok = !__syncthreads_or(!mine);
  }
  float dg = 0.f;
  if (ok && rows_lo) {  // rows 0..63: dq, dk
    mine = umma::mbar_wait(bar_b, 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStMma2);
    umma::fence_after_sync();
    if (mine) {
      const int i = row;
      const bool live = i < L;
      const float4* dk2 = reinterpret_cast<const float4*>(sm + S::kA1) + i * 32;
      float* dqrow = o.dqh + ((s + i) * p.HV + hv) * static_cast<int64_t>(D);
      float* dkrow = o.dkh + ((s + i) * p.HV + hv) * static_cast<int64_t>(D);
      float qd = 0.f, kd = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int c0 = colh * 64 + half * 32;
        float a[32], b[32];
        umma::tmem_ld32(tmem + S::kXh + lane_base + c0, a);
        umma::tmem_ld32(tmem + S::kXq + lane_base + c0, b);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int col = c0 + q8 * 8;
          const uint32_t off = (col >> 6) * kAtom + i * 128 + ((((col & 63) >> 3) ^ (i & 7)) << 4);
          float qv[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kQ + off), qv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            a[q8 * 8 + e] += b[q8 * 8 + e];
            qd = fmaf(qv[e], a[q8 * 8 + e], qd);
          }
        }
        if (live) {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            *reinterpret_cast<float4*>(dqrow + c0 + j4 * 4) = make_float4(a[j4 * 4], a[j4 * 4 + 1], a[j4 * 4 + 2], a[j4 * 4 + 3]);
        }
        umma::tmem_ld32(tmem + S::kXk + lane_base + c0, a);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const float4 t = dk2[((c0 >> 2) + j4) ^ (i & 31)];
          a[j4 * 4] += t.x;
          a[j4 * 4 + 1] += t.y;
          a[j4 * 4 + 2] += t.z;
          a[j4 * 4 + 3] += t.w;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int col = c0 + q8 * 8;
          const uint32_t off = (col >> 6) * kAtom + i * 128 + ((((col & 63) >> 3) ^ (i & 7)) << 4);
          float kv[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kK + off), kv);
#pragma unroll
          for (int e = 0; e < 8; ++e) kd = fmaf(kv[e], a[q8 * 8 + e], kd);
        }
        if (live) {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            *reinterpret_cast<float4*>(dkrow + c0 + j4 * 4) = make_float4(a[j4 * 4], a[j4 * 4 + 1], a[j4 * 4 + 2], a[j4 * 4 + 3]);
        }
      }
      dg = rq[i] * qd - rk[i] * kd;
      if (colh == 1) dgh[i] = dg;
    }
  }
  if (ok) ok = !__syncthreads_or(!mine);
  if (ok) {
    const float hh = dq_block_sum(hp, red);
    const float es = dq_block_sum(esum, red);
    if (rows_lo && colh == 0) {
      const int i = row;
      float a = dg + dgh[i];
      if (i == L - 1) a += exp2f(Gs[L - 1]) * hh + es;
      if (i < L) o.dG[(s + i) * p.HV + hv] = a;
    }
  } else if (warp == 0 && last_bar) {  // drain (bounded) the products still in flight
    umma::mbar_wait(last_bar, 0, 20000000LL);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// The WY-form gradients per (chunk, v-head): prepare_wy_repr_bwd
// (triton/fla/wy_fast.py:173-401)
// ---------------------------------------------------------------------------
// With b = beta, Gam_i = exp(G_i), cw = b Gam, D_ij = exp(G_i - G_j),
// k^ = diag(r_k) k and T = (I + A)^-1, A = tril_strict(diag(b) D * k^ k^^T):
//   X1 = [K; dW] K^T          rows 0..63: S = k^ k^^T (with r_k scales), rows 64..127: dW k^^T
//   X2 = [V; dv] V^T          rows 64..127: dv V^T
//   dT  = (dW k^^T) diag(cw) + (dv V^T) diag(b)
//   dR_w = T^T dW, dR_u = T^T dv, M2 = dT T^T, dA = -T^T M2 (strictly lower)
//   dv_out = diag(b) dR_u
//   dS = diag(b) D * dA,  dk^ += diag(cw) dR_w + dS k^ + dS^T k^
//   db_i = v_i.dR_u,i + Gam_i k^_i.dR_w,i + sum_j<i dA_ij D_ij S_ij
//   dG_i += cw_i k^_i.dR_w,i + sum_j F_ij - sum_j F_ji,  F = dS * S
// T comes from the fp32 solve of the forward WY kernel (solve_tril64_mma);
// every product runs on tcgen05 with bf16 operands (the reference rounds
// each of these operands to the input dtype before its dot).

struct WbSm {
  static constexpr int kKD = 0;                 // K a0 | dW a0 | K a1 | dW a1
  static constexpr int kDV = kKD + 4 * kAtom;   // V a0 | dv a0 | V a1 | dv a1
  static constexpr int kT = kDV + 4 * kAtom;    // T image atom, twice (M = 128 products repeat rows 0..63)
  static constexpr int kDT = kT + 2 * kAtom;    // dT image atom | zero atom; later dS diag(r_k), twice
  static constexpr int kM2 = kDT + 2 * kAtom;   // -M2 image atom; later diag(r_k) dS, twice
  static constexpr int kSk = kM2 + 2 * kAtom;   // S (fp32 [64][kMS])
  static constexpr int kAf = kSk + 64 * kMS * 4;  // A (fp32 [64][kMS]); later dS (fp32)
  static constexpr int kTf = kAf + 64 * kMS * 4;  // T (fp32 [64][kMS])
  static constexpr int kDTf = kTf + 64 * kMS * 4; // dT (fp32 [64][kMS])
  static constexpr int kZ = kDTf + 64 * kMS * 4;  // solve scratch
  static constexpr int kVec = kZ + kMScratch * 4; // G, b, cw, r_k, db, dG, colsum [64] each
  static constexpr int kBar = kVec + 7 * 64 * 4;
  static constexpr int kTmem = kBar + 5 * 8;      // mbarriers: loads, X, R, dA, dK
  static constexpr int kBytes = kTmem + 8 + 1024;
  static constexpr uint32_t kTx = 4 * kAtom + 2 * kVnImg;  // K and V by TMA, the dW and dv images
  static constexpr int kThreads = 256;
  // TMEM columns: X1 0-63, X2 64-127 (then the dK sum 0-127), dR_w 128-255, dR_u 256-383, M2 384-447, dA 448-511
  static constexpr uint32_t kX1 = 0, kX2 = 64, kDK = 0, kRw = 128, kRu = 256, kM = 384, kDA = 448;
  static_assert(kBytes <= 227 * 1024, "shared memory");
};

// byte offset of element (r, c) in a pair of 64-row atoms laid out `stride` bytes apart (columns 0-63, 64-127)
__device__ __forceinline__ uint32_t atom_pair_off(int r, int c, int stride) {
  return static_cast<uint32_t>((c >> 6) * stride + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

template <typename T>
__global__ void __launch_bounds__(WbSm::kThreads, 1)
tc_bwd_wy_kernel(const gdn_chunk_bwd_args p, const Work w, const WyOut o,
                 const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv) {
  using S = WbSm;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  float* Sk = reinterpret_cast<float*>(sm + S::kSk);
  float* Af = reinterpret_cast<float*>(sm + S::kAf);
  float* Tf = reinterpret_cast<float*>(sm + S::kTf);
  float* dTf = reinterpret_cast<float*>(sm + S::kDTf);
  float* Zs = reinterpret_cast<float*>(sm + S::kZ);
  float* Gs = reinterpret_cast<float*>(sm + S::kVec);
  float* bs = Gs + 64;
  float* cw = bs + 64;
  float* rk = cw + 64;
  float* dbv = rk + 64;
  float* dgv = dbv + 64;
  float* csum = dgv + 64;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::kTmem);
  const uint32_t bar_ld = umma::smem_u32(bars), bar_x = umma::smem_u32(bars + 1), bar_r = umma::smem_u32(bars + 2),
                 bar_da = umma::smem_u32(bars + 3), bar_dk = umma::smem_u32(bars + 4);
  int64_t n, lc;
  const int64_t cix = blockIdx.x / static_cast<unsigned>(p.HV);  // chunk-major, the v-heads of a chunk adjacent
  if (!locate_chunk(w.coff, p.N, cix, n, lc)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, colh = warp >> 2, row = quad * 32 + lane;
  const bool rows_lo = quad < 2;
  const int hv = static_cast<int>(blockIdx.x - cix * p.HV), h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t rowK = static_cast<int64_t>(p.HV) * D;
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  const long long wlim = 2000000000LL;

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) umma::mbar_init(bars + i, 1);
    umma::mbar_fence_init();
    umma::mbar_arrive_expect_tx(bar_ld, S::kTx);
    umma::tma_load_3d(sm + S::kKD, &tk, 0, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kKD + 2 * kAtom, &tk, 64, h, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kDV, &tv, 0, hv, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + S::kDV + 2 * kAtom, &tv, 64, hv, static_cast<int>(s), bar_ld);
    const int64_t img = cix * p.HV + hv;
    const uint8_t* dw = o.dw_img + img * kVnImg;
    const uint8_t* dv = o.dv_img + img * kVnImg;
    umma::bulk_g2s(sm + S::kKD + kAtom, dw, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kKD + 3 * kAtom, dw + kAtom, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kDV + kAtom, dv, kAtom, bar_ld);
    umma::bulk_g2s(sm + S::kDV + 3 * kAtom, dv + kAtom, kAtom, bar_ld);
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, 512);
    umma::fence_before_sync();
  }
  for (int e = tid; e < kAtom / 16; e += S::kThreads)  // zero rows 64..127 of [dT; 0]
    reinterpret_cast<uint4*>(sm + S::kDT + kAtom)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid < 64) {
    const bool live = tid < L;
    const float g = live ? o.gc[(s + tid) * p.HV + hv] : 0.f;
    const float bt = live ? p.beta[(s + tid) * p.HV + hv] : 0.f;
    Gs[tid] = g * kLog2e;  // G in the log2 domain
    bs[tid] = bt;
    cw[tid] = live ? bt * exp2f(g * kLog2e) : 0.f;
    csum[tid] = 0.f;
  }
  umma::fence_proxy_async();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  bool mine = umma::mbar_wait(bar_ld, 0, wlim);
  if (!mine) record_error(w.err, 1, kSiteStLoad);
  bool ok = !__syncthreads_or(!mine);
  uint32_t last_bar = 0, last_par = 0;
  auto adv = [](int ks) { return static_cast<uint64_t>(((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4); };
  if (ok) {
    if (warp == 0) {  // X1 = [K; dW] K^T, X2 = [V; dv] V^T
      if (umma::elect_one()) {
        const uint32_t id64 = umma::idesc_f16(128, 64, kBf16, false, false);
        const uint64_t d_kd = umma::smem_desc_sw128(umma::smem_u32(sm + S::kKD), 16, 1024);
        const uint64_t d_dv = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDV), 16, 1024);  // [V; dv]
        const uint64_t d_v = d_dv;                                                             // V (64 rows)
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) umma::mma_f16(tmem + S::kX1, d_kd + adv(ks), d_kd + adv(ks), id64, ks > 0);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) umma::mma_f16(tmem + S::kX2, d_dv + adv(ks), d_v + adv(ks), id64, ks > 0);
        umma::mma_commit(bar_x);
      }
      __syncwarp();
      last_bar = bar_x;
    }
    {  // L2-norm factors of the k rows (two threads per row) while the products run
      if (tid < 128) {
        const int i = tid >> 1, half = tid & 1;
        const uint8_t* at = sm + S::kKD + half * 2 * kAtom + i * 128;
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float x[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(at + c * 16), x);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        if (half == 0) rk[i] = p.use_qk_l2norm ? rsqrtf(ss + 1e-6f) : 1.f;
      }
    }
    __syncthreads();
    mine = umma::mbar_wait(bar_x, 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStMma1);
    umma::fence_after_sync();
    if (mine) {
      if (rows_lo) {  // S and A (rows 0..63)
        const int i = row;
        float x[32];
        umma::tmem_ld32(tmem + S::kX1 + lane_base + colh * 32, x);
        const float ri = rk[i], gi = Gs[i], bi = bs[i];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = colh * 32 + jj;
          const float sv = x[jj] * ri * rk[j];
          Sk[i * kMS + j] = sv;
          Af[i * kMS + j] = (i < L && j < i) ? bi * exp2f(gi - Gs[j]) * sv : 0.f;
        }
      } else {  // dT = (dW k^^T) diag(cw) + (dv V^T) diag(b) (rows 64..127 of X1 and X2)
        const int i = row - 64;
        float x[32], y[32];
        umma::tmem_ld32(tmem + S::kX1 + lane_base + colh * 32, x);
        umma::tmem_ld32(tmem + S::kX2 + lane_base + colh * 32, y);
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = colh * 32 + jj;
          dTf[i * kMS + j] = fmaf(x[jj] * rk[j], cw[j], y[jj] * bs[j]);
        }
      }
    }
    ok = !__syncthreads_or(!mine);
  }
  if (ok) {
    solve_tril64_mma(Af, Tf, Zs);  // T = (I + A)^-1 (starts and ends with a barrier)
    {  // T and dT images: thread -> row r, 32 columns
      const int r = tid >> 2, c0 = (tid & 3) * 16;
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) {
        const int c = c0 + q8 * 8;
        float t8[8], d8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          t8[e] = Tf[r * kMS + c + e];
          d8[e] = dTf[r * kMS + c + e];
        }
        const uint32_t off = r * 128 + (((c >> 3) ^ (r & 7)) << 4);
        const uint4 tp = pack8<T>(t8);
        *reinterpret_cast<uint4*>(sm + S::kT + off) = tp;
        *reinterpret_cast<uint4*>(sm + S::kT + kAtom + off) = tp;  // [T^T | T^T]: rows 64..127 of the products repeat 0..63
        *reinterpret_cast<uint4*>(sm + S::kDT + off) = pack8<T>(d8);
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) {  // dR_w = T^T dW, dR_u = T^T dv, M2 = dT T^T
      umma::fence_after_sync();
      if (umma::elect_one()) {
        const uint32_t idmn = umma::idesc_f16(128, 128, kBf16, true, true);
        const uint32_t idm2 = umma::idesc_f16(128, 64, kBf16, false, false);
        const uint64_t d_tt = umma::smem_desc_sw128(umma::smem_u32(sm + S::kT), kAtom, 1024);      // T^T, MN-major
        const uint64_t d_dw = umma::smem_desc_sw128(umma::smem_u32(sm + S::kKD + kAtom), 2 * kAtom, 1024);
        const uint64_t d_dvb = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDV + kAtom), 2 * kAtom, 1024);
        const uint64_t d_dt = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDT), 16, 1024);      // [dT; 0]
        const uint64_t d_t = umma::smem_desc_sw128(umma::smem_u32(sm + S::kT), 16, 1024);        // T, K-major B
#pragma unroll
        for (int ks = 0; ks < 64 / 16; ++ks)
          umma::mma_f16(tmem + S::kRw, d_tt + ((ks * 2048) >> 4), d_dw + ((ks * 2048) >> 4), idmn, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 64 / 16; ++ks)
          umma::mma_f16(tmem + S::kRu, d_tt + ((ks * 2048) >> 4), d_dvb + ((ks * 2048) >> 4), idmn, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 64 / 16; ++ks)
          umma::mma_f16(tmem + S::kM, d_dt + ((ks * 32) >> 4), d_t + ((ks * 32) >> 4), idm2, ks > 0);
        umma::mma_commit(bar_r);
      }
      __syncwarp();
      last_bar = bar_r;
    }
    mine = rows_lo ? umma::mbar_wait(bar_r, 0, wlim) : true;
    if (!mine) record_error(w.err, 1, kSiteStMma2);
    umma::fence_after_sync();
    if (mine && rows_lo) {  // -M2 image (rows 0..63)
      const int i = row;
      float x[32];
      umma::tmem_ld32(tmem + S::kM + lane_base + colh * 32, x);
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        float m[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) m[e] = -x[q8 * 8 + e];
        const int j0 = colh * 32 + q8 * 8;
        *reinterpret_cast<uint4*>(sm + S::kM2 + i * 128 + ((((j0 >> 3) ^ (i & 7))) << 4)) = pack8<T>(m);
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    ok = !__syncthreads_or(!mine);
  }
  if (ok && warp == 0) {  // dA = T^T (-M2)
    umma::fence_after_sync();
    if (umma::elect_one()) {
      const uint32_t ida = umma::idesc_f16(128, 64, kBf16, true, true);
      const uint64_t d_tt = umma::smem_desc_sw128(umma::smem_u32(sm + S::kT), kAtom, 1024);
      const uint64_t d_m2 = umma::smem_desc_sw128(umma::smem_u32(sm + S::kM2), kAtom, 1024);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem + S::kDA, d_tt + ((ks * 2048) >> 4), d_m2 + ((ks * 2048) >> 4), ida, ks > 0);
      umma::mma_commit(bar_da);
    }
    __syncwarp();
    last_bar = bar_da;
  }
  if (ok) {
    // rows 0..63 of dR_u, dR_w and dA sit twice in TMEM (lanes 0..63 and 64..127), so all eight warps
    // share them: thread -> row i, column part (32 of dR_u / dR_w, 16 of dA)
    mine = umma::mbar_wait(bar_da, 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStMma2);
    umma::fence_after_sync();
    if (mine) {
      const int i = (quad & 1) * 32 + lane, part = colh * 2 + (quad >> 1);
      const bool live = i < L;
      const float bi = bs[i], gi = Gs[i], ri = rk[i];
      float a = 0.f, r = 0.f;
      {  // U path: v_i . dR_u,i and dv = diag(b) dR_u; W path: k_i . dR_w,i
        const int c0 = part * 32;
        T* dvrow = static_cast<T*>(p.dv) + ((s + i) * p.HV + hv) * static_cast<int64_t>(D);
        float x[32];
        umma::tmem_ld32(tmem + S::kRu + lane_base + c0, x);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int c = c0 + q8 * 8;
          float vv[8], o8[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kDV + atom_pair_off(i, c, 2 * kAtom)), vv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            a = fmaf(vv[e], x[q8 * 8 + e], a);
            o8[e] = bi * x[q8 * 8 + e];
          }
          if (live) *reinterpret_cast<uint4*>(dvrow + c) = pack8<T>(o8);
        }
        umma::tmem_ld32(tmem + S::kRw + lane_base + c0, x);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int c = c0 + q8 * 8;
          float kv[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(sm + S::kKD + atom_pair_off(i, c, 2 * kAtom)), kv);
#pragma unroll
          for (int e = 0; e < 8; ++e) r = fmaf(kv[e], x[q8 * 8 + e], r);
        }
      }
      r *= ri;  // k^_i . dR_w,i over this part's columns
      // A path (16 columns of dA): t_i, dS, F row sums, and the dS images (written twice: [dS; dS])
      float x[16];
      umma::tmem_ld16(tmem + S::kDA + lane_base + part * 16, x);
      float t = 0.f, fr = 0.f;
      float dsk[16], dsr[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = part * 16 + jj;
        const bool in = live && j < i;
        const float dd = in ? exp2f(gi - Gs[j]) : 0.f;
        const float sv = Sk[i * kMS + j];
        t = fmaf(x[jj] * dd, sv, t);
        const float ds = in ? bi * dd * x[jj] : 0.f;
        Af[i * kMS + j] = ds;  // dS (fp32) for the column sums
        fr = fmaf(ds, sv, fr);
        dsk[jj] = ds * rk[j];
        dsr[jj] = ds * ri;
      }
#pragma unroll
      for (int q8 = 0; q8 < 2; ++q8) {
        const int j0 = part * 16 + q8 * 8;
        const uint32_t off = i * 128 + ((((j0 >> 3) ^ (i & 7))) << 4);
        const uint4 pk = pack8<T>(dsk + q8 * 8), pr = pack8<T>(dsr + q8 * 8);
        *reinterpret_cast<uint4*>(sm + S::kDT + off) = pk;           // dS diag(r_k)
        *reinterpret_cast<uint4*>(sm + S::kDT + kAtom + off) = pk;
        *reinterpret_cast<uint4*>(sm + S::kM2 + off) = pr;           // diag(r_k) dS
        *reinterpret_cast<uint4*>(sm + S::kM2 + kAtom + off) = pr;
      }
      Zs[part * 64 + i] = a + exp2f(gi) * r + t;  // partial db over this part (the solve scratch is free)
      Zs[256 + part * 64 + i] = cw[i] * r + fr;   // partial dG row terms
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    ok = !__syncthreads_or(!mine);
  }
  if (ok && warp == 0) {  // dK sum = [dS diag(r_k); 0] K + [diag(r_k) dS; 0]^T K  (into the X columns)
    umma::fence_after_sync();
    if (umma::elect_one()) {
      const uint32_t idq = umma::idesc_f16(128, 128, kBf16, false, true);
      const uint32_t idk = umma::idesc_f16(128, 128, kBf16, true, true);
      const uint64_t d_sk = umma::smem_desc_sw128(umma::smem_u32(sm + S::kDT), 16, 1024);
      const uint64_t d_sr = umma::smem_desc_sw128(umma::smem_u32(sm + S::kM2), kAtom, 1024);
      const uint64_t d_k = umma::smem_desc_sw128(umma::smem_u32(sm + S::kKD), 2 * kAtom, 1024);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem + S::kDK, d_sk + ((ks * 32) >> 4), d_k + ((ks * 2048) >> 4), idq, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem + S::kDK, d_sr + ((ks * 2048) >> 4), d_k + ((ks * 2048) >> 4), idk, true);
      umma::mma_commit(bar_dk);
    }
    __syncwarp();
    last_bar = bar_dk;
  }
  if (ok) {
    {  // column sums of F = dS * S (the sum_j F_ji term of dG_i): four threads per column, 16 rows each
      const int col = tid >> 2, part = tid & 3;
      float f = 0.f;
#pragma unroll 4
      for (int j = part * 16; j < part * 16 + 16; ++j) f = fmaf(Af[j * kMS + col], Sk[j * kMS + col], f);
      f += __shfl_xor_sync(0xffffffffu, f, 1);
      f += __shfl_xor_sync(0xffffffffu, f, 2);
      if (part == 0) csum[col] = f;
    }
    mine = umma::mbar_wait(bar_dk, 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStMma2);
    umma::fence_after_sync();
    ok = !__syncthreads_or(!mine);
  }
  if (ok) {  // dk^ += diag(cw) dR_w + dK sum (reductions into the dq/dk kernel's values); db; dG
    const int i = (quad & 1) * 32 + lane, part = colh * 2 + (quad >> 1);
    const bool live = i < L;
    const float ci = cw[i];
    const int c0 = part * 32;
    float* dkrow = o.dkh + ((s + i) * p.HV + hv) * static_cast<int64_t>(D) + c0;
    float x[32], y[32];
    umma::tmem_ld32(tmem + S::kRw + lane_base + c0, x);
    umma::tmem_ld32(tmem + S::kDK + lane_base + c0, y);
    if (live) {
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float v0 = fmaf(ci, x[j4 * 4], y[j4 * 4]), v1 = fmaf(ci, x[j4 * 4 + 1], y[j4 * 4 + 1]);
        const float v2 = fmaf(ci, x[j4 * 4 + 2], y[j4 * 4 + 2]), v3 = fmaf(ci, x[j4 * 4 + 3], y[j4 * 4 + 3]);
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dkrow + j4 * 4), "f"(v0), "f"(v1),
                     "f"(v2), "f"(v3) : "memory");
      }
    }
    if (part == 0 && live) {
      p.dbeta[(s + i) * p.HV + hv] = Zs[i] + Zs[64 + i] + Zs[128 + i] + Zs[192 + i];
      atomicAdd(o.dG + (s + i) * p.HV + hv,
                Zs[256 + i] + Zs[320 + i] + Zs[384 + i] + Zs[448 + i] - csum[i]);
    }
  }
  if (!ok && warp == 0 && last_bar) umma::mbar_wait(last_bar, last_par, 20000000LL);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// dv_local = scale P^T dO per (chunk, v-head): chunk_bwd_dv_local
// (triton/fla/chunk_o.py:233-778).  P is the forward WY kernel's image of
// M * exp(G_i - G_j) * q^_i.k^_j (core-matrix layout, rows i); read with the
// MN-major descriptor it is the A operand P^T (M = 64).  One product per
// tile; dv_local (fp32) goes to the dv workspace, which the state-gradient
// recurrence completes.
constexpr int kDvlThreads = 128;
// dynamic shared memory, padded so that at most four CTAs share an SM (four
// 128-column TMEM allocations fill its 512 columns)
constexpr int kDvlBytes = 56 * 1024;
static_assert(2 * kAtom + kImg64x64 + 64 + 1024 <= kDvlBytes && 5 * (kDvlBytes + 1024) > 228 * 1024,
              "at most four CTAs per SM");

template <typename T>
__global__ void __launch_bounds__(kDvlThreads)
tc_bwd_dvlocal_kernel(const gdn_chunk_bwd_args p, const Work w, float* dvn, float scale,
                      const __grid_constant__ CUtensorMap tdo) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* pim = sm + 2 * kAtom;
  uint64_t* bars = reinterpret_cast<uint64_t*>(pim + kImg64x64);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const uint32_t bar_ld = umma::smem_u32(bars), bar_mma = umma::smem_u32(bars + 1);
  int64_t n, lc;
  const int64_t cix = blockIdx.x / static_cast<unsigned>(p.HV);  // chunk-major, the v-heads of a chunk adjacent
  if (!locate_chunk(w.coff, p.N, cix, n, lc)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hv = static_cast<int>(blockIdx.x - cix * p.HV);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int64_t hc = static_cast<int64_t>(hv) * w.ncu + cix;
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  if (tid == 0) {
    umma::mbar_init(bars, 1);
    umma::mbar_init(bars + 1, 1);
    umma::mbar_fence_init();
    umma::mbar_arrive_expect_tx(bar_ld, 2 * kAtom + kImg64x64);
    umma::tma_load_3d(sm, &tdo, 0, hv, static_cast<int>(s), bar_ld);
    umma::tma_load_3d(sm + kAtom, &tdo, 64, hv, static_cast<int>(s), bar_ld);
    umma::bulk_g2s(pim, w.pimg + hc * kImg64x64, kImg64x64, bar_ld);
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, 128);
    umma::fence_before_sync();
  }
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  bool mine = warp == 0 ? umma::mbar_wait(bar_ld, 0) : true;
  if (!mine) record_error(w.err, 1, kSiteStLoad);
  bool ok = !__syncthreads_or(!mine);
  if (ok && warp == 0) {
    umma::fence_after_sync();
    if (umma::elect_one()) {
      const uint32_t id = umma::idesc_f16(64, 128, kBf16, true, true);
      const uint64_t da = umma::smem_desc(umma::smem_u32(pim), RS64, 128);
      const uint64_t db = umma::smem_desc_sw128(umma::smem_u32(sm), kAtom, 1024);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        umma::mma_f16(tmem, da + ((ks * 2 * RS64) >> 4), db + ((ks * 2048) >> 4), id, ks > 0);
      umma::mma_commit(bar_mma);
    }
    __syncwarp();
  }
  if (ok) {
    mine = umma::mbar_wait(bar_mma, 0);
    if (!mine) record_error(w.err, 1, kSiteStMma1);
    umma::fence_after_sync();
    // M = 64 accumulator: row j in lane j % 16 of warp j / 16
    const int j = warp * 16 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float* dst = dvn + ((s + j) * p.HV + hv) * static_cast<int64_t>(D);
#pragma unroll
    for (int q = 0; q < D / 32; ++q) {
      float x[32];
      umma::tmem_ld32(tmem + lane_base + q * 32, x);
      if (mine && lane < 16 && j < L) {
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          *reinterpret_cast<float4*>(dst + q * 32 + j4 * 4) =
              make_float4(scale * x[j4 * 4], scale * x[j4 * 4 + 1], scale * x[j4 * 4 + 2], scale * x[j4 * 4 + 3]);
      }
    }
  }
  if (warp == 0 && (!ok || !mine))  // drain (bounded) what may still be in flight before the memory is released
    umma::mbar_wait(ok ? bar_mma : bar_ld, 0, 20000000LL);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 128);
}

// [Ttot, HV, 128] tensor with 32-column x 1 head x 64-token boxes, no swizzle.
cudaError_t make_slice_map(CUtensorMap* m, const void* ptr, int heads, int64_t ttot, CUtensorMapDataType dt,
                           int esize) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(ttot)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * esize, static_cast<cuuint64_t>(heads) * D * esize};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(BwdSt::VS), 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_t(const gdn_chunk_bwd_args& b, const Work& w, const float* dvn, uint8_t* dv_img, uint8_t* dh_img,
                     cudaStream_t s) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const int64_t ttot = b.B * b.T;
  CUtensorMap tq, tk, tdo, tdv;
  cudaError_t e;
  if ((e = make_map(&tq, b.q, b.H, ttot, kF16)) != cudaSuccess) return e;
  if ((e = make_map(&tk, b.k, b.H, ttot, kF16)) != cudaSuccess) return e;
  if ((e = make_slice_map(&tdo, b.dout, b.HV, ttot,
                          kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2)) != cudaSuccess)
    return e;
  if ((e = make_slice_map(&tdv, dvn, b.HV, ttot, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4)) != cudaSuccess) return e;
  auto kern = tc_bwd_state_kernel<T>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdSt::kBytes)) != cudaSuccess)
    return e;
  note_launch();
  kern<<<dim3(static_cast<unsigned>(b.N * b.HV * (D / BwdSt::VS))), kSt3Threads, BwdSt::kBytes, s>>>(
      b, w, BwdOut{dv_img, dh_img}, tq, tk, tdo, tdv);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dqkw_t(const gdn_chunk_bwd_args& b, const Work& w, const DqkwOut& o, cudaStream_t s) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const int64_t ttot = b.B * b.T;
  const int64_t nc = chunk_upper_bound(ttot, b.N);
  if (nc == 0) return cudaSuccess;
  CUtensorMap tq, tk, tdo;
  cudaError_t e;
  if ((e = make_map(&tq, b.q, b.H, ttot, kF16)) != cudaSuccess) return e;
  if ((e = make_map(&tk, b.k, b.H, ttot, kF16)) != cudaSuccess) return e;
  if ((e = make_map(&tdo, b.dout, b.HV, ttot, kF16)) != cudaSuccess) return e;
  auto kern = tc_bwd_dqkw_kernel<T>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DqSm::kBytes)) != cudaSuccess)
    return e;
  const float scale = b.scale > 0.f ? b.scale : 1.f / sqrtf(static_cast<float>(b.K));
  note_launch();
  kern<<<dim3(static_cast<unsigned>(nc * b.HV)), DqSm::kThreads, DqSm::kBytes, s>>>(b, w, o, scale, tq, tk, tdo);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_wy_t(const gdn_chunk_bwd_args& b, const Work& w, const WyOut& o, cudaStream_t s) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const int64_t ttot = b.B * b.T;
  const int64_t nc = chunk_upper_bound(ttot, b.N);
  if (nc == 0) return cudaSuccess;
  CUtensorMap tk, tv;
  cudaError_t e;
  if ((e = make_map(&tk, b.k, b.H, ttot, kF16)) != cudaSuccess) return e;
  if ((e = make_map(&tv, b.v, b.HV, ttot, kF16)) != cudaSuccess) return e;
  auto kern = tc_bwd_wy_kernel<T>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, WbSm::kBytes)) != cudaSuccess)
    return e;
  note_launch();
  kern<<<dim3(static_cast<unsigned>(nc * b.HV)), WbSm::kThreads, WbSm::kBytes, s>>>(b, w, o, tk, tv);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dvl_t(const gdn_chunk_bwd_args& b, const Work& w, float* dvn, cudaStream_t s) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const int64_t ttot = b.B * b.T;
  const int64_t nc = chunk_upper_bound(ttot, b.N);
  if (nc == 0) return cudaSuccess;
  CUtensorMap tdo;
  cudaError_t e;
  if ((e = make_map(&tdo, b.dout, b.HV, ttot, kF16)) != cudaSuccess) return e;
  auto kern = tc_bwd_dvlocal_kernel<T>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDvlBytes)) != cudaSuccess)
    return e;
  const float scale = b.scale > 0.f ? b.scale : 1.f / sqrtf(static_cast<float>(b.K));
  note_launch();
  kern<<<dim3(static_cast<unsigned>(nc * b.HV)), kDvlThreads, kDvlBytes, s>>>(b, w, dvn, scale, tdo);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_dvlocal_tc(const gdn_chunk_bwd_args& b, const Work& w, float* dvn, cudaStream_t s) {
  return b.qkv_dtype == GDN_F16 ? launch_dvl_t<__half>(b, w, dvn, s) : launch_dvl_t<__nv_bfloat16>(b, w, dvn, s);
}

cudaError_t launch_bwd_wy_tc(const gdn_chunk_bwd_args& b, const Work& w, const WyOut& o, cudaStream_t s) {
  return b.qkv_dtype == GDN_F16 ? launch_wy_t<__half>(b, w, o, s) : launch_wy_t<__nv_bfloat16>(b, w, o, s);
}

cudaError_t launch_bwd_dqkw_tc(const gdn_chunk_bwd_args& b, const Work& w, const DqkwOut& o, cudaStream_t s) {
  return b.qkv_dtype == GDN_F16 ? launch_dqkw_t<__half>(b, w, o, s) : launch_dqkw_t<__nv_bfloat16>(b, w, o, s);
}

cudaError_t launch_bwd_state_tc(const gdn_chunk_bwd_args& b, const Work& w, const float* dvn, uint8_t* dv_img,
                                uint8_t* dh_img, cudaStream_t s) {
  return b.qkv_dtype == GDN_F16 ? launch_t<__half>(b, w, dvn, dv_img, dh_img, s)
                                : launch_t<__nv_bfloat16>(b, w, dvn, dv_img, dh_img, s);
}

}  // namespace tc
}  // namespace gdn
