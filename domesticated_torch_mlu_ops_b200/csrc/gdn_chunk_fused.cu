// Fused tensor-core chunked prefill: the WY stage and the state recurrence in
// one kernel, so that the WY work runs in the issue slots the serial state
// chain leaves idle instead of as a separate pass before it.
//
// One thread-block cluster of four CTAs per (sequence, v-head); CTA r of the
// cluster owns the 32-column V-slice r of the state (as tc_state3_kernel<32>
// does) and has two roles:
//
//   warps 0-7 (WY): the WY tiles of chunks r, r+4, r+8, ... of the sequence,
//     the arithmetic of tc_wy_kernel (chunk_scaled_dot_kkt.py:25-100,
//     solve_tril, wy_fast.py:18-119, chunk_o.py:133-160).  Both halves of
//     [T';T''][K|V] go to TMEM at once; W, U, P and the row scalars are
//     staged in shared memory, written to the workspace with bulk stores
//     (they stay in L2 until the chain reads them) and published with a
//     per-(v-head, chunk) flag (release after the stores complete).  The WY
//     role never waits for the chain, so it runs ahead of it.
//   warps 8-15 + 16 (state): the state chain of tc_state3_kernel<32>
//     (chunk_delta_h.py:28-197 fused with chunk_o.py:30-170) over two stages.
//     The load warp waits (bounded) for a chunk's flag, then loads its W, U
//     slice, P and scalars with bulk copies and its q and k tiles by TMA.
//
// The cluster launch only guarantees that the four CTAs of a (sequence,
// v-head) are resident together, which a consumer waiting for a partner's
// tile needs; no distributed shared memory and no multicast copy is used.
// Every wait (mbarriers, flags) is bounded and records an error; a role that
// gives up drains what it issued and leaves.

#include "gdn_chunk_tc.cuh"
#include "solve_tril.cuh"

namespace gdn {
namespace tc {

namespace {

constexpr int kFzCluster = 4;    // CTAs per (sequence, v-head): one per 32-column V-slice
constexpr int kFzThreads = 544;  // warps 0-7 WY, 8-15 state epilogue, 16 state loads
constexpr int kBarE1 = 1;        // state warps 8, 9, 12, 13 (128 threads)
constexpr int kBarSt = 2;        // state warps 8-16 (288 threads)
constexpr int kBarWy = 3;        // WY warps 0-7 (256 threads)

struct Fz {
  using S = St3<32>;
  static constexpr int VS = 32;
  static constexpr int kStages = 2;
  static constexpr int kStage = S::kStage;             // W a0 | Q a0 | W a1 | Q a1 | K a0 | K a1 | P | U | scalars
  static constexpr int kH = kStages * kStage;          // h image 128 x 32
  static constexpr int kVn = kH + D * VS * 2;          // v image 64 x 32
  static constexpr int kVt = kVn + 64 * VS * 2;        // diag(b) v image 64 x 32
  static constexpr int kWy = ((kVt + 64 * VS * 2 + 1023) / 1024) * 1024;
  static constexpr int kOps = kWy;                     // K a0 | Q a0 | K a1 | Q a1 (V over the Q atoms)
  static constexpr int kA = kOps + 4 * kAtom;          // f32 [64][kMS]; later the [T';T''] image
  static constexpr int kT = kA + 64 * kMS * 4;         // f32 [64][kMS]
  static constexpr int kZ = kT + 64 * kMS * 4;         // solve scratch
  static constexpr int kVec = kZ + kMScratch * 4;      // gam, beta, rk, rq, cw, cu, cf: f32 [7][64]
  static constexpr int kPl = kVec + 7 * 64 * 4;        // P image of the tile in flight
  static constexpr int kScl = kPl + kImg64x64;         // its scalars (a, b, gamma)
  static constexpr int kBar = kScl + kScal * 4;        // full[2], mma1, dh, o | kq, v, mma
  static constexpr int kTmem = kBar + 8 * 8;           // two TMEM base addresses (WY, state)
  static constexpr int kBytes = kTmem + 8 + 1024;
  // staging of a finished tile for its bulk stores: W over T, U over the [T';T''] image
  static constexpr int kStW = kT, kStU = kA;
  static_assert(kBytes <= 227 * 1024, "shared memory");
  static_assert(kPl % 16 == 0 && kScl % 16 == 0 && (kScal * 4) % 16 == 0, "16-byte bulk copies");
  static_assert(kWy % 1024 == 0 && kStW % 1024 == 0 && 64 * kMS * 4 >= 2 * kAtom, "staging");
};

__device__ __forceinline__ void tmem_alloc_keep(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(umma::smem_u32(dst_smem)), "r"(ncols) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kFzThreads, 1)
tc_fused_kernel(const gdn_chunk_args p, const Work w, float scale,
                const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv) {
  using S = Fz::S;
  constexpr int VS = Fz::VS;
  constexpr int RSV = (VS / 8) * 128;
  constexpr int CW = VS / 2;  // state columns per epilogue thread
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Fz::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + Fz::kTmem);
  const uint32_t bar_mma1 = umma::smem_u32(bars + 2), bar_dh = umma::smem_u32(bars + 3),
                 bar_o = umma::smem_u32(bars + 4), bar_kq = umma::smem_u32(bars + 5),
                 bar_v = umma::smem_u32(bars + 6), bar_mma = umma::smem_u32(bars + 7);
  auto full = [&](int x) { return umma::smem_u32(bars + (x & 1)); };
  auto stage = [&](int x) { return sm + (x & 1) * Fz::kStage; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = static_cast<int>(umma::cluster_ctarank());  // V-slice of this CTA
  const int64_t n = blockIdx.x / kFzCluster;
  const int hv = blockIdx.y, h = hv / (p.HV / p.H);
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int nch = static_cast<int>(eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0);
  const int64_t hc0 = static_cast<int64_t>(hv) * w.ncu + w.coff[n];  // workspace tile of chunk 0
  // test hook (gdn_chunk_fwd_test_stall): the first block runs with short waits
  const bool stall_block = blockIdx.x == 0 && blockIdx.y == 0 && w.stall_chunk >= 0;
  const long long wlim = stall_block ? w.stall_limit : 2000000000LL;

  if (tid == 0) {
    for (int i = 0; i < 8; ++i) umma::mbar_init(bars + i, 1);
    umma::mbar_fence_init();
  }
  if (warp == 0) {  // both TMEM allocations (all 512 columns) from one warp, then give up the permit
    tmem_alloc_keep(tslot, 256);
    umma::tmem_alloc(tslot + 1, 256);
    umma::fence_before_sync();
  }
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem_wy = tslot[0], tmem_st = tslot[1];

  if (warp < 8) {
    // =====================================================================
    // WY role: tiles of chunks rank, rank + 4, ...
    // =====================================================================
    uint8_t* ops = sm + Fz::kOps;
    uint8_t* timg = sm + Fz::kA;
    float* Af = reinterpret_cast<float*>(sm + Fz::kA);
    float* Tf = reinterpret_cast<float*>(sm + Fz::kT);
    float* Zs = reinterpret_cast<float*>(sm + Fz::kZ);
    float* gam = reinterpret_cast<float*>(sm + Fz::kVec);
    float* bet = gam + 64;
    float* rk = bet + 64;
    float* rq = rk + 64;
    float* cw = rq + 64;
    float* cu = cw + 64;
    float* cf = cu + 64;
    uint8_t* pl = sm + Fz::kPl;
    float* scl = reinterpret_cast<float*>(sm + Fz::kScl);
    const int quad = warp & 3, colh = warp >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t nmma = 0;         // tcgen05 commits on bar_mma so far (uniform over the role)
    int kq_tiles = 0, v_tiles = 0;  // tiles whose q/k (v) copies were issued (uniform)
    int64_t pending = -1;      // (thread 0) workspace tile whose bulk stores are issued but not yet published
    // thread 0: once the stores of the pending tile are complete, raise its flag
    auto publish = [&]() {
      if (pending >= 0) {
        umma::bulk_wait_all();
        umma::fence_proxy_async_global();
        umma::st_release_gpu(w.flags + pending, 1);
        pending = -1;
      }
    };
    auto issue_kq = [&](int x) {
      const int s0 = static_cast<int>(bos + static_cast<int64_t>(x) * kChunk);
      umma::mbar_arrive_expect_tx(bar_kq, 2 * kImg64x128);
      umma::tma_load_3d(ops, &tk, 0, h, s0, bar_kq);
      umma::tma_load_3d(ops + kAtom, &tq, 0, h, s0, bar_kq);
      umma::tma_load_3d(ops + 2 * kAtom, &tk, 64, h, s0, bar_kq);
      umma::tma_load_3d(ops + 3 * kAtom, &tq, 64, h, s0, bar_kq);
    };
    if (rank < nch) {
      if (tid == 0) issue_kq(rank);
      kq_tiles = 1;
    }
    bool fail = false;
    int it = 0;
    for (int x = rank; x < nch && !fail; x += kFzCluster, ++it) {
      const int64_t s = bos + static_cast<int64_t>(x) * kChunk;
      const int L = static_cast<int>(min64(kChunk, eos - s));
      if (warp == 1) {  // chunk-local inclusive cumsum of g (log2 domain)
        float g0 = lane < L ? p.g[(s + lane) * p.HV + hv] : 0.f;
        float g1 = lane + 32 < L ? p.g[(s + lane + 32) * p.HV + hv] : 0.f;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          float y0 = __shfl_up_sync(0xffffffffu, g0, o), y1 = __shfl_up_sync(0xffffffffu, g1, o);
          if (lane >= o) { g0 += y0; g1 += y1; }
        }
        g1 += __shfl_sync(0xffffffffu, g0, 31);
        gam[lane] = g0 * kLog2e;
        gam[lane + 32] = g1 * kLog2e;
      } else if (warp == 2) {
        bet[lane] = lane < L ? p.beta[(s + lane) * p.HV + hv] : 0.f;
        bet[lane + 32] = lane + 32 < L ? p.beta[(s + lane + 32) * p.HV + hv] : 0.f;
      }
      bool ok = warp == 0 ? umma::mbar_wait(bar_kq, static_cast<uint32_t>(it & 1), wlim) : true;
      if (!ok) record_error(w.err, 1, kSiteWyLoad);
      if (umma::named_sync_or(kBarWy, 256, !ok)) { fail = true; break; }
      if (warp == 0) {  // [K; Q] [K; Q]^T: S_kk, S_qk and both Gram diagonals
        umma::fence_after_sync();
        const uint32_t id = umma::idesc_f16(128, 128, kBf16, false, false);
        const uint64_t d0 = umma::smem_desc_sw128(umma::smem_u32(ops), 16, 1024);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t d = d0 + (((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4);
          if (umma::elect_one()) umma::mma_f16(tmem_wy, d, d, id, ks > 0);
        }
        if (umma::elect_one()) umma::mma_commit(bar_mma);
        __syncwarp();
      }
      // the previous tile's stores have had the q/k wait and this product to
      // finish: publish it; the staging (reused from the A/P epilogue on) is
      // free once the barrier below is passed
      if (tid == 0) publish();
      ok = warp == 0 ? umma::mbar_wait(bar_mma, nmma & 1u, wlim) : true;
      ++nmma;
      if (!ok) record_error(w.err, 1, kSiteWyMma1);
      if (umma::named_sync_or(kBarWy, 256, !ok)) { fail = true; break; }
      umma::fence_after_sync();
      if (colh == 0) {  // L2-norm factors from the Gram diagonal
        float xd[32];
        umma::tmem_ld32(tmem_wy + lane_base + quad * 32, xd);
        float d = 0.f;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) d = jj == lane ? xd[jj] : d;
        const float r = p.use_qk_l2norm ? rsqrtf(d + 1e-6f) : 1.f;
        if (row < 64) rk[row] = r; else rq[row - 64] = r;
      }
      umma::named_sync(kBarWy, 256);
      if (tid < 64) {
        cw[tid] = bet[tid] * exp2f(gam[tid]) * rk[tid];
        cu[tid] = bet[tid];
        cf[tid] = rk[tid] * exp2f(0.5f * (gam[0] + gam[L - 1]) - gam[tid]);
      }
      umma::fence_proxy_async();
      umma::named_sync(kBarWy, 256);
      if (warp == 3) {  // Q is dead: bring V into its atoms
        if (umma::elect_one()) {
          umma::mbar_arrive_expect_tx(bar_v, kImg64x128);
          umma::tma_load_3d(ops + kAtom, &tv, 0, hv, static_cast<int>(s), bar_v);
          umma::tma_load_3d(ops + 3 * kAtom, &tv, 64, hv, static_cast<int>(s), bar_v);
        }
        __syncwarp();
      }
      ++v_tiles;
      // A rows (fp32, shared) and P rows (bf16 image, kept for delivery)
      if (!(colh == 1 && quad == 0)) {
        const bool is_p = row >= 64;
        const int i = row & 63;
        const int jmax = i < L ? (is_p ? i : i - 1) : -1;
        const float mid = 0.5f * (gam[0] + gam[L - 1]);
        const bool factored = gam[0] - gam[L - 1] < 200.f;
        const float ri = (is_p ? rq[i] : rk[i] * bet[i]) * (factored ? exp2f(gam[i] - mid) : 1.f);
        const float gi = gam[i];
        const bool masked = colh == (quad & 1) || L < kChunk;
        float pv[32];
        if (colh == 1 && quad == 2) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) pv[jj] = 0.f;
        } else {
          float sv[32];
          umma::tmem_ld32(tmem_wy + lane_base + colh * 32, sv);
          if (factored) {
            const float2 r2 = make_float2(ri, ri);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 cj = ld4(cf + colh * 32 + j4 * 4);
              const float2 p0 = __fmul2_rn(r2, __fmul2_rn(make_float2(cj.x, cj.y), make_float2(sv[j4 * 4], sv[j4 * 4 + 1])));
              const float2 p1 = __fmul2_rn(r2, __fmul2_rn(make_float2(cj.z, cj.w), make_float2(sv[j4 * 4 + 2], sv[j4 * 4 + 3])));
              pv[j4 * 4 + 0] = p0.x;
              pv[j4 * 4 + 1] = p0.y;
              pv[j4 * 4 + 2] = p1.x;
              pv[j4 * 4 + 3] = p1.y;
            }
          } else {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const int j = colh * 32 + j4 * 4;
              const float4 gj = ld4(gam + j), rj = ld4(rk + j);
              pv[j4 * 4 + 0] = exp2f(gi - gj.x) * ri * rj.x * sv[j4 * 4 + 0];
              pv[j4 * 4 + 1] = exp2f(gi - gj.y) * ri * rj.y * sv[j4 * 4 + 1];
              pv[j4 * 4 + 2] = exp2f(gi - gj.z) * ri * rj.z * sv[j4 * 4 + 2];
              pv[j4 * 4 + 3] = exp2f(gi - gj.w) * ri * rj.w * sv[j4 * 4 + 3];
            }
          }
          if (masked) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) pv[jj] = colh * 32 + jj <= jmax ? pv[jj] : 0.f;
          }
        }
        if (is_p) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            *reinterpret_cast<uint4*>(pl + umma::img_off(i, colh * 32 + q8 * 8, RS64)) = pack8<T>(pv + q8 * 8);
        } else {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            st4(Af + i * kMS + colh * 32 + j4 * 4, make_float4(pv[j4 * 4], pv[j4 * 4 + 1], pv[j4 * 4 + 2], pv[j4 * 4 + 3]));
        }
      }
      umma::fence_before_sync();
      umma::named_sync(kBarWy, 256);
      solve_tril64_mma<kBarWy>(Af, Tf, Zs);  // T = (I + A)^-1, ends with the role's barrier
      {  // [T'; T''] image: row r < 64 -> T diag(cw), else T diag(beta)
        const int r = tid & 127, i = r & 63, half = tid >> 7;
        const float* coef = r < 64 ? cw : cu;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int col = half * 32 + q8 * 8;
          const float4 t0 = ld4(Tf + i * kMS + col), t1 = ld4(Tf + i * kMS + col + 4);
          const float4 c0 = ld4(coef + col), c1 = ld4(coef + col + 4);
          const float2 x0 = __fmul2_rn(make_float2(t0.x, t0.y), make_float2(c0.x, c0.y));
          const float2 x1 = __fmul2_rn(make_float2(t0.z, t0.w), make_float2(c0.z, c0.w));
          const float2 x2 = __fmul2_rn(make_float2(t1.x, t1.y), make_float2(c1.x, c1.y));
          const float2 x3 = __fmul2_rn(make_float2(t1.z, t1.w), make_float2(c1.z, c1.w));
          const float xv[8] = {x0.x, x0.y, x1.x, x1.y, x2.x, x2.y, x3.x, x3.y};
          *reinterpret_cast<uint4*>(timg + umma::img_off(r, col, RS64)) = pack8<T>(xv);
        }
      }
      if (tid < 64) {  // a_i, b_i, gamma of the chunk
        const float glast = gam[L - 1];
        scl[tid] = tid < L ? scale * exp2f(gam[tid]) * rq[tid] : 0.f;
        scl[64 + tid] = tid < L ? exp2f(glast - gam[tid]) * rk[tid] : 0.f;
        if (tid < 4) scl[128 + tid] = tid == 0 ? exp2f(glast) : 0.f;
      }
      umma::fence_proxy_async();
      umma::named_sync(kBarWy, 256);
      ok = warp == 0 ? umma::mbar_wait(bar_v, static_cast<uint32_t>(it & 1), wlim) : true;
      if (!ok) record_error(w.err, 1, kSiteWyLoad);
      if (umma::named_sync_or(kBarWy, 256, !ok)) { fail = true; break; }

      // [T'; T''] [K | V] as two N = 128 products (column halves 0..63 and
      // 64..127) into TMEM columns 0..127 and 128..255: rows 0..63 are W,
      // rows 64..127 are U.
      if (warp == 0) {
        umma::fence_after_sync();
        const uint32_t id = umma::idesc_f16(128, 128, kBf16, false, true);
        const uint64_t da = umma::smem_desc(umma::smem_u32(timg), 128, RS64);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const uint64_t db = umma::smem_desc_sw128(umma::smem_u32(ops + part * 2 * kAtom), kAtom, 1024);
#pragma unroll
          for (int ks = 0; ks < 64 / 16; ++ks)
            if (umma::elect_one())
              umma::mma_f16(tmem_wy + part * 128, da + ((ks * 256) >> 4), db + ((ks * 2048) >> 4), id, ks > 0);
        }
        if (umma::elect_one()) umma::mma_commit(bar_mma);
        __syncwarp();
      }
      ok = warp == 0 ? umma::mbar_wait(bar_mma, nmma & 1u, wlim) : true;
      ++nmma;
      if (!ok) record_error(w.err, 1, kSiteWyMma2);
      if (umma::named_sync_or(kBarWy, 256, !ok)) { fail = true; break; }
      umma::fence_after_sync();
      if (x + kFzCluster < nch) {  // the tile's operands are consumed: prefetch the next tile's q, k
        if (tid == 0) issue_kq(x + kFzCluster);
        ++kq_tiles;
      }
      {  // stage W (two swizzled atoms, over T) and U (four 32-column slices, over the T image)
        uint8_t* stw = sm + Fz::kStW;
        T* stu = reinterpret_cast<T*>(sm + Fz::kStU);
        const int i = row & 63;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          float xv[32];
          umma::tmem_ld32(tmem_wy + lane_base + part * 128 + (row < 64 ? 0 : 64) + colh * 32, xv);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            const int lcol = colh * 32 + q8 * 8;  // column within the half
            if (row < 64)
              *reinterpret_cast<uint4*>(stw + part * kAtom + i * 128 + ((((lcol >> 3) ^ (i & 7))) << 4)) =
                  pack8<T>(xv + q8 * 8);
            else
              *reinterpret_cast<uint4*>(stu + u_off(i, part * 64 + lcol, VS)) = pack8<T>(xv + q8 * 8);
          }
        }
      }
      umma::fence_proxy_async();
      umma::fence_before_sync();
      umma::named_sync(kBarWy, 256);
      if (tid == 0) {  // to the workspace; published during the next tile (or below)
        const int64_t hc = hc0 + x;
        umma::bulk_s2g(w.wimg + hc * kImg64x128, sm + Fz::kStW, 2 * kAtom);
        umma::bulk_s2g(w.u + hc * (64 * D * 2), sm + Fz::kStU, 64 * D * 2);
        umma::bulk_s2g(w.pimg + hc * kImg64x64, pl, kImg64x64);
        umma::bulk_s2g(w.scal + hc * kScal, scl, kScal * 4);
        umma::bulk_commit();
        pending = hc;
      }
    }
    if (tid == 0) publish();  // the last tile (or a tile stored before a failure)
    if (fail) {
      // wait (bounded) for copies and products this role issued
      const long long drain = wlim < 20000000LL ? wlim : 20000000LL;
      if (tid == 0) {
        if (kq_tiles > 0) umma::mbar_wait(bar_kq, static_cast<uint32_t>((kq_tiles - 1) & 1), drain);
        if (v_tiles > 0) umma::mbar_wait(bar_v, static_cast<uint32_t>((v_tiles - 1) & 1), drain);
        if (nmma > 0) umma::mbar_wait(bar_mma, (nmma - 1) & 1u, drain);
      }
    }
  } else {
    // =====================================================================
    // State role: the chain of tc_state3_kernel<32>, warps 8-15 + load warp 16
    // =====================================================================
    const int sw = warp - 8;
    const bool producer = sw == 8;
    const int quad = sw & 3, colh = (sw >> 2) & 1;
    const int row = quad * 32 + lane;
    const int v0 = rank * VS;
    uint8_t* himg = sm + Fz::kH;
    uint8_t* vnimg = sm + Fz::kVn;
    uint8_t* vtimg = sm + Fz::kVt;
    int fetched[Fz::kStages];  // (load thread) last chunk armed in each stage
#pragma unroll
    for (int i = 0; i < Fz::kStages; ++i) fetched[i] = -1;

    // wait (bounded) for chunk x's tile flag, then load the tile (W, P, U
    // slice, scalars) with bulk copies and the q, k tiles by TMA into stage x
    auto fetch = [&](int x) -> bool {
      if (stall_block && x == w.stall_chunk) return true;  // test hook: stage x is never filled
      const int64_t hc = hc0 + x;
      const long long t0 = clock64();
      while (umma::ld_acquire_gpu(w.flags + hc) == 0) {
        if (clock64() - t0 > wlim) {
          record_error(w.err, 1, kSiteFzReady);
          return false;
        }
        __nanosleep(64);
      }
      umma::fence_proxy_async_global();
      fetched[x & 1] = x;
      uint8_t* b = stage(x);
      const uint32_t bar = full(x);
      const int s0 = static_cast<int>(bos + static_cast<int64_t>(x) * kChunk);
      const uint8_t* wsrc = w.wimg + hc * kImg64x128;
      umma::mbar_arrive_expect_tx(bar, S::kTx);
      umma::bulk_g2s(b + S::kWQ, wsrc, kAtom, bar);
      umma::tma_load_3d(b + S::kWQ + kAtom, &tq, 0, h, s0, bar);
      umma::bulk_g2s(b + S::kWQ + 2 * kAtom, wsrc + kAtom, kAtom, bar);
      umma::tma_load_3d(b + S::kWQ + 3 * kAtom, &tq, 64, h, s0, bar);
      umma::tma_load_3d(b + S::kK, &tk, 0, h, s0, bar);
      umma::tma_load_3d(b + S::kK + kAtom, &tk, 64, h, s0, bar);
      umma::bulk_g2s(b + S::kP, w.pimg + hc * kImg64x64, kImg64x64, bar);
      umma::bulk_g2s(b + S::kU, w.u + ((hc * (D / VS) + rank) * 64 * VS) * 2, S::kUBytes, bar);
      umma::bulk_g2s(b + S::kSc, w.scal + hc * kScal, kScal * 4, bar);
      return true;
    };
    bool fetched_ok = true;
    if (producer && nch > 0) {
      if (lane == 0) fetched_ok = fetch(0);
      fetched_ok = __shfl_sync(0xffffffffu, fetched_ok, 0);
    }

    float hreg[CW];
    if (!producer) {
      const int64_t base = (n * p.HV + hv) * D * D;
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        const int col = v0 + colh * CW + j;
        hreg[j] = !p.initial_state ? 0.f
                  : p.state_v_first ? p.initial_state[base + static_cast<int64_t>(col) * D + row]
                                    : p.initial_state[base + static_cast<int64_t>(row) * D + col];
      }
#pragma unroll
      for (int j8 = 0; j8 < CW / 8; ++j8)
        *reinterpret_cast<uint4*>(himg + umma::img_off(row, colh * CW + j8 * 8, RSV)) = pack8<T>(hreg + j8 * 8);
    }
    umma::fence_proxy_async();
    umma::named_sync(kBarSt, 288);
    umma::fence_after_sync();
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_dh = tmem_st + S::kDH;
    auto t_acc = [&](int x) { return tmem_st + S::kAcc + static_cast<uint32_t>(x & 1) * VS; };
    auto t_o = [&](int x) { return tmem_st + S::kO + static_cast<uint32_t>(x & 1) * VS; };
    const uint32_t id_xy = umma::idesc_f16(128, VS, kBf16, false, true);
    const uint32_t id_dh = umma::idesc_f16(128, VS, kBf16, true, true);
    const uint64_t d_h = umma::smem_desc(umma::smem_u32(himg), RSV, 128);
    const uint64_t d_vt = umma::smem_desc(umma::smem_u32(vtimg), RSV, 128);
    const uint64_t d_vn = umma::smem_desc(umma::smem_u32(vnimg), RSV, 128);
    T* obase = static_cast<T*>(p.o);

    auto emit = [&](int x, float ai) {  // o rows of chunk x (quadrants 2, 3): o = a Y + scale O
      const int64_t s = bos + static_cast<int64_t>(x) * kChunk;
      const int L = static_cast<int>(min64(kChunk, eos - s));
      const int i = row - 64;
      float y[CW], z[CW];
#pragma unroll
      for (int q = 0; q < CW / 16; ++q)
        umma::tmem_ld16x2(t_acc(x) + lane_base + colh * CW + q * 16, t_o(x) + lane_base + colh * CW + q * 16,
                          y + q * 16, z + q * 16);
      if (i < L) {
        T* orow = obase + ((s + i) * p.HV + hv) * D + v0 + colh * CW;
#pragma unroll
        for (int j8 = 0; j8 < CW / 8; ++j8) {
          float ov[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) ov[e] = fmaf(ai, y[j8 * 8 + e], scale * z[j8 * 8 + e]);
          *reinterpret_cast<uint4*>(orow + j8 * 8) = pack8<T>(ov);
        }
      }
    };

    bool ok = true, mine = true;
    float a_prev = 0.f;
    uint32_t last_bar = 0, last_par = 0;  // warp 8: mbarrier and phase of its latest tcgen05 commit
    if (producer && nch > 0) {
      mine = fetched_ok && umma::mbar_wait(full(0), 0, wlim);
      if (fetched_ok && !mine) record_error(w.err, 1, kSiteStLoad);
    }
    for (int c = 0; c < nch; ++c) {
      if (umma::named_sync_or(kBarSt, 288, !mine)) { ok = false; break; }
      umma::fence_after_sync();
      uint8_t* b = stage(c);
      const float* sc = reinterpret_cast<const float*>(b + S::kSc);
      if (sw == 0) {  // MMA1: [X; Y] = [W; Q] h
        if (umma::elect_one()) {
          const uint64_t da = umma::smem_desc_sw128(umma::smem_u32(b + S::kWQ), 16, 1024);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            umma::mma_f16(t_acc(c), da + (((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4),
                          d_h + ((ks * 2 * RSV) >> 4), id_xy, ks > 0);
          umma::mma_commit(bar_mma1);
        }
        __syncwarp();
        last_bar = bar_mma1;
        last_par = static_cast<uint32_t>(c & 1);
      }
      if (producer) {
        if (c >= 1) {  // chunk c+1 goes where chunk c-1 was: its O product must be done
          mine = umma::mbar_wait(bar_o, static_cast<uint32_t>((c - 1) & 1), wlim);
          if (!mine) record_error(w.err, 1, kSiteStMma2);
        }
        if (mine && c + 1 < nch) {
          bool f = true;
          if (lane == 0) f = fetch(c + 1);
          mine = __shfl_sync(0xffffffffu, f, 0);
        }
        if (mine && c + 1 < nch) {
          mine = umma::mbar_wait(full(c + 1), static_cast<uint32_t>(((c + 1) >> 1) & 1), wlim);
          if (!mine) record_error(w.err, 1, kSiteStLoad);
        }
        continue;
      }
      if (quad >= 2) {  // off the chain: the previous chunk's output rows
        if (c >= 1) {
          mine = umma::mbar_wait(bar_o, static_cast<uint32_t>((c - 1) & 1), wlim);
          if (!mine) record_error(w.err, 1, kSiteStMma2);
          umma::fence_after_sync();
          if (mine) emit(c - 1, a_prev);
        }
        a_prev = sc[row - 64];
      } else {  // E1 (rows 0..63): v = U - X, V~ = diag(b) v
        mine = umma::mbar_wait(bar_mma1, static_cast<uint32_t>(c & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStMma1);
        umma::fence_after_sync();
        uint32_t rx[CW];
#pragma unroll
        for (int q = 0; q < CW / 16; ++q) umma::tmem_ld16_nw(t_acc(c) + lane_base + colh * CW + q * 16, rx + q * 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < CW / 16; ++q) umma::reg_fence16(rx + q * 16);
        const int i = row;
        const float bi = sc[64 + i];
        const T* ut = reinterpret_cast<const T*>(b + S::kU);
#pragma unroll
        for (int j8 = 0; j8 < CW / 8; ++j8) {
          const int col = colh * CW + j8 * 8;
          float u8[8], vn[8], vt[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(ut + u_off(i, col, VS)), u8);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            vn[e] = u8[e] - __uint_as_float(rx[j8 * 8 + e]);
            vt[e] = bi * vn[e];
          }
          *reinterpret_cast<uint4*>(vnimg + umma::img_off(i, col, RSV)) = pack8<T>(vn);
          *reinterpret_cast<uint4*>(vtimg + umma::img_off(i, col, RSV)) = pack8<T>(vt);
        }
        umma::fence_proxy_async();
        umma::fence_before_sync();
        umma::named_sync(kBarE1, 128);
        if (sw == 0) {  // MMA2: dH = K^T V~ (the chain), then O = [. ; P] v
          umma::fence_after_sync();
          if (umma::elect_one()) {
            const uint64_t dk = umma::smem_desc_sw128(umma::smem_u32(b + S::kK), kAtom, 1024);
#pragma unroll
            for (int ks = 0; ks < 64 / 16; ++ks)
              umma::mma_f16(t_dh, dk + ((ks * 2048) >> 4), d_vt + ((ks * 2 * RSV) >> 4), id_dh, ks > 0);
            umma::mma_commit(bar_dh);
            const uint64_t dp = umma::smem_desc(umma::smem_u32(b + S::kP - kImg64x64), 128, RS64);
#pragma unroll
            for (int ks = 0; ks < 64 / 16; ++ks)
              umma::mma_f16(t_o(c), dp + ((ks * 256) >> 4), d_vn + ((ks * 2 * RSV) >> 4), id_xy, ks > 0);
            umma::mma_commit(bar_o);
          }
          __syncwarp();
          last_bar = bar_o;
          last_par = static_cast<uint32_t>(c & 1);
        }
      }
      // E2 (rows 0..127): h <- gamma h + dH and the image of h for the next MMA1
      if (mine) {
        mine = umma::mbar_wait(bar_dh, static_cast<uint32_t>(c & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStMma2);
      }
      umma::fence_after_sync();
      if (mine) {
        float d[CW];
#pragma unroll
        for (int q = 0; q < CW / 16; ++q) umma::tmem_ld16(t_dh + lane_base + colh * CW + q * 16, d + q * 16);
        const float g = sc[128];
#pragma unroll
        for (int j = 0; j < CW; ++j) hreg[j] = fmaf(g, hreg[j], d[j]);
        if (c + 1 < nch) {
#pragma unroll
          for (int j8 = 0; j8 < CW / 8; ++j8)
            *reinterpret_cast<uint4*>(himg + umma::img_off(row, colh * CW + j8 * 8, RSV)) = pack8<T>(hreg + j8 * 8);
        }
      }
      umma::fence_proxy_async();
      umma::fence_before_sync();
    }
    if (ok && nch > 0) {  // the last chunk's output rows
      ok = !umma::named_sync_or(kBarSt, 288, !mine);
      if (ok && !producer && quad >= 2) {
        mine = umma::mbar_wait(bar_o, static_cast<uint32_t>((nch - 1) & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStMma2);
        umma::fence_after_sync();
        if (mine) emit(nch - 1, a_prev);
      }
      ok = !umma::named_sync_or(kBarSt, 288, !mine);
    }
    if (ok && !producer && p.final_state) {
      const int64_t base = (n * p.HV + hv) * D * D;
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        const int col = v0 + colh * CW + j;
        if (p.state_v_first) p.final_state[base + static_cast<int64_t>(col) * D + row] = hreg[j];
        else p.final_state[base + static_cast<int64_t>(row) * D + col] = hreg[j];
      }
    }
    if (!ok) {
      const long long drain = wlim < 20000000LL ? wlim : 20000000LL;
      if (producer && lane == 0)
        for (int x = 0; x < Fz::kStages; ++x)
          if (fetched[x] >= 0)
            umma::mbar_wait(full(fetched[x]), static_cast<uint32_t>((fetched[x] >> 1) & 1), drain);
      if (sw == 0 && last_bar) umma::mbar_wait(last_bar, last_par, drain);
    }
  }

  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  if (warp == 0) {
    umma::tmem_dealloc(tmem_wy, 256);
    umma::tmem_dealloc(tmem_st, 256);
  }
}

}  // namespace

bool fused_launchable(bool f16) {
  static int cached[2] = {-1, -1};  // per instantiation: clusters of this kernel fit on the device
  int& c = cached[f16 ? 1 : 0];
  if (c < 0) {
    auto kern = f16 ? tc_fused_kernel<__half> : tc_fused_kernel<__nv_bfloat16>;
    c = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Fz::kBytes) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(kFzCluster, 1);
      cfg.blockDim = dim3(kFzThreads);
      cfg.dynamicSmemBytes = Fz::kBytes;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = kFzCluster;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int nclusters = 0;
      if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) == cudaSuccess && nclusters > 0) c = 1;
    }
    cudaGetLastError();  // a failed query leaves no sticky error behind
  }
  return c == 1;
}

template <typename T>
cudaError_t launch_fused(const gdn_chunk_args& a, const Work& w, float scale, const CUtensorMap& tq,
                         const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t s) {
  auto kern = tc_fused_kernel<T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Fz::kBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.N * kFzCluster), static_cast<unsigned>(a.HV));
  cfg.blockDim = dim3(kFzThreads);
  cfg.dynamicSmemBytes = Fz::kBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kFzCluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, a, w, scale, tq, tk, tv);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template cudaError_t launch_fused<__nv_bfloat16>(const gdn_chunk_args&, const Work&, float, const CUtensorMap&,
                                                 const CUtensorMap&, const CUtensorMap&, cudaStream_t);
template cudaError_t launch_fused<__half>(const gdn_chunk_args&, const Work&, float, const CUtensorMap&,
                                          const CUtensorMap&, const CUtensorMap&, cudaStream_t);

}  // namespace tc
}  // namespace gdn
