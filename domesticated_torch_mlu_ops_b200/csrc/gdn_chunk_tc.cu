// Tensor-core (tcgen05) chunked gated delta-rule forward for bf16/fp16 inputs
// with K = V = 128 and 64-token chunks: the Qwen3-Next GDN prefill.
//
// Two kernels replace the reference's six stages (triton/fla/chunk.py:10-74):
//
// tc_wy_kernel, one CTA per (chunk, v-head), fully parallel, the v-heads of a
// chunk adjacent in launch order:
//   * q, k, v chunk tiles fetched by TMA (128-byte swizzled);
//   * L2-norm factors r_q, r_k of every row (fused_recurrent_fn.py:110-112
//     formula) and the chunk-local cumsum G of g (cumsum.py:20-77);
//   * S_kk = K K^T and S_qk = Q K^T on tcgen05 (bf16 in, fp32 in TMEM);
//   * A = beta_i exp(G_i - G_j) r_k,i r_k,j S_kk, strictly lower
//     (chunk_scaled_dot_kkt.py:25-100); (I + A)^-1 with the blocked solver
//     of solve_tril.cuh (the native solve_tril, include/torch_mlu_ops.h:1052);
//   * W = T diag(beta exp(G) r_k) K and U = T diag(beta) V on tcgen05
//     (wy_fast.py:18-119), with the row scalings folded into the bf16 A
//     operand exactly where the reference rounds to bf16;
//   * P = tril_incl(exp(G_i - G_j) r_q,i r_k,j S_qk) (chunk_o.py:133-160);
//   * per-row output / decay scales a_i = scale exp(G_i) r_q,i,
//     b_i = exp(G_last - G_i) r_k,i and gamma = exp(G_last).
//   W (swizzled) and P are written as ready-to-use UMMA operand images, U as
//   V-slices.  [K;Q] K^T and [T';T''] [K|V] are single M=128 MMAs, so every
//   thread of the epilogues owns one row of the result.
//
// tc_state3_kernel, one CTA per (sequence, v-head, V-slice of VS = 32, 64 or
// 128 columns; the slices of one head are adjacent CTAs), serial over the
// sequence's chunks (chunk_delta_h.py:28-197 fused with chunk_o.py:30-170).
// The fp32 state slice h (128 x VS) lives in registers (two threads per row);
// its bf16 copy in shared memory is the B operand of
//   [X; Y] = [W; Q] h                          (tcgen05, M=128)
//   v_new = U - X, V~ = diag(b) v_new          (rows 0..63, fp32 -> bf16)
//   dH = K^T V~,  [.; O] = [0; P] v_new        (tcgen05, M=128)
//   h <- gamma h + dH,  o = a * Y + scale * O  (all rows / rows 64..127)
// so h and v_new never leave the SM.  A load warp streams the next chunks'
// operands in with TMA / bulk copies while the current chunk computes.
//
// Every mbarrier wait is bounded; on timeout the kernel records an error in
// the workspace error word, waits (bounded) for its own copies and MMAs in
// flight, frees its TMEM and exits.

#include <cuda.h>

#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "conv_math.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_chunk_tc.cuh"
#include "solve_tril.cuh"
#include "umma.cuh"

namespace gdn {

namespace tc {

// ---------------------------------------------------------------------------
// WY kernel
// ---------------------------------------------------------------------------

// Shared memory of the WY kernel (about 51 KB, so 4 CTAs fit per SM; the
// fused-conv variant keeps a second 17 KB region for its input rows and fits
// 3).  The first 32 KiB hold four 64-row swizzled atoms: K(cols 0-63),
// Q(0-63), K(64-127), Q(64-127).  Read 16 KiB at a time they form the
// 128-row operand [K;Q]; once [K;Q]K^T is done, V is loaded over the Q atoms,
// and the atoms read 8 KiB apart form [K_0:64 | V_0:64 | K_64:128 | V_64:128],
// a valid N=256 MN-major operand (uniform atom stride).  A (fp32 [64][kMS])
// is inverted in place into T, whose upper-right block is the solve's
// scratch; the [T';T''] image is then written over it.  W and U leave
// through shared-memory staging and bulk stores: columns 0-63 staged over the
// atoms of K_0:64 and V_0:64 once the first W/U product has read them,
// columns 64-127 over the other two after the second.
template <bool CONV>
struct WySmem {
  static constexpr int kOps = 0;                 // 4 atoms
  static constexpr int kA = 4 * kAtom;           // f32 [64][kMS]: A, then T, then the [T';T''] image
  static constexpr int kX = kA + 64 * kMS * 4;   // fused conv only: the k and v input rows
  static constexpr int kVec = kX + (CONV ? 64 * kMS * 4 : 0);  // gam, beta, rk, rq, cw, cu, cf: f32 [7][64]
  static constexpr int kBar = kVec + 7 * 64 * 4;   // 3 mbarriers
  static constexpr int kTmem = kBar + 24;
  static constexpr int kBytes = kTmem + 8 + 1024;  // + slack for 1 KiB alignment
  static constexpr int kCtas = CONV ? 3 : 4;       // CTAs per SM
  static_assert(kCtas * (kBytes + 1024) <= 228 * 1024, "CTAs per SM");
  static_assert(64 * kMS * 4 >= kImg64x128, "the [T';T''] image fits over T");
  // fused conv: the pre-conv q and k rows s-3 .. s+63 ([67][128] 16-bit each)
  // land over A and X before the first product; the v rows over X after it
  static constexpr int kBox = 67 * 128 * 2;
  static_assert(!CONV || (kA + 2 * kBox <= kVec && kX + kBox <= kVec && kBox % 128 == 0), "conv boxes fit");
};
constexpr int kWyThreads = 256;

// --- the causal conv1d of the fused path (ConvIn) ---------------------------

// Line of sequence n's initial conv window and whether the conv skips the
// sequence (a PAD or null-block line: its outputs are zeros and its line is
// left alone), as causal_conv1d_fn decides (kernels.py:254-289).
__device__ __forceinline__ void conv_seq(const ConvIn& ci, int64_t n, int64_t& line, bool& hinit, bool& skip) {
  line = n;
  if (ci.cache_indices) {
    const int64_t col = ci.apc_init ? load_index(ci.apc_init, ci.apc_dtype, n) : 0;
    line = load_index(ci.cache_indices, ci.idx_dtype, n * ci.ci_stride + col);
  }
  skip = (ci.has_null && line == ci.null_block) || line == ci.pad_slot;
  hinit = ci.has_init && ci.has_init[n] && !skip;
}

// Taps of channels ch .. ch+3 as two channel pairs (w[0]: ch, ch+1; w[1]:
// ch+2, ch+3; per tap), and their bias: weight [dim, 4] rows ch .. ch+3 are
// 16 contiguous elements.
template <typename T>
__device__ __forceinline__ void conv_taps4(const ConvIn& ci, int64_t ch, float2 (&w)[2][4], float2 (&bias)[2]) {
  const uint4* wp = reinterpret_cast<const uint4*>(static_cast<const T*>(ci.weight) + ch * 4);
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    const uint4 r = __ldg(wp + pr);
    const float2 a0 = conv::unpack2<T>(r.x), a1 = conv::unpack2<T>(r.y);  // first channel: taps 0,1 | 2,3
    const float2 b0 = conv::unpack2<T>(r.z), b1 = conv::unpack2<T>(r.w);  // second channel
    w[pr][0] = make_float2(a0.x, b0.x);
    w[pr][1] = make_float2(a0.y, b0.y);
    w[pr][2] = make_float2(a1.x, b1.x);
    w[pr][3] = make_float2(a1.y, b1.y);
  }
  if (ci.bias) {
    const uint2 bb = __ldg(reinterpret_cast<const uint2*>(static_cast<const T*>(ci.bias) + ch));
    bias[0] = conv::unpack2<T>(bb.x);
    bias[1] = conv::unpack2<T>(bb.y);
  } else {
    bias[0] = bias[1] = make_float2(0.f, 0.f);
  }
}

// Input j (0..2) of the window before a sequence's first token, channels
// ch .. ch+3 (two pairs): the initial cache line's entries, or zeros.
template <typename T>
__device__ __forceinline__ void conv_halo4(const ConvIn& ci, int64_t line, bool hinit, int j, int64_t ch,
                                           float2 (&x)[2]) {
  if (!hinit) {
    x[0] = x[1] = make_float2(0.f, 0.f);
    return;
  }
  const uint16_t* st = static_cast<const uint16_t*>(ci.states) + line * ci.st_seq + j * ci.st_tok + ch;
  x[0] = conv::unpack2<T>(static_cast<uint32_t>(st[0]) | (static_cast<uint32_t>(st[1]) << 16));
  x[1] = conv::unpack2<T>(static_cast<uint32_t>(st[2]) | (static_cast<uint32_t>(st[3]) << 16));
}

// One output row of four channels from the window x0..x3 (per pair).
template <typename T>
__device__ __forceinline__ uint2 conv_out4(const float2 (&w)[2][4], const float2 (&bias)[2], const float2 (&x0)[2],
                                           const float2 (&x1)[2], const float2 (&x2)[2], const float2 (&x3)[2],
                                           bool act) {
  uint2 y;
  y.x = conv::conv2_w4<T>(w[0], bias[0], x0[0], x1[0], x2[0], x3[0], act);
  y.y = conv::conv2_w4<T>(w[1], bias[1], x0[1], x1[1], x2[1], x3[1], act);
  return y;
}

// Rows r0 .. r0+NR-1 (r0 a multiple of 8) of one 128-channel conv tile,
// channels c4 .. c4+3 of it: `box` holds the pre-conv rows s-3 .. s+63
// ([67][128], row-major, 16-bit); the outputs go to the 128-byte swizzled
// 64-row operand atoms at `atom` (columns 0-63; columns 64-127 two atoms on)
// or, with `keep`, to registers, and when `gdst` is given also to global rows
// s+i (row stride rs).  Rows at or past L, and every row of a skipped
// sequence, are zeros.  In a sequence's first chunk the window before row 0
// comes from the initial cache line.
template <typename T, int NR>
__device__ __forceinline__ void conv_rows4(const ConvIn& ci, const uint8_t* box, int c4, int64_t ch, int r0,
                                           bool first_chunk, int64_t line, bool hinit, bool skip, int L,
                                           uint8_t* atom, T* gdst, int64_t s, int64_t rs, uint2* keep) {
  float2 w[2][4], bias[2];
  conv_taps4<T>(ci, ch, w, bias);
  const uint2* src = reinterpret_cast<const uint2*>(box) + (c4 >> 2);  // 32 uint2 per row
  auto ld = [&](int r, float2 (&x)[2]) {
    const uint2 u = src[r * 32];
    x[0] = conv::unpack2<T>(u.x);
    x[1] = conv::unpack2<T>(u.y);
  };
  float2 x0[2], x1[2], x2[2];
  if (first_chunk && r0 == 0) {
    conv_halo4<T>(ci, line, hinit, 0, ch, x0);
    conv_halo4<T>(ci, line, hinit, 1, ch, x1);
    conv_halo4<T>(ci, line, hinit, 2, ch, x2);
  } else {
    ld(r0, x0);
    ld(r0 + 1, x1);
    ld(r0 + 2, x2);
  }
  uint8_t* at = atom + (c4 >= 64 ? 2 * kAtom : 0) + r0 * 128 + ((c4 & 7) * 2);
  const int cc = ((c4 & 63) >> 3) << 4;
  T* gd = gdst ? gdst + (s + r0) * rs : nullptr;
  const bool act = ci.act != 0;
  auto emit = [&](int k, uint2 y) {
    if (keep) keep[k] = y;
    else *reinterpret_cast<uint2*>(at + k * 128 + (cc ^ ((k & 7) << 4))) = y;
  };
  if (L >= r0 + NR && !skip) {  // every row of this run is inside the sequence
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      float2 x3[2];
      ld(r0 + k + 3, x3);
      const uint2 y = conv_out4<T>(w, bias, x0, x1, x2, x3, act);
      emit(k, y);
      if (gd) {
        *reinterpret_cast<uint2*>(gd) = y;
        gd += rs;
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        x0[e] = x1[e];
        x1[e] = x2[e];
        x2[e] = x3[e];
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      const int i = r0 + k;
      float2 x3[2];
      ld(i + 3, x3);
      uint2 y = make_uint2(0u, 0u);
      if (i < L && !skip) y = conv_out4<T>(w, bias, x0, x1, x2, x3, act);
      emit(k, y);
      if (gd && i < L) *reinterpret_cast<uint2*>(gd) = y;
      if (gd) gd += rs;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        x0[e] = x1[e];
        x1[e] = x2[e];
        x2[e] = x3[e];
      }
    }
  }
}

// CONV: the q, k, v tiles are the causal conv1d of ci.x, computed here in
// place of their TMA loads (q and k before the first product, v while it
// runs); the CTA of each chunk's first v-head of a q/k head also writes the
// post-conv q and k rows for the state kernel.
template <typename T, bool CONV>
__global__ void __launch_bounds__(kWyThreads, WySmem<CONV>::kCtas)
tc_wy_kernel(const gdn_chunk_args p, const Work w, float scale, const ConvIn ci,
             const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
             const __grid_constant__ CUtensorMap tv) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  using Ly = WySmem<CONV>;
  uint8_t* ops = sm + Ly::kOps;
  uint8_t* timg = sm + Ly::kA;  // [T';T''] 128 x 64 image, written over T after the solve
  float* Af = reinterpret_cast<float*>(sm + Ly::kA);  // A, inverted in place into T
  float* gam = reinterpret_cast<float*>(sm + Ly::kVec);
  float* bet = gam + 64;
  float* rk = bet + 64;
  float* rq = rk + 64;
  float* cw = rq + 64;
  float* cu = cw + 64;
  float* cf = cu + 64;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ly::kBar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + Ly::kTmem);
  const uint32_t bar_kq = umma::smem_u32(bars), bar_v = umma::smem_u32(bars + 1),
                 bar_mma = umma::smem_u32(bars + 2);

  // Without a plan kernel the first block clears the call's error word: an
  // error is recorded only after a wait of about a second, long after the
  // first wave of blocks has started.
  if (w.clear_err && blockIdx.x == 0 && threadIdx.x < 4) w.err[threadIdx.x] = 0;
  // Block = chunk * HV + v-head: the v-heads of a chunk are adjacent blocks,
  // so the q/k tiles a q/k head shares with its HV/H v-heads, and the 32-byte
  // sectors of a token's g and beta rows, come from HBM once and then from L2.
  // With the conv, block = v-head * chunks + chunk (measured about 1 % faster
  // there: its pre-conv boxes are 256-byte pieces of 16 KiB rows).
  const int hv = CONV ? static_cast<int>(blockIdx.x / w.ncu)
                      : static_cast<int>(blockIdx.x % static_cast<unsigned>(p.HV));
  const int h = hv / (p.HV / p.H);
  const int64_t c = CONV ? blockIdx.x - static_cast<int64_t>(hv) * w.ncu
                         : static_cast<int64_t>(blockIdx.x / static_cast<unsigned>(p.HV));
  int64_t n, lc;
  if (w.coff) {
    if (!locate_chunk(w.coff, p.N, c, n, lc)) return;
  } else {
    n = c / w.cps;
    lc = c - n * w.cps;
    if (n >= p.N) return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // TMEM lane quadrant (rows quad*32 .. +31 of every M=128 result) and the
  // 32-column half of the epilogues this warp covers
  const int quad = warp & 3, colh = warp >> 2;
  const int row = quad * 32 + lane;  // result row of this thread (0..127)
  const int64_t hc = static_cast<int64_t>(hv) * w.ncu + c;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int64_t s = bos + lc * kChunk;
  const int L = static_cast<int>(min64(kChunk, eos - s));
  const int us = w.vs < 64 ? w.vs : 64;  // U slice width

  if (tid == 0) {
    umma::mbar_init(bars, 1);
    umma::mbar_init(bars + 1, 1);
    umma::mbar_init(bars + 2, 1);
    umma::mbar_fence_init();
    if constexpr (CONV) {  // pre-conv q and k rows (tv: the x map)
      umma::mbar_arrive_expect_tx(bar_kq, 2 * Ly::kBox);
      umma::tma_load_2d(sm + Ly::kA, &tv, h * D, static_cast<int>(s) - 3, bar_kq);
      umma::tma_load_2d(sm + Ly::kA + Ly::kBox, &tv, (p.H + h) * D, static_cast<int>(s) - 3, bar_kq);
    } else {
      umma::mbar_arrive_expect_tx(bar_kq, 2 * kImg64x128);
      umma::tma_load_3d(ops, &tk, 0, h, static_cast<int>(s), bar_kq);
      umma::tma_load_3d(ops + kAtom, &tq, 0, h, static_cast<int>(s), bar_kq);
      umma::tma_load_3d(ops + 2 * kAtom, &tk, 64, h, static_cast<int>(s), bar_kq);
      umma::tma_load_3d(ops + 3 * kAtom, &tq, 64, h, static_cast<int>(s), bar_kq);
    }
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, 128);
    umma::fence_before_sync();
  }
  if (warp == 1) {  // chunk-local inclusive cumsum of g over 64 rows
    float g0 = lane < L ? p.g[(s + lane) * p.HV + hv] : 0.f;
    float g1 = lane + 32 < L ? p.g[(s + lane + 32) * p.HV + hv] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y0 = __shfl_up_sync(0xffffffffu, g0, o), y1 = __shfl_up_sync(0xffffffffu, g1, o);
      if (lane >= o) { g0 += y0; g1 += y1; }
    }
    g1 += __shfl_sync(0xffffffffu, g0, 31);
    gam[lane] = g0 * kLog2e;  // G in the log2 domain: exp(G_i - G_j) = exp2(gam_i - gam_j)
    gam[lane + 32] = g1 * kLog2e;
    if (w.gc_out) {  // the backward's recompute keeps G
      if (lane < L) w.gc_out[(s + lane) * p.HV + hv] = g0;
      if (lane + 32 < L) w.gc_out[(s + lane + 32) * p.HV + hv] = g1;
    }
  } else if (warp == 2) {
    bet[lane] = lane < L ? p.beta[(s + lane) * p.HV + hv] : 0.f;
    bet[lane + 32] = lane + 32 < L ? p.beta[(s + lane + 32) * p.HV + hv] : 0.f;
  }
  int64_t cline;
  bool chinit, cskip;
  if constexpr (CONV) conv_seq(ci, n, cline, chinit, cskip);
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  bool issued_store = false;
  uint2 vres[8];  // CONV: this thread's eight v output rows until the Q atoms are free
  bool okv;

  // One warp waits on each mbarrier; the block learns the outcome at the
  // barrier that follows (tcgen05 readers fence after it).  The conv tiles are
  // read by every thread, so every thread waits on their loads.
  bool ok = CONV || warp == 0 ? umma::mbar_wait(bar_kq, 0) : true;
  if (!ok) record_error(w.err, 1, kSiteWyLoad);
  if (__syncthreads_or(!ok)) goto teardown;
  if constexpr (CONV) {
    // q and k tiles: even warps q, odd warps k; lane -> four channels, warp
    // pair -> 16 rows; the CTA of a q/k head's first v-head also writes the
    // rows for the state kernel.
    const bool kside = warp & 1;
    const int c4 = lane * 4;
    const int64_t ch = (kside ? static_cast<int64_t>(p.H) * D : 0) + static_cast<int64_t>(h) * D + c4;
    T* gdst = hv % (p.HV / p.H) == 0
                  ? static_cast<T*>(kside ? ci.kc : ci.qc) + static_cast<int64_t>(h) * D + c4 : nullptr;
    conv_rows4<T, 16>(ci, sm + Ly::kA + (kside ? Ly::kBox : 0), c4, ch, (warp >> 1) * 16, lc == 0, cline,
                      chinit, cskip, L, ops + (kside ? 0 : kAtom), gdst, s, static_cast<int64_t>(p.H) * D, nullptr);
    umma::fence_proxy_async();  // the atoms are read by tcgen05; the boxes are rewritten by TMA next
    __syncthreads();
    if (tid == 0) {  // pre-conv v rows over T (the k box there is consumed)
      umma::mbar_arrive_expect_tx(bar_v, Ly::kBox);
      umma::tma_load_2d(sm + Ly::kX, &tv, (2 * p.H + hv) * D, static_cast<int>(s) - 3, bar_v);
    }
  }
  if (warp == 0) {  // [K; Q] [K; Q]^T  (M = 128, N = 128, K = 128): S_kk, S_qk and both Gram diagonals
    umma::fence_after_sync();
    const uint32_t id = umma::idesc_f16(128, 128, kBf16, false, false);
    const uint64_t d0 = umma::smem_desc_sw128(umma::smem_u32(ops), 16, 1024);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const uint64_t d = d0 + (((ks >> 2) * 2 * kAtom + (ks & 3) * 32) >> 4);
      if (umma::elect_one()) umma::mma_f16(tmem, d, d, id, ks > 0);
    }
    if (umma::elect_one()) umma::mma_commit(bar_mma);
  }
  okv = true;
  if constexpr (CONV) {  // v tile while the product runs: lane -> four channels, warp -> 8 rows
    okv = umma::mbar_wait(bar_v, 0);
    if (!okv) record_error(w.err, 1, kSiteWyLoad);
    if (okv) {
      const int c4 = lane * 4;
      const int64_t ch = 2 * static_cast<int64_t>(p.H) * D + static_cast<int64_t>(hv) * D + c4;
      conv_rows4<T, 8>(ci, sm + Ly::kX, c4, ch, warp * 8, lc == 0, cline, chinit, cskip, L, nullptr, nullptr, s,
                       0, vres);
    }
  }
  ok = warp == 0 ? umma::mbar_wait(bar_mma, 0) : true;
  if (!ok) record_error(w.err, 1, kSiteWyMma1);
  if (__syncthreads_or(!ok || !okv)) goto teardown;
  umma::fence_after_sync();
  if constexpr (CONV) {  // Q is dead: v into its atoms (made visible to tcgen05 before the W/U products)
    const int c4 = lane * 4, r0 = warp * 8;
    uint8_t* at = ops + kAtom + (c4 >= 64 ? 2 * kAtom : 0) + r0 * 128 + (c4 & 7) * 2;
    const int cc = ((c4 & 63) >> 3) << 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) *reinterpret_cast<uint2*>(at + k * 128 + (cc ^ ((k & 7) << 4))) = vres[k];
  }
  if (colh == 0) {  // L2-norm factors from the Gram diagonal: row r's |k|^2 or |q|^2 sits in column r
    float x[32];
    umma::tmem_ld32(tmem + lane_base + quad * 32, x);
    float d = 0.f;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) d = jj == lane ? x[jj] : d;
    const float r = p.use_qk_l2norm ? rsqrtf(d + 1e-6f) : 1.f;
    if (row < 64) rk[row] = r; else rq[row - 64] = r;
  }
  __syncthreads();
  if (tid < 64) {
    cw[tid] = bet[tid] * exp2f(gam[tid]) * rk[tid];
    cu[tid] = bet[tid];
    cf[tid] = rk[tid] * exp2f(0.5f * (gam[0] + gam[L - 1]) - gam[tid]);
  }
  umma::fence_proxy_async();
  __syncthreads();
  if (!CONV && warp == 3 && umma::elect_one()) {  // Q is dead: bring V into its atoms
    umma::mbar_arrive_expect_tx(bar_v, kImg64x128);
    umma::tma_load_3d(ops + kAtom, &tv, 0, hv, static_cast<int>(s), bar_v);
    umma::tma_load_3d(ops + 3 * kAtom, &tv, 64, hv, static_cast<int>(s), bar_v);
  }

  // Row `row` of [S_kk; S_qk], columns colh*32 .. +31: an A row (fp32, shared)
  // or a P row (bf16 image, global).  A rows 0..31 have nothing to the right
  // of column 31 and the solve never reads there; P rows 0..31 get zeros.
  // Blocks below the diagonal of a full chunk need no mask.
  if (!(colh == 1 && quad == 0)) {
    const bool is_p = row >= 64;
    const int i = row & 63;
    const int jmax = i < L ? (is_p ? i : i - 1) : -1;  // last nonzero column
    // exp2(gam_i - gam_j) = exp2(gam_i - mid) * exp2(mid - gam_j) when the
    // chunk's decay range keeps both factors far inside fp32 (gam is
    // non-increasing along the chunk); otherwise one exp2 per element.
    const float mid = 0.5f * (gam[0] + gam[L - 1]);
    const bool factored = gam[0] - gam[L - 1] < 200.f;
    const float ri = (is_p ? rq[i] : rk[i] * bet[i]) * (factored ? exp2f(gam[i] - mid) : 1.f);
    const float gi = gam[i];
    const bool masked = colh == (quad & 1) || L < kChunk;  // warp-uniform
    float pv[32];
    if (colh == 1 && quad == 2) {  // P rows 0..31, columns 32..63: all masked
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) pv[jj] = 0.f;
    } else {
      float sv[32];
      umma::tmem_ld32(tmem + lane_base + colh * 32, sv);
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
      uint8_t* pimg = w.pimg + hc * kImg64x64;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8)
        *reinterpret_cast<uint4*>(pimg + umma::img_off(i, colh * 32 + q8 * 8, RS64)) = pack8<T>(pv + q8 * 8);
    } else {
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4)
        st4(Af + i * kMS + colh * 32 + j4 * 4, make_float4(pv[j4 * 4], pv[j4 * 4 + 1], pv[j4 * 4 + 2], pv[j4 * 4 + 3]));
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  solve_tril64_mma_ip(Af);  // T = (I + A)^-1 over A, ends with a barrier
  {  // [T'; T''] image over T: row r < 64 -> T diag(cw), else T diag(beta); 32 columns per thread.
     // Every thread reads its T values before any image row is written.
    const int r = tid & 127, i = r & 63, half = tid >> 7;
    const float* coef = r < 64 ? cw : cu;
    const bool upper = half == 1 && i < 32;  // T's upper-right block: zero (it held the solve's scratch)
    uint4 img[4];
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) {
      const int col = half * 32 + q8 * 8;
      const float4 t0 = upper ? make_float4(0.f, 0.f, 0.f, 0.f) : ld4(Af + i * kMS + col);
      const float4 t1 = upper ? make_float4(0.f, 0.f, 0.f, 0.f) : ld4(Af + i * kMS + col + 4);
      const float4 c0 = ld4(coef + col), c1 = ld4(coef + col + 4);
      const float2 x0 = __fmul2_rn(make_float2(t0.x, t0.y), make_float2(c0.x, c0.y));
      const float2 x1 = __fmul2_rn(make_float2(t0.z, t0.w), make_float2(c0.z, c0.w));
      const float2 x2 = __fmul2_rn(make_float2(t1.x, t1.y), make_float2(c1.x, c1.y));
      const float2 x3 = __fmul2_rn(make_float2(t1.z, t1.w), make_float2(c1.z, c1.w));
      const float x[8] = {x0.x, x0.y, x1.x, x1.y, x2.x, x2.y, x3.x, x3.y};
      img[q8] = pack8<T>(x);
    }
    __syncthreads();
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8)
      *reinterpret_cast<uint4*>(timg + umma::img_off(r, half * 32 + q8 * 8, RS64)) = img[q8];
  }
  if (tid < 64) {
    float* sc = w.scal + hc * kScal;
    const float glast = gam[L - 1];
    sc[tid] = tid < L ? scale * exp2f(gam[tid]) * rq[tid] : 0.f;
    sc[64 + tid] = tid < L ? exp2f(glast - gam[tid]) * rk[tid] : 0.f;
    if (tid < 4) sc[128 + tid] = tid == 0 ? exp2f(glast) : 0.f;
  }
  umma::fence_proxy_async();
  __syncthreads();
  ok = !CONV && warp == 0 ? umma::mbar_wait(bar_v, 0) : true;
  if (!ok) record_error(w.err, 1, kSiteWyLoad);
  if (__syncthreads_or(!ok)) goto teardown;

  // [T'; T''] [K_half | V_half] for column halves 0..63 and 64..127 (M = 128,
  // N = 128, K = 64): rows 0..63 of columns 0..63 are W, rows 64..127 of
  // columns 64..127 are U.  Each half is staged as one 8 KiB W atom and one
  // 8 KiB run of U slices, both contiguous in global memory.
#pragma unroll 1
  for (int part = 0; part < 2; ++part) {
    if (warp == 0) {
      umma::fence_after_sync();
      const uint32_t id = umma::idesc_f16(128, 128, kBf16, false, true);
      const uint64_t da = umma::smem_desc(umma::smem_u32(timg), 128, RS64);
      const uint64_t db = umma::smem_desc_sw128(umma::smem_u32(ops + part * 2 * kAtom), kAtom, 1024);
#pragma unroll
      for (int ks = 0; ks < 64 / 16; ++ks)
        if (umma::elect_one())
          umma::mma_f16(tmem, da + ((ks * 256) >> 4), db + ((ks * 2048) >> 4), id, ks > 0);
      if (umma::elect_one()) umma::mma_commit(bar_mma);
    }
    ok = warp == 0 ? umma::mbar_wait(bar_mma, static_cast<uint32_t>((part + 1) & 1)) : true;
    if (!ok) record_error(w.err, 1, kSiteWyMma2);
    if (__syncthreads_or(!ok)) goto teardown;
    umma::fence_after_sync();
    uint8_t* stage = ops + part * 2 * kAtom;  // W atom, then the U run, over the atoms this product read
    {  // row < 64: W row; row >= 64: U row; 32 of the half's 64 columns per thread
      const int i = row & 63;
      float x[32];
      umma::tmem_ld32(tmem + lane_base + (row < 64 ? 0 : 64) + colh * 32, x);
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        const int lcol = colh * 32 + q8 * 8;  // column within the half
        if (row < 64) {
          *reinterpret_cast<uint4*>(stage + i * 128 + ((((lcol >> 3) ^ (i & 7))) << 4)) = pack8<T>(x + q8 * 8);
        } else {
          T* ust = reinterpret_cast<T*>(stage + kAtom);
          *reinterpret_cast<uint4*>(ust + u_off(i, lcol, us)) = pack8<T>(x + q8 * 8);
        }
      }
    }
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      umma::bulk_s2g(w.wimg + hc * kImg64x128 + part * kAtom, stage, kAtom);
      umma::bulk_s2g(w.u + hc * (64 * D * 2) + part * kAtom, stage + kAtom, kAtom);
      umma::bulk_commit();
      issued_store = true;
    }
  }

teardown:
  if (issued_store) umma::bulk_wait_read_all();  // staging must stay until the copies have read it
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------------------
// Warp-specialised state + output kernel (32- or 64-column V-slices)
// ---------------------------------------------------------------------------
//
// The state recurrence with the work of each chunk spread over
// nine warps, so that only the dependent chain stays serial:
//   MMA1  [X; Y] = [W; Q] h                  warp 0 issues (8 tcgen05.mma)
//   E1    v = U - X, V~ = diag(b) v          warps 0,1,4,5 (rows 0..63)
//   MMA2  dH = K^T V~ (chain), O = [. ; P] v  warp 0 issues, separate commits
//   E2    h <- gamma h + dH, image of h      warps 0..7 (rows 0..127)
// while, off the chain, warps 2,3,6,7 write o = a Y + scale O of the previous
// chunk during MMA1, and warp 8 waits on the loads and streams the chunks
// ahead into a ring of stages (three at VS = 32, two at VS = 64).  A
// tcgen05.mma costs about the same at N = 32 as at N = 64, so the chain is
// bounded by its MMA round trips and two epilogues, not by VS.
// Rows 0..63 of the O product read the K tile that precedes P in its stage
// and are never used.


// STORE (the backward's recompute): also store the fp32 state at every chunk
// start and v_new (Work::hs_out, Work::vnew_out).
template <typename T, int VS_, bool STORE>
__global__ void __launch_bounds__(kSt3Threads, 1)
tc_state3_kernel(const gdn_chunk_args p, const Work w, float scale,
                 const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk) {
  using S = St3<VS_>;
  constexpr int VS = S::VS;
  constexpr int RSV = (VS / 8) * 128;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* himg = sm + S::kH;
  uint8_t* vnimg = sm + S::kVn;
  uint8_t* vtimg = sm + S::kVt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBar);  // full[3], mma1, dh, o
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::kTmem);
  const uint32_t bar_mma1 = umma::smem_u32(bars + S::kStages), bar_dh = umma::smem_u32(bars + S::kStages + 1),
                 bar_o = umma::smem_u32(bars + S::kStages + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool producer = warp == 8;
  const int quad = warp & 3, colh = (warp >> 2) & 1;  // TMEM lane quadrant, column half
  const int row = quad * 32 + lane;
  // Block = (sequence * HV + v-head) * slices + slice: the slices of a chain,
  // and the chains of a q/k head's v-heads, are adjacent blocks and run in
  // step, so the operands they share come from HBM once and then from L2.
  constexpr int kSlices = D / VS;
  constexpr int CW = VS / 2;       // state columns per thread
  const int64_t chain = blockIdx.x / kSlices;
  const int64_t n = chain / p.HV;
  const int hv = static_cast<int>(chain - n * p.HV), h = hv / (p.HV / p.H);
  const int vsl = static_cast<int>(blockIdx.x % kSlices), v0 = vsl * VS;
  int64_t bos, eos;
  seq_bounds(p.cu_seqlens, p.cu_dtype, n, p.T, bos, eos);
  const int nch = static_cast<int>(eos > bos ? (eos - bos + kChunk - 1) / kChunk : 0);
  const int64_t c0 = w.coff ? w.coff[n] : n * w.cps;
  auto stage = [&](int x) { return sm + (x % S::kStages) * S::kStage; };
  auto full = [&](int x) { return umma::smem_u32(bars + x % S::kStages); };
  const bool stall_block = blockIdx.x == 0 && w.stall_chunk >= 0;
  const long long wlim = stall_block ? w.stall_limit : 2000000000LL;  // bound of every wait
  int fetched[S::kStages];  // (load thread) last chunk whose copies were issued into each stage
#pragma unroll
  for (int i = 0; i < S::kStages; ++i) fetched[i] = -1;

  // every operand of chunk x into its stage (one thread)
  auto fetch = [&](int x) {
    if (stall_block && x == w.stall_chunk) return;  // test hook: this stage is never filled
    fetched[x % S::kStages] = x;
    uint8_t* b = stage(x);
    const uint32_t bar = full(x);
    const int s = static_cast<int>(bos + static_cast<int64_t>(x) * kChunk);
    const int64_t hc = static_cast<int64_t>(hv) * w.ncu + c0 + x;
    const uint8_t* wsrc = w.wimg + hc * kImg64x128;
    umma::mbar_arrive_expect_tx(bar, S::kTx);
    umma::bulk_g2s(b + S::kWQ, wsrc, kAtom, bar);
    umma::tma_load_3d(b + S::kWQ + kAtom, &tq, 0, h, s, bar);
    umma::bulk_g2s(b + S::kWQ + 2 * kAtom, wsrc + kAtom, kAtom, bar);
    umma::tma_load_3d(b + S::kWQ + 3 * kAtom, &tq, 64, h, s, bar);
    umma::tma_load_3d(b + S::kK, &tk, 0, h, s, bar);
    umma::tma_load_3d(b + S::kK + kAtom, &tk, 64, h, s, bar);
    umma::bulk_g2s(b + S::kP, w.pimg + hc * kImg64x64, kImg64x64, bar);
    umma::bulk_g2s(b + S::kU, w.u + ((hc * (D / VS) + vsl) * 64 * VS) * 2, S::kUBytes, bar);
    umma::bulk_g2s(b + S::kSc, w.scal + hc * kScal, kScal * 4, bar);
  };

  if (tid == 256) {
    for (int i = 0; i < S::kStages + 3; ++i) umma::mbar_init(bars + i, 1);
    umma::mbar_fence_init();
    for (int x = 0; x < S::kStages - 1 && x < nch; ++x) fetch(x);
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, S::kCols);
    umma::fence_before_sync();
  }
  // state slice: thread `row` (warps 0..7) owns h[row][v0 + colh*16 .. +16] in fp32
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
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t t_dh = tmem + S::kDH;
  auto t_acc = [&](int x) { return tmem + S::kAcc + static_cast<uint32_t>(x & 1) * VS; };
  auto t_o = [&](int x) { return tmem + S::kO + static_cast<uint32_t>((x & 1) * (S::kOBufs - 1)) * VS; };
  constexpr bool kBf16 = !std::is_same<T, __half>::value;
  const uint32_t id_xy = umma::idesc_f16(128, VS, kBf16, false, true);
  const uint32_t id_dh = umma::idesc_f16(128, VS, kBf16, true, true);
  const uint64_t d_h = umma::smem_desc(umma::smem_u32(himg), RSV, 128);
  const uint64_t d_vt = umma::smem_desc(umma::smem_u32(vtimg), RSV, 128);
  const uint64_t d_vn = umma::smem_desc(umma::smem_u32(vnimg), RSV, 128);
  T* obase = static_cast<T*>(p.o);

  // o rows of chunk x (warps of quadrants 2, 3): o = a Y + scale O
  auto emit = [&](int x, float ai) {
    const int64_t s = bos + static_cast<int64_t>(x) * kChunk;
    const int L = static_cast<int>(min64(kChunk, eos - s));
    const int i = row - 64;
    T* orow = obase + ((s + i) * p.HV + hv) * D + v0 + colh * CW;
#pragma unroll
    for (int q = 0; q < CW / 16; ++q) {  // 16 columns at a time
      float y[16], z[16];
      umma::tmem_ld16x2(t_acc(x) + lane_base + colh * CW + q * 16, t_o(x) + lane_base + colh * CW + q * 16, y, z);
      if (i < L && obase) {
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
          float ov[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) ov[e] = fmaf(ai, y[h8 * 8 + e], scale * z[h8 * 8 + e]);
          *reinterpret_cast<uint4*>(orow + q * 16 + h8 * 8) = pack8<T>(ov);
        }
      }
    }
  };

  bool ok = true;   // uniform: changes only at block-wide barriers
  bool mine = true; // this thread's own waits since the last barrier
  float a_prev = 0.f;  // emit warps: a of the previous chunk's row
  uint32_t last_bar = 0, last_par = 0;  // warp 0: mbarrier and phase of its latest tcgen05 commit
  if (producer && nch > 0) {
    mine = umma::mbar_wait(full(0), 0, wlim);
    if (!mine) record_error(w.err, 1, kSiteStLoad);
  }
  for (int c = 0; c < nch; ++c) {
    if (__syncthreads_or(!mine)) { ok = false; break; }
    umma::fence_after_sync();
    uint8_t* b = stage(c);
    const float* sc = reinterpret_cast<const float*>(b + S::kSc);
    if (warp == 0) {  // MMA1: [X; Y] = [W; Q] h
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
      // chunk c + kStages - 1 goes where chunk c-1 was: its O product must be done
      if (c >= 1) {
        mine = umma::mbar_wait(bar_o, static_cast<uint32_t>((c - 1) & 1), wlim);
        if (!mine) record_error(w.err, 1, kSiteStMma2);
      }
      if (mine && c + S::kStages - 1 < nch && lane == 0) fetch(c + S::kStages - 1);
      __syncwarp();
      if (mine && c + 1 < nch) {  // operands of the next chunk
        mine = umma::mbar_wait(full(c + 1), static_cast<uint32_t>(((c + 1) / S::kStages) & 1), wlim);
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
      if constexpr (S::kOBufs == 1) {  // this chunk's O product reuses the buffer emit just read
        umma::fence_before_sync();
        umma::named_sync(1, 256);
      }
    } else {  // E1 (rows 0..63): v = U - X, V~ = diag(b) v
      // U and b have been in the stage since its loads completed: read them
      // while MMA1 runs
      const int i = row;
      const float bi = sc[64 + i];
      const T* ut = reinterpret_cast<const T*>(b + S::kU);
      constexpr int GW = CW < 32 ? CW : 32;  // columns per group of TMEM loads
      uint4 uraw[GW / 8];
#pragma unroll
      for (int j8 = 0; j8 < GW / 8; ++j8)
        uraw[j8] = *reinterpret_cast<const uint4*>(ut + u_off(i, colh * CW + j8 * 8, S::kUS));
      mine = umma::mbar_wait(bar_mma1, static_cast<uint32_t>(c & 1), wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma1);
      umma::fence_after_sync();
#pragma unroll
      for (int gq = 0; gq < CW / GW; ++gq) {
      if (gq > 0) {
#pragma unroll
        for (int j8 = 0; j8 < GW / 8; ++j8)
          uraw[j8] = *reinterpret_cast<const uint4*>(ut + u_off(i, colh * CW + gq * GW + j8 * 8, S::kUS));
      }
      uint32_t rx[GW];
#pragma unroll
      for (int q = 0; q < GW / 16; ++q)
        umma::tmem_ld16_nw(t_acc(c) + lane_base + colh * CW + gq * GW + q * 16, rx + q * 16);
      umma::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < GW / 16; ++q) umma::reg_fence16(rx + q * 16);
#pragma unroll
      for (int j8 = 0; j8 < GW / 8; ++j8) {
        const int col = colh * CW + gq * GW + j8 * 8;
        float u8[8], vn[8], vt[8];
        unpack8<T>(uraw[j8], u8);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          vn[e] = u8[e] - __uint_as_float(rx[j8 * 8 + e]);
          vt[e] = bi * vn[e];
        }
        *reinterpret_cast<uint4*>(vnimg + umma::img_off(i, col, RSV)) = pack8<T>(vn);
        *reinterpret_cast<uint4*>(vtimg + umma::img_off(i, col, RSV)) = pack8<T>(vt);
        if constexpr (STORE)  // every row, so that the image holds no stale values
          *reinterpret_cast<uint4*>(w.vn_img + ((c0 + c) * p.HV + hv) * kVnImg + bwd_img_off(i, v0 + col, 64)) =
              pack8<T>(vn);
      }
      }
      umma::fence_proxy_async();
      umma::fence_before_sync();
      umma::named_sync(1, S::kOBufs == 1 ? 256 : 128);  // warps 0, 1, 4, 5 (and the emit warps at one O buffer)
      if (warp == 0) {  // MMA2: dH = K^T V~ (the chain), then O = [. ; P] v
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
      constexpr int DW = CW < 32 ? CW : 32;  // columns per group of TMEM loads
      float d[CW];
#pragma unroll
      for (int gq = 0; gq < CW / DW; ++gq) {
        uint32_t rd[DW];
#pragma unroll
        for (int q = 0; q < DW / 16; ++q)
          umma::tmem_ld16_nw(t_dh + lane_base + colh * CW + gq * DW + q * 16, rd + q * 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < DW / 16; ++q) umma::reg_fence16(rd + q * 16);
#pragma unroll
        for (int j = 0; j < DW; ++j) d[gq * DW + j] = __uint_as_float(rd[j]);
      }
      const float g = sc[128];
      if constexpr (STORE) {  // the state at this chunk's start (as its products used it), for the backward
        uint8_t* dst = w.hs_img + ((c0 + c) * p.HV + hv) * static_cast<int64_t>(kStateImg);
#pragma unroll
        for (int j8 = 0; j8 < CW / 8; ++j8)
          *reinterpret_cast<uint4*>(dst + bwd_img_off(row, v0 + colh * CW + j8 * 8, 128)) = pack8<T>(hreg + j8 * 8);
      }
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
    ok = !__syncthreads_or(!mine);
    if (ok && !producer && quad >= 2) {
      mine = umma::mbar_wait(bar_o, static_cast<uint32_t>((nch - 1) & 1), wlim);
      if (!mine) record_error(w.err, 1, kSiteStMma2);
      umma::fence_after_sync();
      if (mine) emit(nch - 1, a_prev);
    }
    ok = !__syncthreads_or(!mine);
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
    // After a timeout, copies and MMAs this CTA issued may still be in
    // flight: wait (bounded) for the last fill of every stage and for warp
    // 0's latest tcgen05 commit (which covers all its earlier MMAs) before
    // the shared memory and TMEM are released.
    const long long drain = wlim < 20000000LL ? wlim : 20000000LL;
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
// Host side
// ---------------------------------------------------------------------------


EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;  // resolved once; the entry point never changes
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// The conv input x ((dim, tokens) channel-last, token stride sx elements):
// 128-channel x 67-token boxes, no swizzle, zeros outside the tensor.
cudaError_t make_map_x(CUtensorMap* m, const void* ptr, int64_t dim, int64_t ttot, int64_t sx, bool f16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(ttot)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(sx) * 2};
  const cuuint32_t box[2] = {128, 67};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// [Ttot, heads, 128] tensor, 64 x 64 boxes with 128-byte swizzle.
// tstride: elements between token rows (0: packed, heads * 128).
cudaError_t make_map(CUtensorMap* m, const void* ptr, int heads, int64_t ttot, bool f16, int64_t tstride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(ttot)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                                 static_cast<cuuint64_t>(tstride > 0 ? tstride : int64_t(heads) * D) * 2};
  const cuuint32_t box[3] = {64, 1, 64};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <typename T, int VS, bool STORE = false>
cudaError_t launch_state3(const gdn_chunk_args& a, const Work& w, float scale, const CUtensorMap& tq,
                          const CUtensorMap& tk, cudaStream_t s, LaunchHooks& hk) {
  using S = St3<VS>;
  auto kern = tc_state3_kernel<T, VS, STORE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
  if (e != cudaSuccess) return e;
  hk.pre(s);
  kern<<<dim3(static_cast<unsigned>(a.N * a.HV * (D / VS))), kSt3Threads, S::kBytes, s>>>(a, w, scale, tq, tk);
  return cudaGetLastError();
}

// V-slice width of the state kernel.  Every (sequence, v-head) chain takes
// 128 / VS CTAs of one SM each, so the kernel runs about
// ceil(N * HV * 128 / VS / SMs) waves, each as long as a chain; a chunk step
// of a chain costs about 2.2 K cycles at VS = 32, 3.7 K at VS = 64 and 5.5 K
// at VS = 128 (measured on a B200: the wider slices share their operand loads
// and synchronisations across more columns).  The width with the fewest
// cycles wins: 32-column slices for a few chains (config 1: 128 CTAs, one
// wave), 128-column slices for many (configs 2 and 4).  GDN_TC_VS=32, 64 or
// 128 in the environment overrides the choice (results are the same for every
// width: each column's arithmetic does not depend on it).
int sm_count() {
  static int n = 0;  // of the first device asked; B200s have 148
  if (n == 0) {
    int dev = 0, v = 0;
    n = cudaGetDevice(&dev) == cudaSuccess &&
                cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0
            ? v
            : 148;
  }
  return n;
}

int choose_vs(const gdn_chunk_args& a) {
  const char* v = getenv("GDN_TC_VS");
  if (v && (!strcmp(v, "32") || !strcmp(v, "64") || !strcmp(v, "128"))) return atoi(v);
  const int64_t chains = a.N * a.HV, sms = sm_count();
  int best = 32;
  double best_cost = 0.0;
  const int widths[3] = {32, 64, 128};
  const double step_cost[3] = {2.2, 3.7, 5.5};
  for (int i = 0; i < 3; ++i) {
    const int64_t ctas = chains * (D / widths[i]);
    const double cost = static_cast<double>((ctas + sms - 1) / sms) * step_cost[i];
    if (i == 0 || cost < best_cost) {
      best = widths[i];
      best_cost = cost;
    }
  }
  return best;
}

// The fused cluster kernel (gdn_chunk_fused.cu) is opt-in: GDN_TC_FUSED=1 in
// the environment selects it where clusters of it fit.  Measured on a B200 at
// the Qwen3-Next prefill shape it is slower than this pair (0.31 vs 0.26 ms):
// with one CTA per SM it has one WY tile in flight per SM, where the separate
// WY kernel keeps three, so its WY role (about 16 K cycles a tile, one tile
// per four chunks) cannot keep up with the 2.1 K-cycle chain.  Both paths run
// the same arithmetic (bit-identical results with 32-column slices).
bool choose_fused(bool f16) {
  const char* v = getenv("GDN_TC_FUSED");
  return v && v[0] == '1' && fused_launchable(f16);
}

// The WY kernel's blocks: chunk * HV + v-head (v-head * chunks + chunk with
// the conv); the state kernel's: (sequence * HV + v-head) * slices + slice.
// Both are one-dimensional grids (x limit 2^31 - 1).
static bool grids_fit(const gdn_chunk_args& a, const Work& w) {
  return w.ncu * a.HV <= 0x7fffffffLL && a.N * a.HV * (D / 32) <= 0x7fffffffLL;
}
static dim3 wy_blocks(const Work& w, int HV) { return dim3(static_cast<unsigned>(w.ncu * HV)); }

template <typename T>
cudaError_t run(const gdn_chunk_args& a, cudaStream_t s, int64_t stall_chunk, long long stall_limit,
                const gdn_conv1d_fn_args* conv) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const bool cv = conv != nullptr;
  const Layout l = plan(a, cv);
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  Work w{};  // every field not set below (the backward's store pointers) stays null
  w.coff = reinterpret_cast<const int64_t*>(ws + l.coff);
  w.err = reinterpret_cast<int*>(ws + l.err);
  w.wimg = ws + l.wimg;
  w.u = ws + l.u;
  w.pimg = ws + l.pimg;
  w.scal = reinterpret_cast<float*>(ws + l.scal);
  w.flags = reinterpret_cast<int*>(ws + l.flags);
  w.ncu = chunk_upper_bound(a.B * a.T, a.N);
  const bool fused = !cv && choose_fused(kF16);
  w.vs = fused ? 32 : choose_vs(a);  // the fused kernel writes and reads 32-column U slices
  w.stall_chunk = stall_chunk;
  w.stall_limit = stall_limit;
  if (!grids_fit(a, w)) return cudaErrorInvalidConfiguration;
  const int64_t ttot = a.B * a.T;
  const float scale = a.scale > 0.f ? a.scale : 1.f / sqrtf(static_cast<float>(a.K));
  ConvIn ci{};
  if (cv) {
    ci.x = conv->x; ci.weight = conv->weight; ci.bias = conv->bias; ci.states = conv->conv_states;
    ci.cache_indices = conv->cache_indices; ci.has_init = conv->has_initial_state;
    ci.apc_init = conv->block_idx_last ? conv->initial_state_idx : nullptr;
    ci.qc = ws + l.qc; ci.kc = ws + l.kc;
    ci.sx = conv->stride_x_token; ci.st_seq = conv->stride_state_seq; ci.st_tok = conv->stride_state_tok;
    ci.ci_stride = conv->cache_indices ? (conv->stride_cache_indices > 0 ? conv->stride_cache_indices : 1) : 0;
    ci.pad_slot = conv->pad_slot_id; ci.null_block = conv->null_block_id; ci.has_null = conv->has_null_block;
    ci.idx_dtype = conv->idx_dtype; ci.apc_dtype = conv->apc_dtype; ci.act = conv->activation == GDN_ACT_SILU;
  }
  CUtensorMap tq, tk, tv;
  cudaError_t e;
  if (ttot > 0) {  // with the conv, the state kernel reads the post-conv q and k that the WY kernel writes
    if ((e = make_map(&tq, cv ? ci.qc : a.q, a.H, ttot, kF16, cv ? 0 : a.q_token_stride)) != cudaSuccess) return e;
    if ((e = make_map(&tk, cv ? ci.kc : a.k, a.H, ttot, kF16, cv ? 0 : a.k_token_stride)) != cudaSuccess) return e;
    if (cv) {  // the WY kernel's third map is the conv input
      if ((e = make_map_x(&tv, conv->x, conv->dim, ttot, conv->stride_x_token, kF16)) != cudaSuccess) return e;
    } else if ((e = make_map(&tv, a.v, a.HV, ttot, kF16, a.v_token_stride)) != cudaSuccess) return e;
  }
  LaunchHooks hk(a.stage_events, a.n_stage_events);
  // Sequences of equal length need no chunk table: the kernels compute the
  // offsets and the WY kernel clears the error word (the fused kernel's flags,
  // packed sequences, the fused conv and empty calls still use the plan kernel)
  if (!a.cu_seqlens && !fused && !cv && ttot > 0) {
    w.coff = nullptr;
    w.cps = (a.T + kChunk - 1) / kChunk;
    w.clear_err = 1;
    hk.mark(s);
  } else {
    hk.pre(s);
    e = launch_chunk_plan(a.cu_seqlens, a.cu_dtype, a.N, a.T, reinterpret_cast<int64_t*>(ws + l.coff), s, 64,
                          w.err, fused ? w.flags : nullptr, fused ? static_cast<int64_t>(a.HV) * w.ncu : 0);
    if (e != cudaSuccess) return e;
  }
  if (ttot > 0) {
    if (fused) {
      hk.pre(s);
      if ((e = launch_fused<T>(a, w, scale, tq, tk, tv, s)) != cudaSuccess) return e;
    } else {
      auto wy = cv ? tc_wy_kernel<T, true> : tc_wy_kernel<T, false>;
      const int wy_bytes = cv ? WySmem<true>::kBytes : WySmem<false>::kBytes;
      if ((e = cudaFuncSetAttribute(wy, cudaFuncAttributeMaxDynamicSharedMemorySize, wy_bytes)) !=
          cudaSuccess)
        return e;
      hk.pre(s);
      wy<<<wy_blocks(w, a.HV), kWyThreads, wy_bytes, s>>>(a, w, scale, ci, tq, tk, tv);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
      if (w.vs == 32) e = launch_state3<T, 32>(a, w, scale, tq, tk, s, hk);
      else if (w.vs == 64) e = launch_state3<T, 64>(a, w, scale, tq, tk, s, hk);
      else e = launch_state3<T, 128>(a, w, scale, tq, tk, s, hk);
      if (e != cudaSuccess) return e;
      // the cache lines change only after every reader of the initial lines is done
      if (cv && (e = launch_conv_fn_states(*conv, s)) != cudaSuccess) return e;
    }
  } else if (a.final_state) {  // no tokens: the final states are the initial ones
    const size_t bytes = static_cast<size_t>(a.N) * a.HV * D * D * sizeof(float);
    e = a.initial_state ? cudaMemcpyAsync(a.final_state, a.initial_state, bytes, cudaMemcpyDeviceToDevice, s)
                        : cudaMemsetAsync(a.final_state, 0, bytes, s);
    if (e != cudaSuccess) return e;
  }
  hk.end(s);
  return cudaSuccess;
}

template <typename T>
cudaError_t run_wy_only(const gdn_chunk_args& a, void* wsv, cudaStream_t s, Work& w, float* gc_out) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const Layout l = plan(a);
  uint8_t* ws = static_cast<uint8_t*>(wsv);
  w = Work{};
  w.coff = reinterpret_cast<const int64_t*>(ws + l.coff);
  w.err = reinterpret_cast<int*>(ws + l.err);
  w.wimg = ws + l.wimg;
  w.u = ws + l.u;
  w.pimg = ws + l.pimg;
  w.scal = reinterpret_cast<float*>(ws + l.scal);
  w.flags = reinterpret_cast<int*>(ws + l.flags);
  w.ncu = chunk_upper_bound(a.B * a.T, a.N);
  w.vs = 32;
  w.stall_chunk = -1;
  w.gc_out = gc_out;
  if (!grids_fit(a, w)) return cudaErrorInvalidConfiguration;
  const int64_t ttot = a.B * a.T;
  const float scale = a.scale > 0.f ? a.scale : 1.f / sqrtf(static_cast<float>(a.K));
  note_launch();
  cudaError_t e = launch_chunk_plan(a.cu_seqlens, a.cu_dtype, a.N, a.T, reinterpret_cast<int64_t*>(ws + l.coff), s,
                                    64, w.err);
  if (e != cudaSuccess || ttot == 0) return e;
  CUtensorMap tq, tk, tv;
  if ((e = make_map(&tq, a.q, a.H, ttot, kF16, a.q_token_stride)) != cudaSuccess) return e;
  if ((e = make_map(&tk, a.k, a.H, ttot, kF16, a.k_token_stride)) != cudaSuccess) return e;
  if ((e = make_map(&tv, a.v, a.HV, ttot, kF16, a.v_token_stride)) != cudaSuccess) return e;
  auto wy = tc_wy_kernel<T, false>;
  if ((e = cudaFuncSetAttribute(wy, cudaFuncAttributeMaxDynamicSharedMemorySize, WySmem<false>::kBytes)) != cudaSuccess)
    return e;
  note_launch();
  wy<<<wy_blocks(w, a.HV), kWyThreads, WySmem<false>::kBytes, s>>>(a, w, scale, ConvIn{}, tq, tk, tv);
  return cudaGetLastError();
}

template <typename T>
cudaError_t run_state_store(const gdn_chunk_args& a, const Work& w0, uint8_t* hs, uint8_t* vn, cudaStream_t s) {
  constexpr bool kF16 = std::is_same<T, __half>::value;
  const int64_t ttot = a.B * a.T;
  if (ttot == 0) return cudaSuccess;
  Work w = w0;
  w.hs_img = hs;
  w.vn_img = vn;
  const float scale = a.scale > 0.f ? a.scale : 1.f / sqrtf(static_cast<float>(a.K));
  CUtensorMap tq, tk;
  cudaError_t e;
  if ((e = make_map(&tq, a.q, a.H, ttot, kF16, a.q_token_stride)) != cudaSuccess) return e;
  if ((e = make_map(&tk, a.k, a.H, ttot, kF16, a.k_token_stride)) != cudaSuccess) return e;
  LaunchHooks hk(nullptr, 0);
  return launch_state3<T, 32, true>(a, w, scale, tq, tk, s, hk);
}

cudaError_t launch_state_store(const gdn_chunk_args& a, const Work& w, uint8_t* hs, uint8_t* vn, cudaStream_t s) {
  return a.qkv_dtype == GDN_F16 ? run_state_store<__half>(a, w, hs, vn, s)
                                : run_state_store<__nv_bfloat16>(a, w, hs, vn, s);
}

cudaError_t launch_wy_only(const gdn_chunk_args& a, void* ws, cudaStream_t s, Work& w, float* gc_out) {
  return a.qkv_dtype == GDN_F16 ? run_wy_only<__half>(a, ws, s, w, gc_out)
                                : run_wy_only<__nv_bfloat16>(a, ws, s, w, gc_out);
}

}  // namespace tc

bool tc_path_applies(const gdn_chunk_args& a) {
  return (a.qkv_dtype == GDN_BF16 || a.qkv_dtype == GDN_F16) && a.K == tc::D && a.V == tc::D &&
         a.B * a.T < (int64_t(1) << 31);
}

size_t tc_workspace_bytes(const gdn_chunk_args& a) { return tc::plan(a).total; }
size_t tc_conv_workspace_bytes(const gdn_chunk_args& a) { return tc::plan(a, true).total; }

cudaError_t launch_chunk_tc(const gdn_chunk_args& a, cudaStream_t s, int64_t stall_chunk,
                            long long stall_limit, const gdn_conv1d_fn_args* conv) {
  return a.qkv_dtype == GDN_F16 ? tc::run<__half>(a, s, stall_chunk, stall_limit, conv)
                                : tc::run<__nv_bfloat16>(a, s, stall_chunk, stall_limit, conv);
}

}  // namespace gdn
