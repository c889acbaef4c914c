// Causal depthwise conv1d (the short convolution in front of the GDN layer),
// the three reference ops behind torch_mlu_ops.triton_ops:
//   causal_conv1d       -> triton/conv/ops.py:35-99,   kernels.py:24-153
//   causal_conv1d_fn    -> triton/conv/ops.py:101-349, kernels.py:157-609
//   causal_conv1d_update-> triton/conv/ops.py:584-644, kernels.py:850-934
//
// All three are HBM streams (W <= 4 taps per channel), so the kernels are
// built for bandwidth, not tensor cores:
//   * channel-last tiles: a thread owns one 16-byte vector of channels
//     (8 x bf16/f16 or 4 x f32) and walks a 64-token tile, so every warp load
//     is 512 contiguous bytes; the W-1 previous inputs stay in registers and
//     each input is read once (plus a W-1 token halo per tile);
//   * tiles run over the flat token range and find their sequence by binary
//     search in cu_seqlens / query_start_loc on the device (no host sync);
//     at a sequence start the window is refilled from the initial state (or
//     zeros), so tiles may straddle sequences;
//   * the vLLM cache update (each sequence's last W-1 tokens into its line)
//     is a second small kernel, so no tile reads a line another tile has
//     already overwritten (the reference orders this inside one program);
//   * the decode update is one thread per channel.
// Accumulation is fp32; outputs are rounded to nearest even.

#include "conv_math.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>

namespace gdn {
namespace conv {

constexpr int kTT = 64;        // tokens per tile
constexpr int kU = 8;          // tokens loaded ahead per thread (vector path)
constexpr int kThreads = 128;  // threads per CTA (each owns one channel vector)
constexpr int kMaxW = 16;

__device__ __forceinline__ float ld_any(const void* p, int dtype, int64_t i) {
  if (dtype == GDN_F32) return static_cast<const float*>(p)[i];
  if (dtype == GDN_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void st_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == GDN_F32) static_cast<float*>(p)[i] = v;
  else if (dtype == GDN_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

// VEC consecutive elements <-> floats; one 128-bit access when VEC fills 16 B.
template <typename T, int VEC>
__device__ __forceinline__ void ldv(const T* p, float* v) {
  if constexpr (VEC * sizeof(T) == 16) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = to_f<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = to_f<T>(p[i]);
  }
}
template <typename T, int VEC>
__device__ __forceinline__ void stv(T* p, const float* v) {
  if constexpr (VEC * sizeof(T) == 16 && sizeof(T) == 2) {  // two lanes per rounding instruction
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[i], v[i + 1]);
        w[i / 2] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 b = __floats2half2_rn(v[i], v[i + 1]);
        w[i / 2] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    *reinterpret_cast<uint4*>(p) = u;
  } else if constexpr (VEC * sizeof(T) == 16) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < VEC; ++i) e[i] = from_f<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = from_f<T>(v[i]);
  }
}

struct FwdParams {
  const void* x;
  void* y;
  const void* residual;  // fla only, [total, D] contiguous
  const void* weight;    // [D, W]
  const void* bias;      // [D]
  const void* init;      // fla: initial_state [N, D, W]; fn: conv_states
  const void* cu;        // [nseq + 1] or null (fla equal-length batch)
  const void* cache_indices;
  const uint8_t* has_init;
  int64_t total, D, T, nseq;
  int64_t sx, sy;          // token strides of x, y (elements)
  int64_t st_seq, st_tok;  // fn: conv_states strides (elements)
  int64_t pad_slot, null_block;
  int64_t nblk, upc;  // channel blocks; tokens per CTA run
  int has_null, fn_mode;
  int W, w_dtype, init_dtype, cu_dtype, idx_dtype, act;
  // fn prefix caching (apc_last non-null): 2-D cache_indices, block states
  const void *apc_first, *apc_last, *apc_init, *apc_ncomp;
  int64_t ci_stride, bsz;
  int apc_dtype;
};

// Cache line holding sequence n's initial window (fn mode).
__device__ __forceinline__ int64_t input_line(const FwdParams& p, int64_t n) {
  if (!p.cache_indices) return n;
  const int64_t col = p.apc_last ? load_index(p.apc_init, p.apc_dtype, n) : 0;
  return load_index(p.cache_indices, p.idx_dtype, n * p.ci_stride + col);
}

// Sequence n with cu[n] <= t < cu[n+1] (the last such n when empty
// sequences share the boundary).
__device__ __forceinline__ void find_seq(const FwdParams& p, int64_t t, int64_t& n, int64_t& bos,
                                         int64_t& eos) {
  if (!p.cu) {
    n = t / p.T;
    bos = n * p.T;
    eos = bos + p.T;
    return;
  }
  int64_t lo = 0, hi = p.nseq;  // cu[lo] <= t < cu[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (load_index(p.cu, p.cu_dtype, mid) <= t) lo = mid; else hi = mid;
  }
  n = lo;
  bos = load_index(p.cu, p.cu_dtype, n);
  eos = load_index(p.cu, p.cu_dtype, n + 1);
}

// One thread's channel vector [c, c + VEC) walking a run of tokens: the
// weights, the W-1 previous inputs and the current sequence.  enter(t)
// moves to the sequence holding token t and, at a sequence start, fills the
// window from the sequence's own inputs, its initial state or zeros (or
// marks a PAD / null-block sequence, whose outputs are zeros); step(t, x)
// writes output t from input x and shifts the window.
template <typename T, int VEC, int KW>
struct ConvLane {
  static constexpr int WM = KW > 0 ? KW : kMaxW;
  float w[WM][VEC], bias[VEC];
  float win[WM][VEC];  // win[j] = input at token t - (W-1) + j, j < W-1
  int w_rt;            // the width when it is not a template constant
  int64_t c, n, bos, eos;
  bool fresh, skip;

  __device__ __forceinline__ void init(const FwdParams& p, int64_t c_, int64_t t0) {
    w_rt = p.W;
    const int W = KW > 0 ? KW : w_rt;
    c = c_;
    bool loaded = false;
    if constexpr (VEC == 8 && KW > 0) {
      // 16-bit taps of channels c..c+7 are 8 * KW contiguous elements: KW 16-byte loads
      const bool h16 = p.w_dtype == GDN_BF16 || p.w_dtype == GDN_F16;
      const uintptr_t wa = reinterpret_cast<uintptr_t>(p.weight) + static_cast<uintptr_t>(c) * KW * 2;
      const uintptr_t ba = reinterpret_cast<uintptr_t>(p.bias) + static_cast<uintptr_t>(c) * 2;
      if (h16 && (wa & 15) == 0 && (!p.bias || (ba & 15) == 0)) {
        uint4 raw[KW + 1];
#pragma unroll
        for (int r = 0; r < KW; ++r) raw[r] = __ldg(reinterpret_cast<const uint4*>(wa) + r);
        raw[KW] = p.bias ? __ldg(reinterpret_cast<const uint4*>(ba)) : make_uint4(0u, 0u, 0u, 0u);
        const uint16_t* u = reinterpret_cast<const uint16_t*>(raw);
        auto f16 = [&](uint16_t b) {
          return p.w_dtype == GDN_BF16 ? __uint_as_float(static_cast<uint32_t>(b) << 16)
                                       : __half2float(__ushort_as_half(b));
        };
#pragma unroll
        for (int i = 0; i < KW; ++i)
#pragma unroll
          for (int e = 0; e < 8; ++e) w[i][e] = f16(u[e * KW + i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) bias[e] = f16(u[KW * 8 + e]);
        loaded = true;
      }
    }
    if (!loaded) {
#pragma unroll
      for (int i = 0; i < WM; ++i)
#pragma unroll
        for (int e = 0; e < VEC; ++e) w[i][e] = i < W ? ld_any(p.weight, p.w_dtype, (c + e) * W + i) : 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) bias[e] = p.bias ? ld_any(p.bias, p.w_dtype, c + e) : 0.f;
    }
    find_seq(p, t0, n, bos, eos);
    fresh = true;
    skip = false;
  }

  __device__ __forceinline__ void enter(const FwdParams& p, int64_t t) {
    while (t >= eos) {  // next (possibly empty) sequence
      ++n;
      bos = eos;
      eos = p.cu ? load_index(p.cu, p.cu_dtype, n + 1) : bos + p.T;
      fresh = true;
    }
    if (!fresh) return;
    fresh = false;
    const int W = KW > 0 ? KW : w_rt;
    const T* x = static_cast<const T*>(p.x);
    bool hinit;
    int64_t line = n;
    if (p.fn_mode) {
      line = input_line(p, n);
      skip = (p.has_null && line == p.null_block) || line == p.pad_slot;
      hinit = p.has_init && p.has_init[n];
    } else {
      hinit = p.init != nullptr;
    }
#pragma unroll
    for (int j = 0; j < WM - 1; ++j) {
      if (j >= W - 1) break;
      const int64_t u = t - (W - 1) + j;
      if (u >= bos) {
        ldv<T, VEC>(x + u * p.sx + c, win[j]);
      } else if (hinit && !skip) {
        const int64_t local = u - bos;  // -(W-1) .. -1
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          win[j][e] = p.fn_mode
              ? ld_any(p.init, p.init_dtype, line * p.st_seq + (local + W - 1) * p.st_tok + c + e)
              : ld_any(p.init, p.init_dtype, (n * p.D + c + e) * W + local + W);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) win[j][e] = 0.f;
      }
    }
  }

  __device__ __forceinline__ void step(const FwdParams& p, int64_t t, const float* xv) {
    T* y = static_cast<T*>(p.y);
    const int W = KW > 0 ? KW : w_rt;
    float acc[VEC];
    if (skip) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = bias[e];
#pragma unroll
      for (int j = 0; j < WM - 1; ++j)
        if (j < W - 1) fma_vec<VEC>(acc, w[j], win[j]);
      fma_vec<VEC>(acc, w[W - 1], xv);
      if (p.act == GDN_ACT_SILU) silu_vec<T, VEC>(acc);
      if (p.residual) {
        float r[VEC];
        ldv<T, VEC>(static_cast<const T*>(p.residual) + t * p.D + c, r);
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] += r[e];
      }
    }
    stv<T, VEC>(y + t * p.sy + c, acc);
#pragma unroll
    for (int j = 0; j + 1 < WM - 1; ++j)
      if (j + 1 < W - 1)
#pragma unroll
        for (int e = 0; e < VEC; ++e) win[j][e] = win[j + 1][e];
    if (W >= 2)
#pragma unroll
      for (int e = 0; e < VEC; ++e) win[W - 2][e] = xv[e];
  }
};

// CTA b owns channel block b % nblk over the (b / nblk)-th equal run of
// tokens, so the nblk CTAs of one run (adjacent in launch order) stream
// whole token rows together.  Inputs come straight from global memory, kU
// (or 4) independent loads in flight per thread.
template <typename T, int VEC, int KW>
__global__ void __launch_bounds__(kThreads, 3) conv_fwd_kernel(const FwdParams p) {
  const int64_t cb = blockIdx.x % p.nblk, share = blockIdx.x / p.nblk;
  const int64_t t0 = share * p.upc;
  const int64_t t1 = min64(p.total, t0 + p.upc);
  const int64_t c = (cb * kThreads + threadIdx.x) * VEC;
  if (c >= p.D || t0 >= t1) return;
  const T* x = static_cast<const T*>(p.x);
  ConvLane<T, VEC, KW> L;
  L.init(p, c, t0);
  int64_t t = t0;
  while (t < t1) {
    L.enter(p, t);
    const int64_t end = min64(t1, L.eos);
    if (VEC * sizeof(T) == 16 && t + kU <= end) {  // kU independent loads in flight, kept packed
      if constexpr (VEC * sizeof(T) == 16) {
        uint4 raw[kU];
#pragma unroll
        for (int k = 0; k < kU; ++k) raw[k] = __ldg(reinterpret_cast<const uint4*>(x + (t + k) * p.sx + c));
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          float xv[VEC];
          const T* e = reinterpret_cast<const T*>(&raw[k]);
#pragma unroll
          for (int i = 0; i < VEC; ++i) xv[i] = to_f<T>(e[i]);
          L.step(p, t + k, xv);
        }
      }
      t += kU;
    } else if (t + 4 <= end) {  // four loads in flight
      float xv[4][VEC];
#pragma unroll
      for (int k = 0; k < 4; ++k) ldv<T, VEC>(x + (t + k) * p.sx + c, xv[k]);
#pragma unroll
      for (int k = 0; k < 4; ++k) L.step(p, t + k, xv[k]);
      t += 4;
    } else {
      float xv[VEC];
      ldv<T, VEC>(x + t * p.sx + c, xv);
      L.step(p, t, xv);
      ++t;
    }
  }
}

// vLLM cache update: line <- the last W-1 entries of [old line (or zeros),
// the sequence's inputs] (kernels.py:381-484).  Runs after conv_fwd_kernel.
template <typename T, int VEC>
__global__ void __launch_bounds__(kThreads) conv_state_kernel(const FwdParams p) {
  const int64_t s = blockIdx.x;
  const int64_t c = (static_cast<int64_t>(blockIdx.y) * kThreads + threadIdx.x) * VEC;
  if (c >= p.D) return;
  const int sl = p.W - 1;
  const int64_t line = input_line(p, s);
  if ((p.has_null && line == p.null_block) || line == p.pad_slot) return;
  const bool hinit = p.has_init && p.has_init[s];
  const int64_t bos = load_index(p.cu, p.cu_dtype, s), L = load_index(p.cu, p.cu_dtype, s + 1) - bos;
  if (L <= 0) return;  // an empty sequence runs no program and leaves its line alone
  // final state: to the scheduled last block (prefix caching) when the
  // sequence covers W-1 inputs, else shifted within the initial line
  const int64_t out_line = p.apc_last && L >= sl
      ? load_index(p.cache_indices, p.idx_dtype, s * p.ci_stride + load_index(p.apc_last, p.apc_dtype, s))
      : line;
  const T* x = static_cast<const T*>(p.x);
  float nv[3][VEC];  // W <= 4
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    if (j >= sl) break;
    const int64_t u = L + j;  // index into [line ; inputs]
    if (u < sl) {
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        nv[j][e] = hinit ? ld_any(p.init, p.init_dtype, line * p.st_seq + u * p.st_tok + c + e) : 0.f;
    } else {
      ldv<T, VEC>(x + (bos + u - sl) * p.sx + c, nv[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    if (j >= sl) break;
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      st_any(const_cast<void*>(p.init), p.init_dtype, out_line * p.st_seq + j * p.st_tok + c + e, nv[j][e]);
  }
  if (!p.apc_last) return;
  // prefix caching: the W-1 inputs before each block-aligned block end, one
  // block per 64-token chunk after the first (kernels.py:519-554)
  const int64_t first = load_index(p.apc_first, p.apc_dtype, s);
  const int64_t nb = load_index(p.apc_last, p.apc_dtype, s) - first;
  const int64_t B = p.bsz;
  const int64_t comp_off = B - load_index(p.apc_ncomp, p.apc_dtype, s) % B;
  const int64_t end_off = (L - comp_off) % B;  // remainder with the dividend's sign
  const int64_t last_full = bos + L - end_off - (end_off == 0 ? B : 0);
  const int64_t nchunks = (L + 63) / 64;
  for (int64_t j = 0; j < nb && j + 1 < nchunks; ++j) {
    const int64_t start = last_full - (nb - j - 1) * B - sl;
    const int64_t bl = load_index(p.cache_indices, p.idx_dtype, s * p.ci_stride + first + j);
    for (int u = 0; u < sl; ++u) {
      float v[VEC];
      if (start + u >= 0) {
        ldv<T, VEC>(x + (start + u) * p.sx + c, v);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        st_any(const_cast<void*>(p.init), p.init_dtype, bl * p.st_seq + u * p.st_tok + c + e, v[e]);
    }
  }
}

struct UpdParams {
  const void* x;
  void* cache;
  const void* residual;
  const void* weight;
  const void* bias;
  void* y;
  int64_t sxn, N, D;
  int W, cache_dtype, w_dtype, act;
};

template <typename T, int KW>
__global__ void __launch_bounds__(kThreads) conv_update_kernel(const UpdParams p) {
  constexpr int WM = KW > 0 ? KW : kMaxW;
  const int W = KW > 0 ? KW : p.W;
  const int64_t n = blockIdx.y;
  const int64_t d = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (d >= p.D) return;
  const float xv = to_f<T>(static_cast<const T*>(p.x)[n * p.sxn + d]);
  const int64_t cb = (n * p.D + d) * W;
  float win[WM];
#pragma unroll
  for (int j = 0; j < WM; ++j) {
    if (j >= W) break;
    win[j] = !p.cache ? 0.f : j + 1 < W ? ld_any(p.cache, p.cache_dtype, cb + j + 1) : xv;
  }
  float acc = p.bias ? ld_any(p.bias, p.w_dtype, d) : 0.f;
#pragma unroll
  for (int j = 0; j < WM; ++j) {
    if (j >= W) break;
    acc = fmaf(win[j], p.weight ? ld_any(p.weight, p.w_dtype, d * W + j) : 1.f, acc);
  }
  if (p.act == GDN_ACT_SILU) acc = sizeof(T) == 2 ? silu16(acc) : silu(acc);
  if (p.residual) acc += to_f<T>(static_cast<const T*>(p.residual)[n * p.D + d]);
  static_cast<T*>(p.y)[n * p.D + d] = from_f<T>(acc);
  if (p.cache)
#pragma unroll
    for (int j = 0; j < WM; ++j) {
      if (j >= W) break;
      st_any(p.cache, p.cache_dtype, cb + j, win[j]);
    }
}

// Vectorised decode update for the common layout (x, cache, weight, bias,
// residual, y all of type T; D a multiple of 8; 16-byte aligned): a thread
// owns 8 consecutive channels, whose cache rows, weights, inputs and
// outputs are contiguous runs moved with 128-bit accesses.
template <typename T, int KW>
__global__ void __launch_bounds__(kThreads) conv_update_vec_kernel(const UpdParams p) {
  static_assert(sizeof(T) == 2, "16-bit types");
  constexpr int C8 = 8;                // channels per thread
  constexpr int NV = C8 * KW / 8;      // 16-byte vectors in the thread's cache run
  const int64_t n = blockIdx.y;
  const int64_t d = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * C8;
  if (d >= p.D) return;
  const T* xs = static_cast<const T*>(p.x) + n * p.sxn + d;
  T* cache = static_cast<T*>(p.cache) + (n * p.D + d) * KW;
  const T* wt = static_cast<const T*>(p.weight) + d * KW;
  float xv[C8], cf[C8 * KW], wf[C8 * KW], acc[C8];
  ldv<T, C8>(xs, xv);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    ldv<T, 8>(cache + v * 8, cf + v * 8);
    ldv<T, 8>(wt + v * 8, wf + v * 8);
  }
  if (p.bias) ldv<T, C8>(static_cast<const T*>(p.bias) + d, acc);
  else
#pragma unroll
    for (int e = 0; e < C8; ++e) acc[e] = 0.f;
#pragma unroll
  for (int e = 0; e < C8; ++e) {
#pragma unroll
    for (int j = 0; j < KW; ++j) {
      const float v = j + 1 < KW ? cf[e * KW + j + 1] : xv[e];
      cf[e * KW + j] = v;  // shifted window, in place
      acc[e] = fmaf(v, wf[e * KW + j], acc[e]);
    }
    if (p.act == GDN_ACT_SILU) acc[e] = silu16(acc[e]);
  }
  if (p.residual) {
    float r[C8];
    ldv<T, C8>(static_cast<const T*>(p.residual) + n * p.D + d, r);
#pragma unroll
    for (int e = 0; e < C8; ++e) acc[e] += r[e];
  }
  stv<T, C8>(static_cast<T*>(p.y) + n * p.D + d, acc);
#pragma unroll
  for (int v = 0; v < NV; ++v) stv<T, 8>(cache + v * 8, cf + v * 8);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return set_last_error(code, "%s", buf);
}
bool fdtype_ok(int d) { return d == GDN_F32 || d == GDN_BF16 || d == GDN_F16; }
bool idtype_ok(int d) { return d == GDN_I32 || d == GDN_I64; }
int esize(int d) { return d == GDN_F32 ? 4 : 2; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Resident CTAs of conv_fwd_kernel<T, VEC, KW> on this device (queried once
// per instantiation: the static lives in each instantiation of this template).
template <typename T, int VEC, int KW>
int resident_ctas() {
  static int cached = 0;
  if (!cached) {
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv_fwd_kernel<T, VEC, KW>, kThreads, 0);
    cached = sms * (per_sm > 0 ? per_sm : 1);
  }
  return cached;
}

template <typename T, int VEC, int KW>
cudaError_t launch_fwd_w(FwdParams p, cudaStream_t s) {
  auto kern = conv_fwd_kernel<T, VEC, KW>;
  p.nblk = (p.D + VEC * kThreads - 1) / (VEC * kThreads);
  // as many equal token runs (of at least kTT tokens) as the resident CTAs
  // cover with every channel block: one wave, no tail
  const int64_t shares = std::max<int64_t>(
      1, std::min<int64_t>(resident_ctas<T, VEC, KW>() / std::max<int64_t>(p.nblk, 1), (p.total + kTT - 1) / kTT));
  p.upc = (p.total + shares - 1) / shares;  // tokens per run
  const int64_t grid = p.nblk * shares;
  note_launch();
  kern<<<static_cast<unsigned>(grid), kThreads, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T, int VEC>
cudaError_t launch_fwd_v(const FwdParams& p, cudaStream_t s) {
  cudaError_t e;
  switch (p.W) {
    case 2: e = launch_fwd_w<T, VEC, 2>(p, s); break;
    case 3: e = launch_fwd_w<T, VEC, 3>(p, s); break;
    case 4: e = launch_fwd_w<T, VEC, 4>(p, s); break;
    default: e = launch_fwd_w<T, VEC, 0>(p, s); break;
  }
  if (e != cudaSuccess || !p.fn_mode) return e;
  const dim3 g2(static_cast<unsigned>(p.nseq),
                static_cast<unsigned>((p.D + VEC * kThreads - 1) / (VEC * kThreads)));
  note_launch();
  conv_state_kernel<T, VEC><<<g2, kThreads, 0, s>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_fwd(const FwdParams& p, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = p.D % V == 0 && p.sx % V == 0 && p.sy % V == 0 && aligned16(p.x) && aligned16(p.y) &&
                   (!p.residual || aligned16(p.residual));
  return vec ? launch_fwd_v<T, V>(p, s) : launch_fwd_v<T, 1>(p, s);
}

cudaError_t dispatch_fwd(const FwdParams& p, int x_dtype, cudaStream_t s) {
  if (x_dtype == GDN_F32) return launch_fwd<float>(p, s);
  if (x_dtype == GDN_BF16) return launch_fwd<__nv_bfloat16>(p, s);
  return launch_fwd<__half>(p, s);
}

template <typename T>
cudaError_t launch_update(const UpdParams& p, int x_dtype, cudaStream_t s) {
  if constexpr (sizeof(T) == 2) {
    const bool vec = p.cache && p.weight && p.cache_dtype == x_dtype && p.w_dtype == x_dtype &&
                     p.W >= 2 && p.W <= 4 && p.D % 8 == 0 && p.sxn % 8 == 0 && aligned16(p.x) &&
                     aligned16(p.cache) && aligned16(p.weight) && aligned16(p.y) &&
                     (!p.bias || aligned16(p.bias)) && (!p.residual || aligned16(p.residual));
    if (vec) {
      const dim3 grid(static_cast<unsigned>((p.D / 8 + kThreads - 1) / kThreads), static_cast<unsigned>(p.N));
      note_launch();
      if (p.W == 4) conv_update_vec_kernel<T, 4><<<grid, kThreads, 0, s>>>(p);
      else if (p.W == 3) conv_update_vec_kernel<T, 3><<<grid, kThreads, 0, s>>>(p);
      else conv_update_vec_kernel<T, 2><<<grid, kThreads, 0, s>>>(p);
      return cudaGetLastError();
    }
  }
  const dim3 grid(static_cast<unsigned>((p.D + kThreads - 1) / kThreads), static_cast<unsigned>(p.N));
  note_launch();
  switch (p.W) {
    case 2: conv_update_kernel<T, 2><<<grid, kThreads, 0, s>>>(p); break;
    case 3: conv_update_kernel<T, 3><<<grid, kThreads, 0, s>>>(p); break;
    case 4: conv_update_kernel<T, 4><<<grid, kThreads, 0, s>>>(p); break;
    default: conv_update_kernel<T, 0><<<grid, kThreads, 0, s>>>(p); break;
  }
  return cudaGetLastError();
}

}  // namespace conv
}  // namespace gdn

using namespace gdn;
using namespace gdn::conv;

extern "C" GDN_API int gdn_causal_conv1d_fwd(const gdn_conv1d_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  if (!a->x || !a->weight || !a->y) return fail(GDN_ERR_INVALID, "x, weight and y must be non-null");
  if (a->B <= 0 || a->T < 0 || a->D <= 0) return fail(GDN_ERR_INVALID, "bad shape B=%lld T=%lld D=%lld",
                                                      (long long)a->B, (long long)a->T, (long long)a->D);
  if (a->W < 1 || a->W > kMaxW) return fail(GDN_ERR_UNSUPPORTED, "kernel width W=%d outside [1, %d]", a->W, kMaxW);
  if (!fdtype_ok(a->x_dtype) || !fdtype_ok(a->w_dtype) || (a->initial_state && !fdtype_ok(a->state_dtype)))
    return fail(GDN_ERR_INVALID, "x, weight and state dtypes must be F32, BF16 or F16");
  if (a->activation != GDN_ACT_NONE && a->activation != GDN_ACT_SILU)
    return fail(GDN_ERR_INVALID, "activation must be GDN_ACT_NONE or GDN_ACT_SILU");
  int64_t nseq = a->B;
  if (a->cu_seqlens) {
    if (!idtype_ok(a->cu_dtype)) return fail(GDN_ERR_INVALID, "cu_seqlens dtype must be I32 or I64");
    if (a->B != 1) return fail(GDN_ERR_INVALID, "cu_seqlens requires B == 1 (got B=%lld)", (long long)a->B);
    if (a->N < 1) return fail(GDN_ERR_INVALID, "cu_seqlens needs N >= 1 sequences");
    nseq = a->N;
  } else if (a->N != a->B) {
    return fail(GDN_ERR_INVALID, "without cu_seqlens N must equal B (N=%lld B=%lld)", (long long)a->N,
                (long long)a->B);
  }
  FwdParams p{};
  p.x = a->x; p.y = a->y; p.residual = a->residual; p.weight = a->weight; p.bias = a->bias;
  p.init = a->initial_state; p.cu = a->cu_seqlens; p.cu_dtype = a->cu_dtype;
  p.total = a->B * a->T; p.D = a->D; p.T = a->T; p.nseq = nseq;
  p.sx = a->D; p.sy = a->D;
  p.W = a->W; p.w_dtype = a->w_dtype; p.init_dtype = a->state_dtype; p.act = a->activation;
  p.pad_slot = INT64_MIN;
  if (p.total == 0) return GDN_OK;
  cudaError_t e = dispatch_fwd(p, a->x_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_causal_conv1d_fwd: %s", cudaGetErrorString(e));
  return GDN_OK;
}

namespace gdn {
namespace conv {

// Checks causal_conv1d_fn's arguments and fills its kernel parameters;
// GDN_OK or an error code with the message set.  `fused`: the conv is
// applied inside the prefill, which has no `out` tensor.
int fn_params(const gdn_conv1d_fn_args* a, FwdParams& p, bool fused) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  if (!a->x || (!fused && !a->out) || !a->weight || !a->conv_states || !a->query_start_loc)
    return fail(GDN_ERR_INVALID, fused ? "x, weight, conv_states and query_start_loc must be non-null"
                                       : "x, out, weight, conv_states and query_start_loc must be non-null");
  if (a->batch < 0 || a->dim <= 0 || a->total_tokens < 0 || a->num_cache_lines < 0)
    return fail(GDN_ERR_INVALID, "bad shape batch=%lld dim=%lld total=%lld", (long long)a->batch,
                (long long)a->dim, (long long)a->total_tokens);
  if (a->W < 2 || a->W > 4) return fail(GDN_ERR_UNSUPPORTED, "kernel width W=%d outside [2, 4]", a->W);
  if (!fdtype_ok(a->x_dtype) || !fdtype_ok(a->w_dtype) || !fdtype_ok(a->state_dtype))
    return fail(GDN_ERR_INVALID, "x, weight and conv_states dtypes must be F32, BF16 or F16");
  if (!idtype_ok(a->qsl_dtype) || (a->cache_indices && !idtype_ok(a->idx_dtype)))
    return fail(GDN_ERR_INVALID, "query_start_loc and cache_indices dtypes must be I32 or I64");
  if (a->activation != GDN_ACT_NONE && a->activation != GDN_ACT_SILU)
    return fail(GDN_ERR_INVALID, "activation must be GDN_ACT_NONE or GDN_ACT_SILU");
  if (a->stride_x_token < a->dim || (!fused && a->stride_o_token < a->dim))
    return fail(GDN_ERR_INVALID, "token strides must be >= dim (channel-last layout)");
  p = FwdParams{};
  p.x = a->x; p.y = fused ? nullptr : a->out; p.weight = a->weight; p.bias = a->bias; p.init = a->conv_states;
  p.cu = a->query_start_loc; p.cu_dtype = a->qsl_dtype;
  p.cache_indices = a->cache_indices; p.idx_dtype = a->idx_dtype; p.has_init = a->has_initial_state;
  p.total = a->total_tokens; p.D = a->dim; p.nseq = a->batch;
  p.sx = a->stride_x_token; p.sy = fused ? a->dim : a->stride_o_token;
  p.st_seq = a->stride_state_seq; p.st_tok = a->stride_state_tok;
  p.pad_slot = a->pad_slot_id; p.null_block = a->null_block_id; p.has_null = a->has_null_block;
  p.fn_mode = 1; p.W = a->W; p.w_dtype = a->w_dtype; p.init_dtype = a->state_dtype; p.act = a->activation;
  p.ci_stride = a->cache_indices ? (a->stride_cache_indices > 0 ? a->stride_cache_indices : 1) : 0;
  if (a->block_idx_last) {
    if (!a->block_idx_first || !a->initial_state_idx || !a->num_computed_tokens || !a->cache_indices)
      return fail(GDN_ERR_INVALID, "prefix caching needs cache_indices and all four block arrays");
    if (!idtype_ok(a->apc_dtype)) return fail(GDN_ERR_INVALID, "block array dtype must be I32 or I64");
    if (a->block_size_to_align <= 0 || a->block_size_to_align % 64 != 0)
      return fail(GDN_ERR_INVALID, "block_size_to_align=%lld must be a positive multiple of 64",
                  (long long)a->block_size_to_align);
    p.apc_first = a->block_idx_first; p.apc_last = a->block_idx_last;
    p.apc_init = a->initial_state_idx; p.apc_ncomp = a->num_computed_tokens;
    p.apc_dtype = a->apc_dtype; p.bsz = a->block_size_to_align;
  }
  return GDN_OK;
}

}  // namespace conv

int check_conv_fn_args(const gdn_conv1d_fn_args* a) {
  conv::FwdParams p;
  return conv::fn_params(a, p, true);
}

// The cache-line update of causal_conv1d_fn alone (conv_state_kernel), for
// the prefill that applied the conv itself; runs after every reader of the
// initial lines.
cudaError_t launch_conv_fn_states(const gdn_conv1d_fn_args& a, cudaStream_t s) {
  conv::FwdParams p;
  if (conv::fn_params(&a, p, true) != GDN_OK) return cudaErrorInvalidValue;
  if (p.total == 0 || p.nseq == 0) return cudaSuccess;
  const int vec = 16 / conv::esize(a.x_dtype);
  const bool v = p.D % vec == 0 && p.sx % vec == 0 && conv::aligned16(p.x);
  const dim3 g2(static_cast<unsigned>(p.nseq),
                static_cast<unsigned>((p.D + (v ? vec : 1) * conv::kThreads - 1) / ((v ? vec : 1) * conv::kThreads)));
  note_launch();
  if (a.x_dtype == GDN_F16) {
    if (v) conv::conv_state_kernel<__half, 8><<<g2, conv::kThreads, 0, s>>>(p);
    else conv::conv_state_kernel<__half, 1><<<g2, conv::kThreads, 0, s>>>(p);
  } else if (a.x_dtype == GDN_BF16) {
    if (v) conv::conv_state_kernel<__nv_bfloat16, 8><<<g2, conv::kThreads, 0, s>>>(p);
    else conv::conv_state_kernel<__nv_bfloat16, 1><<<g2, conv::kThreads, 0, s>>>(p);
  } else {
    if (v) conv::conv_state_kernel<float, 4><<<g2, conv::kThreads, 0, s>>>(p);
    else conv::conv_state_kernel<float, 1><<<g2, conv::kThreads, 0, s>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace gdn

extern "C" GDN_API int gdn_causal_conv1d_fn(const gdn_conv1d_fn_args* a, void* stream) {
  FwdParams p;
  const int rc = fn_params(a, p, false);
  if (rc != GDN_OK) return rc;
  if (p.total == 0 || p.nseq == 0) return GDN_OK;
  cudaError_t e = dispatch_fwd(p, a->x_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_causal_conv1d_fn: %s", cudaGetErrorString(e));
  return GDN_OK;
}

extern "C" GDN_API int gdn_causal_conv1d_update(const gdn_conv1d_update_args* a, void* stream) {
  if (!a) return fail(GDN_ERR_INVALID, "null args");
  if (!a->x || !a->y) return fail(GDN_ERR_INVALID, "x and y must be non-null");
  if (a->N < 0 || a->D <= 0 || a->stride_x_n < a->D)
    return fail(GDN_ERR_INVALID, "bad shape N=%lld D=%lld stride=%lld", (long long)a->N, (long long)a->D,
                (long long)a->stride_x_n);
  if (a->W < 1 || a->W > kMaxW) return fail(GDN_ERR_UNSUPPORTED, "kernel width W=%d outside [1, %d]", a->W, kMaxW);
  if (!fdtype_ok(a->x_dtype) || ((a->weight || a->bias) && !fdtype_ok(a->w_dtype)) ||
      (a->cache && !fdtype_ok(a->cache_dtype)))
    return fail(GDN_ERR_INVALID, "x, weight and cache dtypes must be F32, BF16 or F16");
  if (a->activation != GDN_ACT_NONE && a->activation != GDN_ACT_SILU)
    return fail(GDN_ERR_INVALID, "activation must be GDN_ACT_NONE or GDN_ACT_SILU");
  if (a->N == 0) return GDN_OK;
  UpdParams p{};
  p.x = a->x; p.cache = a->cache; p.residual = a->residual; p.weight = a->weight; p.bias = a->bias; p.y = a->y;
  p.sxn = a->stride_x_n; p.N = a->N; p.D = a->D; p.W = a->W;
  p.cache_dtype = a->cache_dtype; p.w_dtype = a->w_dtype; p.act = a->activation;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = a->x_dtype == GDN_F32    ? launch_update<float>(p, a->x_dtype, s)
                  : a->x_dtype == GDN_BF16 ? launch_update<__nv_bfloat16>(p, a->x_dtype, s)
                                           : launch_update<__half>(p, a->x_dtype, s);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_causal_conv1d_update: %s", cudaGetErrorString(e));
  return GDN_OK;
}
