// Arithmetic of the causal depthwise conv1d shared by the standalone conv
// kernels (gdn_conv.cu) and the prefill that applies the conv as it loads
// its tiles (gdn_chunk_tc.cu), so both produce the same bits:
//   y = bias + w_0 x_{t-W+1} + ... + w_{W-1} x_t   (fp32, taps in this order)
//   y = silu(y)                                     (optional)
// then rounded to nearest even in the output dtype.

#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

namespace gdn {
namespace conv {

// y * sigmoid(y) with the hardware exponential and divide (a few ulp).
__device__ __forceinline__ float silu(float y) { return __fdividef(y, 1.f + __expf(-y)); }

// For 16-bit outputs: y * sigmoid(y) = h + h * tanh(h) with h = y / 2, one
// special-function instruction (tanh.approx, relative error about 2^-11,
// under half an output ulp of bf16 and at the half-ulp of fp16).
__device__ __forceinline__ float silu16(float y) {
  const float h = 0.5f * y;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

// SiLU over VEC lanes: silu16 for 16-bit outputs with the halving and the
// final FMA on packed fp32 pairs (same bits as lane by lane), silu for fp32.
template <typename T, int VEC>
__device__ __forceinline__ void silu_vec(float* acc) {
  if constexpr (sizeof(T) == 2 && VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      const float2 h = __fmul2_rn(make_float2(acc[e], acc[e + 1]), make_float2(0.5f, 0.5f));
      float t0, t1;
      asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(h.x));
      asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(h.y));
      const float2 r = __ffma2_rn(h, make_float2(t0, t1), h);
      acc[e] = r.x;
      acc[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = sizeof(T) == 2 ? silu16(acc[e]) : silu(acc[e]);
  }
}

// acc += w * x over VEC lanes, two lanes per packed fp32 FMA when VEC is even.
template <int VEC>
__device__ __forceinline__ void fma_vec(float* acc, const float* w, const float* x) {
  if constexpr (VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      const float2 r = __ffma2_rn(make_float2(w[e], w[e + 1]), make_float2(x[e], x[e + 1]),
                                  make_float2(acc[e], acc[e + 1]));
      acc[e] = r.x;
      acc[e + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = fmaf(w[e], x[e], acc[e]);
  }
}

// Two 16-bit values (bf16 or fp16 bits, the first in the low half) as fp32.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (std::is_same<T, __half>::value) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  } else {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
}

// Two channels, width 4: bias + w0 x_{t-3} + w1 x_{t-2} + w2 x_{t-1} + w3 x_t
// (each w_i the taps of the two channels), then SiLU when `act`, rounded to T
// and packed (first channel in the low half).  Lane by lane the same fp32
// operations as the standalone kernels' fma_vec / silu_vec.
template <typename T>
__device__ __forceinline__ uint32_t conv2_w4(const float2 (&w)[4], float2 bias, float2 x0, float2 x1, float2 x2,
                                             float2 x3, bool act) {
  float2 a = __ffma2_rn(w[0], x0, bias);
  a = __ffma2_rn(w[1], x1, a);
  a = __ffma2_rn(w[2], x2, a);
  a = __ffma2_rn(w[3], x3, a);
  if (act) {
    float v[2] = {a.x, a.y};
    silu_vec<T, 2>(v);
    a = make_float2(v[0], v[1]);
  }
  if constexpr (std::is_same<T, __half>::value) {
    const __half2 h = __floats2half2_rn(a.x, a.y);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a.x, a.y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

}  // namespace conv
}  // namespace gdn
