// Shared device helpers for the GDN kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_b200.h"

namespace gdn {

constexpr int kChunk = 64;  // chunk length of the WY form (reference BT = 64)

// ---- element conversion ----------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Load 4 consecutive elements as floats (address aligned to 4 elements).
template <typename T> __device__ __forceinline__ float4 load4(const T* p);
template <> __device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <> __device__ __forceinline__ float4 load4<__half>(const __half* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&u.x);
  __half2 b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

// Streaming 128-bit state traffic: read once, write once.
__device__ __forceinline__ float4 ld_stream(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

__device__ __forceinline__ int64_t load_index(const void* p, int dtype, int64_t i) {
  return dtype == GDN_I64 ? static_cast<const int64_t*>(p)[i]
                          : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// Sequence bounds: packed varlen (cu_seqlens) or equal-length batch.
__device__ __forceinline__ void seq_bounds(const void* cu, int cu_dtype, int64_t n,
                                           int64_t T, int64_t& bos, int64_t& eos) {
  if (cu) {
    bos = load_index(cu, cu_dtype, n);
    eos = load_index(cu, cu_dtype, n + 1);
  } else {
    bos = n * T;
    eos = bos + T;
  }
}

// Map a global chunk id to (sequence, local chunk) by binary search over the
// per-sequence chunk offsets (chunk_offsets[N] = total chunks).
__device__ __forceinline__ bool locate_chunk(const int64_t* chunk_offsets, int64_t N,
                                             int64_t c, int64_t& n, int64_t& lc) {
  if (c >= chunk_offsets[N]) return false;
  int64_t lo = 0, hi = N;  // invariant: offsets[lo] <= c < offsets[hi]
  while (hi - lo > 1) {
    int64_t mid = (lo + hi) >> 1;
    if (chunk_offsets[mid] <= c) lo = mid; else hi = mid;
  }
  n = lo;
  lc = c - chunk_offsets[lo];
  return true;
}

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// ---- device error word -----------------------------------------------------
// int32[4]: code, site, block (linear CTA id, or the sequence for a slot
// error), info (thread, or the offending index).  The first failure of a
// call wins (compare-and-swap on the code); later ones are dropped.
enum ErrCode { kErrWaitTimeout = 1, kErrSlotRange = 2 };
enum ErrSite {
  kSiteWyLoad = 1, kSiteWyMma1 = 2, kSiteWyMma2 = 3,       // tc_wy_kernel
  kSiteStLoad = 4, kSiteStMma1 = 5, kSiteStMma2 = 6,       // tc_state3_kernel
  kSiteDecodeRelease = 7, kSiteDecodeLoad = 8,             // decode_stream_kernel waits
  kSiteSlotInitial = 9, kSiteSlotFinal = 10,               // state index >= num_slots
  kSiteFzReady = 11                                        // tc_fused_kernel: stage-ready wait
};

__device__ __forceinline__ void record_device_error(int* err, int code, int site, int block, int info) {
  if (err && atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = block;
    err[3] = info;
    __threadfence();
  }
}
__device__ __forceinline__ int linear_block_id() {
  return static_cast<int>(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
}

template <int W>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

}  // namespace gdn
