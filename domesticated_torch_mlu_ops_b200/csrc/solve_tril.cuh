// Blocked inverse of a 64 x 64 unit lower-triangular matrix in shared memory:
// T = (I + A)^-1 for strictly lower-triangular A (the solve_tril op,
// include/torch_mlu_ops.h:1052-1054; semantics of triton/fla/solve_tril.py:491-537).
//
// Recursive doubling over 16 / 32 / 64-row blocks:
//   1. the four 16 x 16 diagonal blocks by forward substitution (one thread
//      per column, the column in registers);
//   2. the 32 x 32 diagonal blocks: T_10 = -T_11 (A_10 T_00), likewise T_32;
//   3. the lower-left 32 x 32 block: T_lo,hi = -T_hi (A_hi,lo T_lo).
// Steps 2 and 3 are small products computed as register micro-tiles (one row
// or two rows by four columns per thread), so every thread carries four to
// eight independent FMA chains and reads T rows as float4.
#pragma once

namespace gdn {

constexpr int kTrilStride = 65;  // row stride (floats) of A
constexpr int kTS = 68;          // row stride (floats) of T: rows 16-byte aligned
constexpr int kZS = 36;          // row stride (floats) of the scratch Z
constexpr int kTrilScratch = 32 * kZS;  // floats of scratch

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void fma4(float4& acc, float a, float4 b) {
  acc.x = fmaf(a, b.x, acc.x);
  acc.y = fmaf(a, b.y, acc.y);
  acc.z = fmaf(a, b.z, acc.z);
  acc.w = fmaf(a, b.w, acc.w);
}

// A: [64][65], T: [64][68] (16-byte aligned), Z: kTrilScratch floats
// (16-byte aligned).  All threads of the block call this (blockDim.x >= 64);
// it ends with a __syncthreads.
__device__ __forceinline__ void solve_tril64(const float* __restrict__ A, float* __restrict__ T,
                                             float* __restrict__ Z) {
  const int tid = threadIdx.x, nt = blockDim.x;
  // 1. diagonal 16 x 16 blocks
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15, j = 16 * b + jj;
    const float* Ab = A + (16 * b) * kTrilStride + 16 * b;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == jj) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int m = 0; m + 1 < i; m += 2) {
        a0 = fmaf(Ab[i * kTrilStride + m], x[m], a0);
        a1 = fmaf(Ab[i * kTrilStride + m + 1], x[m + 1], a1);
      }
      if (i & 1) a0 = fmaf(Ab[i * kTrilStride + i - 1], x[i - 1], a0);
      if (i > jj) x[i] = -(a0 + a1);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) T[(16 * b + i) * kTS + j] = x[i];
  }
  for (int e = tid; e < 64 * 16; e += nt) {  // zero the blocks above the diagonal
    const int r = e >> 4, c = (e & 15) * 4;
    if ((r >> 4) < (c >> 4)) st4(T + r * kTS + c, make_float4(0.f, 0.f, 0.f, 0.f));
  }
  __syncthreads();
  // 2. T_10 = -T_11 (A_10 T_00) and T_32 = -T_33 (A_32 T_22)
  for (int o = tid; o < 128; o += nt) {
    const int blk = o >> 6, r = (o >> 2) & 15, cq = (o & 3) * 4;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) fma4(z, A[(rb + r) * kTrilStride + cb + m], ld4(T + (cb + m) * kTS + cb + cq));
    st4(Z + (blk * 16 + r) * kZS + cq, z);
  }
  __syncthreads();
  for (int o = tid; o < 128; o += nt) {
    const int blk = o >> 6, r = (o >> 2) & 15, cq = (o & 3) * 4;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) fma4(x, T[(rb + r) * kTS + rb + m], ld4(Z + (blk * 16 + m) * kZS + cq));
    st4(T + (rb + r) * kTS + cb + cq, make_float4(-x.x, -x.y, -x.z, -x.w));
  }
  __syncthreads();
  // 3. T[32:64, 0:32] = -T_hi (A[32:64, 0:32] T_lo)
  for (int o = tid; o < 128; o += nt) {
    const int r0 = (o >> 3) * 2, cq = (o & 7) * 4;
    float4 z0 = make_float4(0.f, 0.f, 0.f, 0.f), z1 = z0;
    const float* a0 = A + (32 + r0) * kTrilStride;
    const float* a1 = a0 + kTrilStride;
#pragma unroll 8
    for (int m = 0; m < 32; ++m) {
      const float4 t = ld4(T + m * kTS + cq);
      fma4(z0, a0[m], t);
      fma4(z1, a1[m], t);
    }
    st4(Z + r0 * kZS + cq, z0);
    st4(Z + (r0 + 1) * kZS + cq, z1);
  }
  __syncthreads();
  for (int o = tid; o < 128; o += nt) {
    const int r0 = (o >> 3) * 2, cq = (o & 7) * 4;
    float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
    const float* t0 = T + (32 + r0) * kTS + 32;
    const float* t1 = t0 + kTS;
#pragma unroll 8
    for (int m = 0; m < 32; ++m) {
      const float4 z = ld4(Z + m * kZS + cq);
      fma4(x0, t0[m], z);
      fma4(x1, t1[m], z);
    }
    st4(T + (32 + r0) * kTS + cq, make_float4(-x0.x, -x0.y, -x0.z, -x0.w));
    st4(T + (33 + r0) * kTS + cq, make_float4(-x1.x, -x1.y, -x1.z, -x1.w));
  }
  __syncthreads();
}

}  // namespace gdn
