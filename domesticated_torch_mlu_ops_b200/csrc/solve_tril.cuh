// Blocked inverse of a 64 x 64 unit lower-triangular matrix in shared memory:
// Ti = (I + A)^-1 for strictly lower-triangular A (the solve_tril op,
// include/torch_mlu_ops.h:1052-1054; semantics of triton/fla/solve_tril.py:491-537).
//
// The matrix is split into 4 x 4 blocks of 16.  The four diagonal blocks are
// inverted in parallel by forward substitution (one thread per column, the
// column in registers), then the off-diagonal blocks follow level by level:
//   T_ij = -T_ii * sum_{k=j}^{i-1} A_ik T_kj      (i > j, block indices)
// which is 3 levels of small block products spread over the whole CTA,
// instead of one 64-step dependent chain per column.
#pragma once

namespace gdn {

constexpr int kTrilStride = 65;  // row stride (floats) of A and Ti
constexpr int kTrilZStride = 17;

// A, Ti: [64][65] floats; Z: scratch of 64 * 17 floats.  All threads of the
// block call this (blockDim.x >= 64); it ends with a __syncthreads.
__device__ __forceinline__ void solve_tril64(const float* __restrict__ A, float* __restrict__ Ti,
                                             float* __restrict__ Z) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15, j = 16 * b + jj;
    const float* Ab = A + (16 * b) * kTrilStride + 16 * b;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == jj) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc += Ab[i * kTrilStride + m] * x[m];
      if (i > jj) x[i] = -acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) Ti[(16 * b + i) * kTrilStride + j] = x[i];
  }
  for (int e = tid; e < 64 * 64; e += nt) {  // blocks above the diagonal
    const int r = e >> 6, c = e & 63;
    if ((r >> 4) < (c >> 4)) Ti[r * kTrilStride + c] = 0.f;
  }
  __syncthreads();
#pragma unroll 1
  for (int d = 1; d < 4; ++d) {
    const int outputs = (4 - d) * 256;
    for (int e = tid; e < outputs; e += nt) {  // Z = sum_k A_ik T_kj
      const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, cc = e & 15;
      const float* arow = A + (16 * ib + r) * kTrilStride;
      float acc = 0.f;
      for (int kb = jb; kb < ib; ++kb) {
#pragma unroll
        for (int m = 0; m < 16; ++m)
          acc += arow[16 * kb + m] * Ti[(16 * kb + m) * kTrilStride + 16 * jb + cc];
      }
      Z[(jb * 16 + r) * kTrilZStride + cc] = acc;
    }
    __syncthreads();
    for (int e = tid; e < outputs; e += nt) {  // T_ij = -T_ii Z
      const int jb = e >> 8, ib = jb + d, r = (e >> 4) & 15, cc = e & 15;
      const float* trow = Ti + (16 * ib + r) * kTrilStride + 16 * ib;
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m)
        if (m <= r) acc += trow[m] * Z[(jb * 16 + m) * kTrilZStride + cc];
      Ti[(16 * ib + r) * kTrilStride + 16 * jb + cc] = -acc;
    }
    __syncthreads();
  }
}

}  // namespace gdn
