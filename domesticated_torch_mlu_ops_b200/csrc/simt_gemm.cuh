// Register-tiled fp32 SIMT products for the full-precision chunk kernels
// (generic forward and backward): one CTA of kGemmThreads threads computes a
// 64-row block C[i][n], i < 64, n < 16 * NJ, each thread owning rows
// tr*4 .. tr*4+3 (tr = tid / 16) and columns tc + 16 j (tc = tid % 16).
//
//   gemm_smem: both operands in shared memory, read in place.  A(i, k) =
//     a[i*asi + k*ask], B(k, n) = b[k*bsk + n*bsn]; the caller zero-pads rows
//     and columns past the valid extent.  With the padded layouts used here
//     (row strides 65 / 129, or transposed reads of them) each warp reads
//     two A addresses (broadcast) and 16 distinct banks of B.
//   gemm_staged: operands anywhere (global or shared, fp32 or 16-bit),
//     staged 16 deep through `st` (kGemmStage floats) with bounds: A rows
//     i >= ma, B columns n >= nb and k >= Kd read as zero.  The next 16-deep
//     block is fetched into registers while the current one is multiplied.
// Both store C (shared or global, row stride ldc) for rows i < mc and
// columns n < N, as C = alpha * AB or C += alpha * AB (ACC), and both begin
// and end with a barrier; C may alias an operand of gemm_smem.
#pragma once

#include "gdn_common.cuh"

namespace gdn {

constexpr int kGemmThreads = 256;
constexpr int kGemmStage = 64 * 17 + 16 * 129;  // floats of staging for gemm_staged

template <int NJ, bool ACC>
__device__ __forceinline__ void gemm_store(float (&acc)[4][NJ], float* C, int64_t ldc, int mc, int N,
                                           float alpha) {
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tr * 4 + r;
    if (i >= mc) continue;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int n = tc + 16 * j;
      if (n < N) {
        float* c = C + i * ldc + n;
        *c = ACC ? fmaf(alpha, acc[r][j], *c) : alpha * acc[r][j];
      }
    }
  }
}

template <int NJ, bool ACC>
__device__ __forceinline__ void gemm_smem_nj(float* C, int64_t ldc, int mc, int N, int Kd, const float* a,
                                             int asi, int ask, const float* b, int bsk, int bsn,
                                             float alpha) {
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  float acc[4][NJ];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[r][j] = 0.f;
  const float* ap = a + (tr * 4) * asi;
  const float* bp = b + tc * bsn;
  __syncthreads();
#pragma unroll 4
  for (int k = 0; k < Kd; ++k) {
    float av[4], bv[NJ];
#pragma unroll
    for (int r = 0; r < 4; ++r) av[r] = ap[r * asi + k * ask];
#pragma unroll
    for (int j = 0; j < NJ; ++j) bv[j] = bp[k * bsk + 16 * j * bsn];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < NJ; ++j) acc[r][j] = fmaf(av[r], bv[j], acc[r][j]);
  }
  __syncthreads();
  gemm_store<NJ, ACC>(acc, C, ldc, mc, N, alpha);
  __syncthreads();
}

// N <= 128; operands in shared memory (C may be global).
template <bool ACC>
__device__ __forceinline__ void gemm_smem(float* C, int64_t ldc, int mc, int N, int Kd, const float* a, int asi,
                                          int ask, const float* b, int bsk, int bsn, float alpha = 1.f) {
  if (N <= 32) gemm_smem_nj<2, ACC>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
  else if (N <= 64) gemm_smem_nj<4, ACC>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
  else gemm_smem_nj<8, ACC>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
}

template <int NJ, bool ACC, typename TA, typename TB>
__device__ __forceinline__ void gemm_staged_nj(float* C, int64_t ldc, int mc, int N, int Kd, const TA* a,
                                               int64_t asi, int64_t ask, int ma, const TB* b, int64_t bsk,
                                               int64_t bsn, int nb, float alpha, float* st) {
  constexpr int NC = 16 * NJ;
  constexpr int AE = 64 * 16 / kGemmThreads;  // A elements per thread per k-block
  constexpr int BE = 16 * NC / kGemmThreads;  // B elements per thread per k-block
  float* As = st;            // [64][17]
  float* Bs = st + 64 * 17;  // [16][129]
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  // index order follows the operand's unit stride so that global reads coalesce
  const bool a_k_fast = ask == 1, b_k_fast = bsk == 1 && bsn != 1;
  float ra[AE], rb[BE];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int u = 0; u < AE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int i = a_k_fast ? e >> 4 : e & 63, k = k0 + (a_k_fast ? e & 15 : e >> 6);
      ra[u] = (i < ma && k < Kd) ? to_f<TA>(a[i * asi + k * ask]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < BE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int n = b_k_fast ? e >> 4 : e % NC, k = k0 + (b_k_fast ? e & 15 : e / NC);
      rb[u] = (k < Kd && n < nb) ? to_f<TB>(b[k * bsk + n * bsn]) : 0.f;
    }
  };
  float acc[4][NJ];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[r][j] = 0.f;
  __syncthreads();  // shared-memory operands written just before the call are complete
  if (Kd > 0) fetch(0);
  for (int k0 = 0; k0 < Kd; k0 += 16) {
#pragma unroll
    for (int u = 0; u < AE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int i = a_k_fast ? e >> 4 : e & 63, kk = a_k_fast ? e & 15 : e >> 6;
      As[i * 17 + kk] = ra[u];
    }
#pragma unroll
    for (int u = 0; u < BE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int n = b_k_fast ? e >> 4 : e % NC, kk = b_k_fast ? e & 15 : e / NC;
      Bs[kk * 129 + n] = rb[u];
    }
    __syncthreads();
    if (k0 + 16 < Kd) fetch(k0 + 16);  // global latency overlaps the products below
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[NJ];
#pragma unroll
      for (int r = 0; r < 4; ++r) av[r] = As[(tr * 4 + r) * 17 + kk];
#pragma unroll
      for (int j = 0; j < NJ; ++j) bv[j] = Bs[kk * 129 + tc + 16 * j];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[r][j] = fmaf(av[r], bv[j], acc[r][j]);
    }
    __syncthreads();
  }
  gemm_store<NJ, ACC>(acc, C, ldc, mc, N, alpha);
  __syncthreads();
}

template <bool ACC, typename TA, typename TB>
__device__ __forceinline__ void gemm_staged(float* C, int64_t ldc, int mc, int N, int Kd, const TA* a,
                                            int64_t asi, int64_t ask, int ma, const TB* b, int64_t bsk,
                                            int64_t bsn, int nb, float alpha, float* st) {
  if (N <= 32) gemm_staged_nj<2, ACC>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
  else if (N <= 64) gemm_staged_nj<4, ACC>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
  else gemm_staged_nj<8, ACC>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
}

// Block-wide sum of one value per thread, returned to every thread (`red`
// holds kGemmThreads / 32 floats).
__device__ __forceinline__ float block_sum(float x, float* red) {
  x = group_sum<32>(x);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kGemmThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

// 4-byte asynchronous global -> shared copy (zero-filled when !ok; the
// source is not read then).
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool ok) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(ok ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace gdn
