// 64-row fp32 products for the full-precision chunk kernels (generic
// forward and backward) on warp-level tensor-core MMA (m16n8k8, TF32): every
// operand is split into a TF32 head and the TF32-rounded remainder, and the
// three products head*head + head*tail + tail*head are accumulated in fp32,
// which keeps fp32 accuracy (relative error about 2^-21 per product).  One
// CTA of kGemmThreads (8 warps) computes C[i][n], i < 64, n < N <= 128: warp
// w owns rows 16*(w % 4) .. +15 and the 8-column tiles w / 4, w / 4 + 2, ...,
// so each A fragment is split once and used for all of the warp's tiles.
//
//   gemm_smem: both operands in shared memory, read in place.  A(i, k) =
//     a[i*asi + k*ask], B(k, n) = b[k*bsk + n*bsn]; k >= Kd reads as zero.
//     Rows i < 64 of A and columns n < 16 * ceil(N / 16) of B must be
//     readable (their values past the valid extent only reach outputs that
//     are not stored).
//   gemm_staged: operands anywhere (global or shared, fp32 or 16-bit),
//     staged 16 deep through `st` (kGemmStage floats) with bounds: A rows
//     i >= ma, B columns n >= nb and k >= Kd read as zero.  The next 16-deep
//     block is fetched into registers while the current one is multiplied.
// Row strides for conflict-free fragment reads (32 banks): a row-major A
// (k contiguous) or a k-contiguous B wants a stride of 4 (mod 32) words
// (kRowK below); a transposed A or an n-contiguous B wants 8 (mod 32)
// (kRowN, kRow32 for 32-column tiles).
// Both store C (shared or global, row stride ldc) for rows i < mc and
// columns n < N, as C = alpha * AB or C += alpha * AB (ACC), and both begin
// and end with a barrier; C may alias an operand of gemm_smem.
// SPLIT = false (kernels of 16-bit inputs): one TF32 product per step, no
// tails.  16-bit values are exact in TF32, and fp32 intermediates are rounded
// to 10 mantissa bits, finer than the reference's bf16 roundings of the same
// operands; the fp32 path keeps the split.
#pragma once

#include <type_traits>

#include "gdn_common.cuh"
#include "solve_tril.cuh"

namespace gdn {

constexpr int kGemmThreads = 256;
constexpr int kRowK = 132;  // 64 x 128 tiles read k-contiguous (row-major A, B = X^T)
constexpr int kRowN = 136;  // 64 x 128 tiles read transposed (A = X^T) or n-contiguous (B = X)
constexpr int kRow32 = 40;  // 128 x 32 tiles read n-contiguous (B = X)
constexpr int kStA = 20;   // row stride of the staged A block (64 x 16): conflict-free fragment reads
constexpr int kStB = 136;  // row stride of the staged B block (16 x 128)
constexpr int kGemmStage = 64 * kStA + 16 * kStB;  // floats of staging for gemm_staged

// Fragment store of a warp's column tiles: d[j] + e[j] is the 16 x 8 tile at
// rows 16*rt .. +15, columns 8*(ch + 2j) .. +7.
template <int CW, bool ACC>
__device__ __forceinline__ void mma_store(const float (&d)[CW][4], const float (&e)[CW][4], float* C,
                                          int64_t ldc, int mc, int N, float alpha) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r0 = (warp & 3) * 16 + g, ch = warp >> 2;
#pragma unroll
  for (int j = 0; j < CW; ++j) {
    const int n0 = (ch + 2 * j) * 8 + 2 * t;
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int i = r0 + (x >> 1) * 8, n = n0 + (x & 1);
      if (i < mc && n < N) {
        float* c = C + i * ldc + n;
        const float v = d[j][x] + e[j][x];
        *c = ACC ? fmaf(alpha, v, *c) : alpha * v;
      }
    }
  }
}

#define GDN_MMA_TF32_ACC(D, A, B0, B1)                                                      \
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, "          \
               "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                     \
               : "+f"(D[0]), "+f"(D[1]), "+f"(D[2]), "+f"(D[3])                            \
               : "r"(A[0]), "r"(A[1]), "r"(A[2]), "r"(A[3]), "r"(B0), "r"(B1))

// One 8-deep step of a warp: A fragment at columns k0.., B fragments of the
// warp's column tiles; reads at k >= kmax give zero.  Head products go to d,
// the two tail products to e, issued tile by tile so that consecutive MMAs
// are independent.
__device__ __forceinline__ uint32_t tf32_round(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return h;
}

template <int CW, bool SPLIT = true, typename LA, typename LB>
__device__ __forceinline__ void mma_kstep(float (&d)[CW][4], float (&e)[CW][4], int k0, int kmax, LA lda,
                                          LB ldb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ch = threadIdx.x >> 7;
  const int ka = k0 + t, kb = k0 + t + 4;
  const bool va = ka < kmax, vb = kb < kmax;
  if constexpr (!SPLIT) {
    uint32_t a[4], bb[CW][2];
    a[0] = tf32_round(va ? lda(g, ka) : 0.f);
    a[1] = tf32_round(va ? lda(g + 8, ka) : 0.f);
    a[2] = tf32_round(vb ? lda(g, kb) : 0.f);
    a[3] = tf32_round(vb ? lda(g + 8, kb) : 0.f);
#pragma unroll
    for (int j = 0; j < CW; ++j) {
      const int n = (ch + 2 * j) * 8 + g;
      bb[j][0] = tf32_round(va ? ldb(ka, n) : 0.f);
      bb[j][1] = tf32_round(vb ? ldb(kb, n) : 0.f);
    }
#pragma unroll
    for (int j = 0; j < CW; ++j) GDN_MMA_TF32_ACC(d[j], a, bb[j][0], bb[j][1]);
    return;
  }
  uint32_t ah[4], al[4], bh[CW][2], bl[CW][2];
  tf32_split(va ? lda(g, ka) : 0.f, ah[0], al[0]);
  tf32_split(va ? lda(g + 8, ka) : 0.f, ah[1], al[1]);
  tf32_split(vb ? lda(g, kb) : 0.f, ah[2], al[2]);
  tf32_split(vb ? lda(g + 8, kb) : 0.f, ah[3], al[3]);
#pragma unroll
  for (int j = 0; j < CW; ++j) {
    const int n = (ch + 2 * j) * 8 + g;
    tf32_split(va ? ldb(ka, n) : 0.f, bh[j][0], bl[j][0]);
    tf32_split(vb ? ldb(kb, n) : 0.f, bh[j][1], bl[j][1]);
  }
#pragma unroll
  for (int j = 0; j < CW; ++j) GDN_MMA_TF32_ACC(e[j], al, bh[j][0], bh[j][1]);
#pragma unroll
  for (int j = 0; j < CW; ++j) GDN_MMA_TF32_ACC(d[j], ah, bh[j][0], bh[j][1]);
#pragma unroll
  for (int j = 0; j < CW; ++j) GDN_MMA_TF32_ACC(e[j], ah, bl[j][0], bl[j][1]);
}
#undef GDN_MMA_TF32_ACC

template <int CW, bool ACC, bool SPLIT>
__device__ __forceinline__ void gemm_smem_cw(float* C, int64_t ldc, int mc, int N, int Kd, const float* a,
                                             int asi, int ask, const float* b, int bsk, int bsn, float alpha) {
  float d[CW][4], e[CW][4];
#pragma unroll
  for (int j = 0; j < CW; ++j)
#pragma unroll
    for (int x = 0; x < 4; ++x) d[j][x] = e[j][x] = 0.f;
  const float* ap = a + ((threadIdx.x >> 5) & 3) * 16 * asi;
  auto lda = [&](int r, int k) { return ap[r * asi + k * ask]; };
  auto ldb = [&](int k, int n) { return b[k * bsk + n * bsn]; };
  __syncthreads();
#pragma unroll 2
  for (int k0 = 0; k0 < Kd; k0 += 8) mma_kstep<CW, SPLIT>(d, e, k0, Kd, lda, ldb);
  __syncthreads();
  mma_store<CW, ACC>(d, e, C, ldc, mc, N, alpha);
  __syncthreads();
}

// N <= 128; operands in shared memory (C may be global).
template <bool ACC, bool SPLIT = true>
__device__ __forceinline__ void gemm_smem(float* C, int64_t ldc, int mc, int N, int Kd, const float* a, int asi,
                                          int ask, const float* b, int bsk, int bsn, float alpha = 1.f) {
  if (N <= 16) gemm_smem_cw<1, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
  else if (N <= 32) gemm_smem_cw<2, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
  else if (N <= 64) gemm_smem_cw<4, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
  else gemm_smem_cw<8, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, b, bsk, bsn, alpha);
}

template <int CW, bool ACC, bool SPLIT, typename TA, typename TB>
__device__ __forceinline__ void gemm_staged_cw(float* C, int64_t ldc, int mc, int N, int Kd, const TA* a,
                                               int64_t asi, int64_t ask, int ma, const TB* b, int64_t bsk,
                                               int64_t bsn, int nb, float alpha, float* st) {
  constexpr int NC = 16 * CW;                  // staged B columns
  constexpr int AE = 64 * 16 / kGemmThreads;   // A elements per thread per k-block
  constexpr int BE = (16 * NC + kGemmThreads - 1) / kGemmThreads;  // B elements per thread per k-block
  float* As = st;              // [64][kStA]
  float* Bs = st + 64 * kStA;  // [16][kStB]
  const int tid = threadIdx.x;
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
      rb[u] = (e < 16 * NC && k < Kd && n < nb) ? to_f<TB>(b[k * bsk + n * bsn]) : 0.f;
    }
  };
  float d[CW][4], e[CW][4];
#pragma unroll
  for (int j = 0; j < CW; ++j)
#pragma unroll
    for (int x = 0; x < 4; ++x) d[j][x] = e[j][x] = 0.f;
  const float* ap = As + ((tid >> 5) & 3) * 16 * kStA;
  auto lda = [&](int r, int k) { return ap[r * kStA + k]; };
  auto ldb = [&](int k, int n) { return Bs[k * kStB + n]; };
  __syncthreads();  // shared-memory operands written just before the call are complete
  if (Kd > 0) fetch(0);
  for (int k0 = 0; k0 < Kd; k0 += 16) {
#pragma unroll
    for (int u = 0; u < AE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int i = a_k_fast ? e >> 4 : e & 63, kk = a_k_fast ? e & 15 : e >> 6;
      As[i * kStA + kk] = ra[u];
    }
#pragma unroll
    for (int u = 0; u < BE; ++u) {
      const int e = tid + u * kGemmThreads;
      const int n = b_k_fast ? e >> 4 : e % NC, kk = b_k_fast ? e & 15 : e / NC;
      if (e < 16 * NC) Bs[kk * kStB + n] = rb[u];
    }
    __syncthreads();
    if (k0 + 16 < Kd) fetch(k0 + 16);  // global latency overlaps the products below
    mma_kstep<CW, SPLIT>(d, e, 0, 16, lda, ldb);
    mma_kstep<CW, SPLIT>(d, e, 8, 16, lda, ldb);
    __syncthreads();
  }
  mma_store<CW, ACC>(d, e, C, ldc, mc, N, alpha);
  __syncthreads();
}

template <bool ACC, bool SPLIT = true, typename TA, typename TB>
__device__ __forceinline__ void gemm_staged(float* C, int64_t ldc, int mc, int N, int Kd, const TA* a,
                                            int64_t asi, int64_t ask, int ma, const TB* b, int64_t bsk,
                                            int64_t bsn, int nb, float alpha, float* st) {
  if (N <= 16) gemm_staged_cw<1, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
  else if (N <= 32) gemm_staged_cw<2, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
  else if (N <= 64) gemm_staged_cw<4, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
  else gemm_staged_cw<8, ACC, SPLIT>(C, ldc, mc, N, Kd, a, asi, ask, ma, b, bsk, bsn, nb, alpha, st);
}

// Whether the products of a kernel on T inputs split their operands (fp32)
// or take one TF32 product (16-bit inputs).
template <typename T>
constexpr bool kSplit = std::is_same<T, float>::value;

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

namespace gdn {

__device__ __forceinline__ void cp_async16z(float* dst, const float* src, bool ok) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

// Asynchronous copy of a row tile: rows i < rows, columns c < cpad of dst
// (row stride dstride floats, 16-byte aligned rows) from src + i * sstride
// (global); rows i >= L and columns c >= cols are zero-filled.  A warp per
// row, 16-byte copies when the source rows allow them.  All kGemmThreads
// threads call it; the caller commits and waits.
__device__ __forceinline__ void tile_async(float* dst, int dstride, const float* src, int64_t sstride, int L,
                                           int rows, int cols, int cpad) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool vec = (cols & 3) == 0 && (cpad & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(sstride * 4)) & 15) == 0;
  if (vec) {
    for (int i = warp; i < rows; i += kGemmThreads / 32)
      for (int c = lane * 4; c < cpad; c += 128) {
        const bool ok = i < L && c < cols;
        cp_async16z(dst + i * dstride + c, ok ? src + i * sstride + c : src, ok);
      }
  } else {
    for (int i = warp; i < rows; i += kGemmThreads / 32)
      for (int c = lane; c < cpad; c += 32) {
        const bool ok = i < L && c < cols;
        cp_async4(dst + i * dstride + c, ok ? src + i * sstride + c : src, ok);
      }
  }
}

}  // namespace gdn
