// Blocked inverse of a 64 x 64 unit lower-triangular matrix in shared memory:
// T = (I + A)^-1 for strictly lower-triangular A (the solve_tril op,
// include/torch_mlu_ops.h:1052-1054; semantics of triton/fla/solve_tril.py:491-537).
//
// Recursive doubling over 16 / 32 / 64-row blocks:
//   1. the four 16 x 16 diagonal blocks by right-looking forward substitution
//      (one thread per column, the column and its running sums in registers,
//      so the dependent chain is one FMA per row);
//   2. the 32 x 32 diagonal blocks: T_10 = -T_11 (A_10 T_00), likewise T_32;
//   3. the lower-left 32 x 32 block: T_lo,hi = -T_hi (A_hi,lo T_lo).
// Steps 2 and 3 are small products computed as register micro-tiles sized to
// the block (128 or 256 threads), reading T rows as float2 / float4.
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
// (16-byte aligned).  All NT threads of the block call this (NT = blockDim.x,
// 128 or 256); it ends with a __syncthreads.
template <int NT>
__device__ __forceinline__ void solve_tril64_nt(const float* __restrict__ A, float* __restrict__ T,
                                                float* __restrict__ Z) {
  static_assert(NT == 128 || NT == 256, "solve_tril64 runs on 128 or 256 threads");
  const int tid = threadIdx.x;
  // 1. diagonal 16 x 16 blocks: x = column jj of the block's inverse
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15, j = 16 * b + jj;
    const float* Ab = A + (16 * b) * kTrilStride + 16 * b;
    float x[16], acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      x[m] = m == jj ? 1.f : (m > jj ? -acc[m] : 0.f);
#pragma unroll
      for (int i = m + 1; i < 16; ++i) acc[i] = fmaf(Ab[i * kTrilStride + m], x[m], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) T[(16 * b + i) * kTS + j] = x[i];
  }
  for (int e = tid; e < 64 * 16; e += NT) {  // zero the blocks above the diagonal
    const int r = e >> 4, c = (e & 15) * 4;
    if ((r >> 4) < (c >> 4)) st4(T + r * kTS + c, make_float4(0.f, 0.f, 0.f, 0.f));
  }
  __syncthreads();
  // 2. T_10 = -T_11 (A_10 T_00) and T_32 = -T_33 (A_32 T_22)
  if constexpr (NT == 128) {
    const int blk = tid >> 6, r = (tid >> 2) & 15, cq = (tid & 3) * 4;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) fma4(z, A[(rb + r) * kTrilStride + cb + m], ld4(T + (cb + m) * kTS + cb + cq));
    st4(Z + (blk * 16 + r) * kZS + cq, z);
    __syncthreads();
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) fma4(x, T[(rb + r) * kTS + rb + m], ld4(Z + (blk * 16 + m) * kZS + cq));
    st4(T + (rb + r) * kTS + cb + cq, make_float4(-x.x, -x.y, -x.z, -x.w));
  } else {
    const int blk = tid >> 7, r = (tid >> 3) & 15, cq = (tid & 7) * 2;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float2 z = make_float2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float a = A[(rb + r) * kTrilStride + cb + m];
      const float2 t = *reinterpret_cast<const float2*>(T + (cb + m) * kTS + cb + cq);
      z.x = fmaf(a, t.x, z.x);
      z.y = fmaf(a, t.y, z.y);
    }
    *reinterpret_cast<float2*>(Z + (blk * 16 + r) * kZS + cq) = z;
    __syncthreads();
    float2 x = make_float2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float t = T[(rb + r) * kTS + rb + m];
      const float2 zz = *reinterpret_cast<const float2*>(Z + (blk * 16 + m) * kZS + cq);
      x.x = fmaf(t, zz.x, x.x);
      x.y = fmaf(t, zz.y, x.y);
    }
    *reinterpret_cast<float2*>(T + (rb + r) * kTS + cb + cq) = make_float2(-x.x, -x.y);
  }
  __syncthreads();
  // 3. T[32:64, 0:32] = -T_hi (A[32:64, 0:32] T_lo)
  if constexpr (NT == 128) {
    const int r0 = (tid >> 3) * 2, cq = (tid & 7) * 4;
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
    __syncthreads();
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
  } else {
    const int r = tid >> 3, cq = (tid & 7) * 4;
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* a0 = A + (32 + r) * kTrilStride;
#pragma unroll 8
    for (int m = 0; m < 32; ++m) fma4(z, a0[m], ld4(T + m * kTS + cq));
    st4(Z + r * kZS + cq, z);
    __syncthreads();
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* t0 = T + (32 + r) * kTS + 32;
#pragma unroll 8
    for (int m = 0; m < 32; ++m) fma4(x, t0[m], ld4(Z + m * kZS + cq));
    st4(T + (32 + r) * kTS + cq, make_float4(-x.x, -x.y, -x.z, -x.w));
  }
  __syncthreads();
}

// 128-thread form used by the fp32 path and the standalone solve_tril op.
__device__ __forceinline__ void solve_tril64(const float* __restrict__ A, float* __restrict__ T,
                                             float* __restrict__ Z) {
  solve_tril64_nt<128>(A, T, Z);
}

// ---------------------------------------------------------------------------
// Warp-MMA variant for 256-thread blocks (the tensor-core WY kernel).
//
// Same recursive doubling, but the block products of steps 2 and 3 run on
// mma.sync m16n8k8 TF32 with each operand split into a TF32 head and an fp32
// tail (a*b ~ ah*bh + ah*bl + al*bh), which keeps fp32-level accuracy; the
// diagonal 16 x 16 blocks stay on the FMA pipe.  A and T rows are 68 floats
// apart (16-byte aligned, conflict-free A fragments), Z rows 40 apart
// (conflict-free B fragments).
// ---------------------------------------------------------------------------
constexpr int kMS = 68;                 // row stride (floats) of A and T
constexpr int kMZS = 40;                // row stride (floats) of Z
constexpr int kMScratch = 32 * kMZS;    // floats of Z

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  hi = h;
  lo = __float_as_uint(x - __uint_as_float(h));
}

// d += a * b for one m16n8k8 tile; a = A[16 x 8] row-major fragments, b =
// B[8 x 8] column fragments, each given as (head, tail) pairs.
__device__ __forceinline__ void mma_tf32x3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                           const uint32_t (&bh)[2], const uint32_t (&bl)[2]) {
#define GDN_MMA_TF32(A, B)                                                                   \
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, "           \
               "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                      \
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])                             \
               : "r"(A[0]), "r"(A[1]), "r"(A[2]), "r"(A[3]), "r"(B[0]), "r"(B[1]))
  GDN_MMA_TF32(al, bh);
  GDN_MMA_TF32(ah, bl);
  GDN_MMA_TF32(ah, bh);
#undef GDN_MMA_TF32
}

// D(16 x 8) += X[r0.., k0..k0+8*ksteps) * Y[k0.., c0..c0+8), X and Y fp32 in
// shared memory with row strides xs, ys.  The head x head products and the
// two head x tail corrections go to separate accumulators, so the three
// MMAs of a k-step do not wait for one another; the corrections are added
// to the main sum at the end.
__device__ __forceinline__ void mma_rows(float (&d)[4], const float* X, int xs, const float* Y, int ys,
                                         int ksteps) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
#define GDN_MMA_TF32_ACC(D, A, B)                                                            \
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, "           \
               "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                      \
               : "+f"(D[0]), "+f"(D[1]), "+f"(D[2]), "+f"(D[3])                             \
               : "r"(A[0]), "r"(A[1]), "r"(A[2]), "r"(A[3]), "r"(B[0]), "r"(B[1]))
#pragma unroll
  for (int kk = 0; kk < ksteps; ++kk) {
    uint32_t ah[4], al[4], bh[2], bl[2];
    const float* x = X + kk * 8;
    tf32_split(x[g * xs + t], ah[0], al[0]);
    tf32_split(x[(g + 8) * xs + t], ah[1], al[1]);
    tf32_split(x[g * xs + t + 4], ah[2], al[2]);
    tf32_split(x[(g + 8) * xs + t + 4], ah[3], al[3]);
    const float* y = Y + kk * 8 * ys;
    tf32_split(y[t * ys + g], bh[0], bl[0]);
    tf32_split(y[(t + 4) * ys + g], bh[1], bl[1]);
    GDN_MMA_TF32_ACC(c1, al, bh);
    GDN_MMA_TF32_ACC(c2, ah, bl);
    GDN_MMA_TF32_ACC(d, ah, bh);
  }
#undef GDN_MMA_TF32_ACC
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] += c1[i] + c2[i];
}

// A: [64][kMS] (strictly lower part read), T: [64][kMS], Z: kMScratch floats;
// 16-byte aligned.  256 threads (thread ids 0..255 of the block) call this;
// they synchronise on named barrier BAR (0 with 256 threads is
// __syncthreads in a 256-thread block), and it ends with that barrier.
template <int BAR = 0>
__device__ __forceinline__ void solve_tril64_mma(const float* __restrict__ A, float* __restrict__ T,
                                                 float* __restrict__ Z) {
  auto sync = [] { asm volatile("bar.sync %0, 256;" :: "n"(BAR) : "memory"); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // 1. diagonal 16 x 16 blocks, right-looking substitution (one column per thread)
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15, j = 16 * b + jj;
    const float* Ab = A + (16 * b) * kMS + 16 * b;
    float x[16], acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      x[m] = m == jj ? 1.f : (m > jj ? -acc[m] : 0.f);
#pragma unroll
      for (int i = m + 1; i < 16; ++i) acc[i] = fmaf(Ab[i * kMS + m], x[m], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) T[(16 * b + i) * kMS + j] = x[i];
  }
  for (int e = tid; e < 64 * 16; e += 256) {  // zero the blocks above the diagonal
    const int r = e >> 4, c = (e & 15) * 4;
    if ((r >> 4) < (c >> 4)) st4(T + r * kMS + c, make_float4(0.f, 0.f, 0.f, 0.f));
  }
  sync();
  // 2. T_10 = -T_11 (A_10 T_00), T_32 = -T_33 (A_32 T_22): warp w < 4 owns
  //    block w >> 1 and the 8-column half w & 1 of its 16 x 16 result
  if (warp < 4) {
    const int blk = warp >> 1, nh = (warp & 1) * 8;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, A + rb * kMS + cb, kMS, T + cb * kMS + cb + nh, kMS, 2);
    float* z = Z + blk * 16 * kMZS + nh;
    *reinterpret_cast<float2*>(z + g * kMZS + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kMZS + 2 * t) = make_float2(d[2], d[3]);
  }
  sync();
  if (warp < 4) {
    const int blk = warp >> 1, nh = (warp & 1) * 8;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, T + rb * kMS + rb, kMS, Z + blk * 16 * kMZS + nh, kMZS, 2);
    float* o = T + rb * kMS + cb + nh;
    *reinterpret_cast<float2*>(o + g * kMS + 2 * t) = make_float2(-d[0], -d[1]);
    *reinterpret_cast<float2*>(o + (g + 8) * kMS + 2 * t) = make_float2(-d[2], -d[3]);
  }
  sync();
  // 3. T[32:64, 0:32] = -T_hi (A[32:64, 0:32] T_lo): warp w owns rows
  //    32 + 16 (w >> 2) .. +16 and columns 8 (w & 3) .. +8
  {
    const int mr = 16 * (warp >> 2), nc = 8 * (warp & 3);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, A + (32 + mr) * kMS, kMS, T + nc, kMS, 4);
    float* z = Z + mr * kMZS + nc;
    *reinterpret_cast<float2*>(z + g * kMZS + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kMZS + 2 * t) = make_float2(d[2], d[3]);
    sync();
    float e[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(e, T + (32 + mr) * kMS + 32, kMS, Z + nc, kMZS, 4);
    float* o = T + (32 + mr) * kMS + nc;
    *reinterpret_cast<float2*>(o + g * kMS + 2 * t) = make_float2(-e[0], -e[1]);
    *reinterpret_cast<float2*>(o + (g + 8) * kMS + 2 * t) = make_float2(-e[2], -e[3]);
  }
  sync();
}

// In-place form of solve_tril64_mma for the tensor-core WY kernel: AT holds
// the strictly lower A ([64][kMS], 16-byte aligned; the diagonal and the
// upper triangle are not read) and receives T = (I + A)^-1 over it.  The
// upper-right 32 x 32 block (rows 0..31, columns 32..63), where T is zero,
// serves as the scratch of the block products and holds garbage on return:
// callers read it as zeros.  The other blocks above the diagonal are zeroed.
// 256 threads; named barrier BAR; ends with that barrier.
template <int BAR = 0>
__device__ __forceinline__ void solve_tril64_mma_ip(float* __restrict__ AT) {
  auto sync = [] { asm volatile("bar.sync %0, 256;" :: "n"(BAR) : "memory"); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  float* Z = AT + 32;  // the upper-right block, row stride kMS
  // 1. diagonal 16 x 16 blocks, right-looking substitution (one column per
  //    thread) into registers; written over A once every thread has read it
  float x[16];
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15;
    const float* Ab = AT + (16 * b) * kMS + 16 * b;
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      x[m] = m == jj ? 1.f : (m > jj ? -acc[m] : 0.f);
#pragma unroll
      for (int i = m + 1; i < 16; ++i) acc[i] = fmaf(Ab[i * kMS + m], x[m], acc[i]);
    }
  } else if (tid < 64 + 128) {  // zero the 16 x 16 blocks (0, 1) and (2, 3)
    const int e = tid - 64, blk = e >> 6, r = (e >> 2) & 15, c4 = (e & 3) * 4;
    st4(AT + (32 * blk + r) * kMS + 32 * blk + 16 + c4, make_float4(0.f, 0.f, 0.f, 0.f));
  }
  sync();
  if (tid < 64) {
    const int b = tid >> 4, jj = tid & 15;
#pragma unroll
    for (int i = 0; i < 16; ++i) AT[(16 * b + i) * kMS + 16 * b + jj] = x[i];
  }
  sync();
  // 2. T_10 = -T_11 (A_10 T_00), T_32 = -T_33 (A_32 T_22): warp w < 4 owns
  //    block w >> 1 and the 8-column half w & 1 of its 16 x 16 result
  if (warp < 4) {
    const int blk = warp >> 1, nh = (warp & 1) * 8;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, AT + rb * kMS + cb, kMS, AT + cb * kMS + cb + nh, kMS, 2);
    float* z = Z + blk * 16 * kMS + nh;
    *reinterpret_cast<float2*>(z + g * kMS + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kMS + 2 * t) = make_float2(d[2], d[3]);
  }
  sync();
  if (warp < 4) {
    const int blk = warp >> 1, nh = (warp & 1) * 8;
    const int rb = 16 * (2 * blk + 1), cb = 16 * (2 * blk);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, AT + rb * kMS + rb, kMS, Z + blk * 16 * kMS + nh, kMS, 2);
    float* o = AT + rb * kMS + cb + nh;
    *reinterpret_cast<float2*>(o + g * kMS + 2 * t) = make_float2(-d[0], -d[1]);
    *reinterpret_cast<float2*>(o + (g + 8) * kMS + 2 * t) = make_float2(-d[2], -d[3]);
  }
  sync();
  // 3. T[32:64, 0:32] = -T_hi (A[32:64, 0:32] T_lo): warp w owns rows
  //    32 + 16 (w >> 2) .. +16 and columns 8 (w & 3) .. +8
  {
    const int mr = 16 * (warp >> 2), nc = 8 * (warp & 3);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(d, AT + (32 + mr) * kMS, kMS, AT + nc, kMS, 4);
    float* z = Z + mr * kMS + nc;
    *reinterpret_cast<float2*>(z + g * kMS + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(z + (g + 8) * kMS + 2 * t) = make_float2(d[2], d[3]);
    sync();
    float e[4] = {0.f, 0.f, 0.f, 0.f};
    mma_rows(e, AT + (32 + mr) * kMS + 32, kMS, Z + nc, kMS, 4);
    float* o = AT + (32 + mr) * kMS + nc;
    *reinterpret_cast<float2*>(o + g * kMS + 2 * t) = make_float2(-e[0], -e[1]);
    *reinterpret_cast<float2*>(o + (g + 8) * kMS + 2 * t) = make_float2(-e[2], -e[3]);
  }
  sync();
}

}  // namespace gdn
