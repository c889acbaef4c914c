// Test-only kernel: one tcgen05 MMA D[M][N] = sum_k A(m,k) B(n,k) with the
// operand layouts, descriptors and TMEM read-back conventions of the product
// kernels (domesticated_torch_mlu_ops_b200/csrc/umma.cuh).  A is given as
// [M][K] (K-major) or [K][M] (a_mn), B as [N][K] or [K][N] (b_mn), bf16.
// Each operand is stored either as a no-swizzle image or as 128-byte
// swizzled atoms (the layout TMA writes with SWIZZLE_128B).
#include <cuda_bf16.h>
#include <stdint.h>

#include "umma.cuh"

using namespace gdn::umma;

// Swizzled tiles: 64-column atoms of rows x 128 bytes placed ST bytes apart
// (ST = 0 means back to back).
template <int ROWS, int COLS, bool SW, int ST>
__device__ uint32_t tile_off(int r, int c) {
  constexpr int stride = ST ? ST : ROWS * 128;
  return SW ? static_cast<uint32_t>((c >> 6) * stride) + sw128_off(r, c & 63, ROWS)
            : img_off(r, c, (COLS / 8) * 128);
}

template <int ROWS, int COLS, bool MN, bool SW, int ST>
__device__ uint64_t op_desc(uint32_t base, int ks) {
  constexpr int stride = ST ? ST : ROWS * 128;
  if (SW) {
    if (MN) return smem_desc_sw128(base + ks * 16 * 128, stride, 1024);
    return smem_desc_sw128(base + ((ks * 16) >> 6) * stride + ((ks * 16) & 63) * 2, 16, 1024);
  }
  constexpr int RS = (COLS / 8) * 128;
  if (MN) return smem_desc(base + ks * 2 * RS, RS, 128);
  return smem_desc(base + ks * 256, 128, RS);
}

template <int M, int N, int K, bool AMN, bool BMN, bool ASW, bool BSW, int AST, int BST>
__global__ void __launch_bounds__(128) selftest(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                                float* Dout, int* status) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int ACOLS = AMN ? M : K, AROWS = AMN ? K : M;
  constexpr int BCOLS = BMN ? N : K, BROWS = BMN ? K : N;
  constexpr int ABYTES = (ASW && AST) ? (ACOLS / 64) * AST : AROWS * ACOLS * 2;
  constexpr int BBYTES = (BSW && BST) ? (BCOLS / 64) * BST : BROWS * BCOLS * 2;
  uint8_t* aimg = sm;
  uint8_t* bimg = sm + ((ABYTES + 1023) / 1024) * 1024;
  uint64_t* bar = reinterpret_cast<uint64_t*>(bimg + ((BBYTES + 1023) / 1024) * 1024);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < AROWS * ACOLS; e += 128)
    *reinterpret_cast<__nv_bfloat16*>(aimg + tile_off<AROWS, ACOLS, ASW, AST>(e / ACOLS, e % ACOLS)) = A[e];
  for (int e = tid; e < BROWS * BCOLS; e += 128)
    *reinterpret_cast<__nv_bfloat16*>(bimg + tile_off<BROWS, BCOLS, BSW, BST>(e / BCOLS, e % BCOLS)) = B[e];
  if (warp == 0) { tmem_alloc(tslot, 256); fence_before_sync(); }
  if (tid == 0) { mbar_init(bar, 1); mbar_fence_init(); }
  fence_proxy_async();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    const uint32_t id = idesc_f16(M, N, true, AMN, BMN);
    const uint32_t aa = smem_u32(aimg), ba = smem_u32(bimg);
    for (int ks = 0; ks < K / 16; ++ks)
      mma_f16(tmem, op_desc<AROWS, ACOLS, AMN, ASW, AST>(aa, ks),
              op_desc<BROWS, BCOLS, BMN, BSW, BST>(ba, ks), id, ks > 0);
    mma_commit(smem_u32(bar));
  }
  const bool ok = mbar_wait(smem_u32(bar), 0, 200000000LL);
  if (!ok && tid == 0) atomicExch(status, 1);
  if (!__syncthreads_or(!ok)) {
    fence_after_sync();
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int row = M == 128 ? tid : (lane < 16 ? warp * 16 + lane : -1);
    for (int q = 0; q < N / 32; ++q) {
      float x[32];
      tmem_ld32(tmem + lane_base + q * 32, x);
      if (row >= 0)
        for (int e = 0; e < 32; ++e) Dout[row * N + q * 32 + e] = x[e];
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <int M, int N, int K, bool AMN, bool BMN, bool ASW = false, bool BSW = false,
          int AST = 0, int BST = 0>
static int run(const void* A, const void* B, float* D, int* st) {
  auto k = selftest<M, N, K, AMN, BMN, ASW, BSW, AST, BST>;
  const int smem = 2 * (M * K + N * K) * 2 + 4096;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k<<<1, 128, smem>>>(static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, st);
  return static_cast<int>(cudaDeviceSynchronize());
}

extern "C" int umma_selftest(int which, const void* A, const void* B, float* D, int* st) {
  switch (which) {
    case 0: return run<64, 64, 128, false, false>(A, B, D, st);   // S = K K^T (no swizzle)
    case 1: return run<64, 128, 64, false, true>(A, B, D, st);    // W = T' K
    case 2: return run<128, 32, 64, true, true>(A, B, D, st);     // dH = K^T V~
    case 3: return run<64, 32, 128, false, true>(A, B, D, st);    // X = W h
    case 4: return run<128, 128, 64, true, true>(A, B, D, st);    // dH, VS = 128
    case 5: return run<64, 64, 64, false, true>(A, B, D, st);     // O = P v_new, VS = 64
    case 6: return run<64, 64, 128, false, false, true, true>(A, B, D, st);   // S = K K^T, TMA tiles
    case 7: return run<64, 128, 64, false, true, false, true>(A, B, D, st);   // W = T' K, K swizzled
    case 8: return run<128, 32, 64, true, true, true, false>(A, B, D, st);    // dH = K^T V~, K swizzled
    case 9: return run<64, 32, 128, false, true, true, false>(A, B, D, st);   // Y = Q h, Q swizzled
    case 10: return run<128, 128, 64, true, true, true, false>(A, B, D, st);  // dH, VS = 128
    // stacked operands of the restructured kernels
    case 11: return run<128, 64, 128, false, false, true, true, 0, 16384>(A, B, D, st);   // [K;Q] K^T
    case 12: return run<128, 256, 64, false, true, false, true, 0, 16384>(A, B, D, st);   // [T';T''] [K|V]
    case 13: return run<128, 32, 128, false, true, true, false>(A, B, D, st);             // [W;Q] h
    case 14: return run<128, 32, 64, false, true, false, false>(A, B, D, st);             // [0;P] v_new
    case 15: return run<128, 128, 128, false, true, true, false>(A, B, D, st);            // [W;Q] h, VS=128
    default: return -1;
  }
}
