// Test-only kernel: one tcgen05 MMA D[M][N] = sum_k A(m,k) B(n,k) with the
// operand images, descriptors and TMEM read-back conventions of the product
// kernels (domesticated_torch_mlu_ops_b200/csrc/umma.cuh).  A is given as
// [M][K] (K-major) or [K][M] (a_mn), B as [N][K] or [K][N] (b_mn), bf16.
#include <cuda_bf16.h>
#include <stdint.h>

#include "umma.cuh"

using namespace gdn::umma;

template <int M, int N, int K, bool AMN, bool BMN>
__global__ void __launch_bounds__(128) selftest(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                                float* Dout, int* status) {
  extern __shared__ __align__(1024) uint8_t sm[];
  constexpr int ACOLS = AMN ? M : K, AROWS = AMN ? K : M;
  constexpr int BCOLS = BMN ? N : K, BROWS = BMN ? K : N;
  constexpr int RSA = (ACOLS / 8) * 128, RSB = (BCOLS / 8) * 128;
  uint8_t* aimg = sm;
  uint8_t* bimg = sm + AROWS * ACOLS * 2;
  uint64_t* bar = reinterpret_cast<uint64_t*>(bimg + BROWS * BCOLS * 2);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < AROWS * ACOLS; e += 128) {
    const int r = e / ACOLS, c = e % ACOLS;
    *reinterpret_cast<__nv_bfloat16*>(aimg + img_off(r, c, RSA)) = A[e];
  }
  for (int e = tid; e < BROWS * BCOLS; e += 128) {
    const int r = e / BCOLS, c = e % BCOLS;
    *reinterpret_cast<__nv_bfloat16*>(bimg + img_off(r, c, RSB)) = B[e];
  }
  if (warp == 0) { tmem_alloc(tslot, 256); fence_before_sync(); }
  if (tid == 0) { mbar_init(bar, 1); mbar_fence_init(); }
  fence_proxy_async();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    const uint32_t id = idesc_f16(M, N, true, AMN, BMN);
    const uint32_t aa = smem_u32(aimg), ba = smem_u32(bimg);
    for (int ks = 0; ks < K / 16; ++ks) {
      const uint64_t ad = AMN ? smem_desc(aa + ks * 2 * RSA, RSA, 128) : smem_desc(aa + ks * 256, 128, RSA);
      const uint64_t bd = BMN ? smem_desc(ba + ks * 2 * RSB, RSB, 128) : smem_desc(ba + ks * 256, 128, RSB);
      mma_f16(tmem, ad, bd, id, ks > 0);
    }
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

template <int M, int N, int K, bool AMN, bool BMN>
static int run(const void* A, const void* B, float* D, int* st) {
  auto k = selftest<M, N, K, AMN, BMN>;
  const int smem = (M * K + N * K) * 2 + 64;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k<<<1, 128, smem>>>(static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, st);
  return static_cast<int>(cudaDeviceSynchronize());
}

extern "C" int umma_selftest(int which, const void* A, const void* B, float* D, int* st) {
  switch (which) {
    case 0: return run<64, 64, 128, false, false>(A, B, D, st);   // S = K K^T
    case 1: return run<64, 128, 64, false, true>(A, B, D, st);    // W = T' K
    case 2: return run<128, 32, 64, true, true>(A, B, D, st);     // dH = K^T V~
    case 3: return run<64, 32, 128, false, true>(A, B, D, st);    // X = W h
    case 4: return run<128, 128, 64, true, true>(A, B, D, st);    // dH, VS = 128
    case 5: return run<64, 64, 64, false, true>(A, B, D, st);     // O = P v_new, VS = 64
    default: return -1;
  }
}
