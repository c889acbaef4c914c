// solve_tril: (I + A)^-1 for each BT x BT chunk block of a strictly
// lower-triangular A, the op declared at include/torch_mlu_ops.h:1052-1054
// (Python wrapper _ops.py:6232-6257) whose native binary the reference does
// not ship.  Semantics follow the Python-level contract in
// triton/fla/solve_tril.py:491-537: A [B, T, H, BT] f32, output of the same
// shape in f32/bf16/f16, chunks of BT rows per sequence.
//
// The op has no workspace argument, so the grid is (sequence, head, slice)
// and slice z of a sequence solves its chunks z, z + S, z + 2S, ...; no chunk
// table is needed.  Each block is zero-padded to 64 x 64 in shared memory and
// inverted with the blocked solver of solve_tril.cuh, then written with
// explicit zeros above the diagonal and past a partial chunk's last row.

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "solve_tril.cuh"

namespace gdn {

template <typename TO>
__global__ void __launch_bounds__(128)
solve_tril_kernel(const float* __restrict__ A, TO* __restrict__ out, const void* cu, int cu_dtype,
                  int64_t T, int H, int BT) {
  __shared__ __align__(16) float As[64 * kTrilStride];
  __shared__ __align__(16) float Ts[64 * kTS];
  __shared__ __align__(16) float Zs[kTrilScratch];
  const int64_t n = blockIdx.x;
  const int h = blockIdx.y;
  int64_t bos, eos;
  seq_bounds(cu, cu_dtype, n, T, bos, eos);
  for (int64_t s = bos + static_cast<int64_t>(blockIdx.z) * BT; s < eos;
       s += static_cast<int64_t>(gridDim.z) * BT) {
    const int L = static_cast<int>(min64(BT, eos - s));
    for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {  // zero-padded to 64 x 64
      const int i = e >> 6, j = e & 63;
      As[i * kTrilStride + j] = (i < L && j < i) ? A[((s + i) * H + h) * BT + j] : 0.f;
    }
    __syncthreads();
    solve_tril64(As, Ts, Zs);
    for (int e = threadIdx.x; e < L * BT; e += blockDim.x) {
      const int i = e / BT, j = e % BT;
      out[((s + i) * H + h) * BT + j] = from_f<TO>(j < L ? Ts[i * kTS + j] : 0.f);
    }
    __syncthreads();
  }
}

cudaError_t launch_solve_tril(const float* A, void* out, int out_dtype, const void* cu,
                              int cu_dtype, int64_t N, int64_t B, int64_t T, int H, int BT,
                              cudaStream_t s) {
  const int64_t tot = cu ? T : B * T;
  if (N == 0 || H == 0 || tot == 0) return cudaSuccess;
  const int64_t avg_chunks = ((tot + BT - 1) / BT + N - 1) / N;
  const unsigned slices = static_cast<unsigned>(avg_chunks < 1 ? 1 : (avg_chunks > 1024 ? 1024 : avg_chunks));
  dim3 grid(static_cast<unsigned>(N), H, slices);
  note_launch();
  switch (out_dtype) {
    case GDN_F32:
      solve_tril_kernel<float><<<grid, 128, 0, s>>>(A, static_cast<float*>(out), cu, cu_dtype, T, H, BT);
      break;
    case GDN_BF16:
      solve_tril_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(A, static_cast<__nv_bfloat16*>(out), cu, cu_dtype, T, H, BT);
      break;
    case GDN_F16:
      solve_tril_kernel<__half><<<grid, 128, 0, s>>>(A, static_cast<__half*>(out), cu, cu_dtype, T, H, BT);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace gdn
