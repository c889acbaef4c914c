// Shared pieces of the tensor-core (tcgen05) chunked prefill kernels
// (gdn_chunk_tc.cu: separate WY and state kernels; gdn_chunk_fused.cu: the
// cluster kernel that computes both): sizes, the workspace carve-up, operand
// image layouts and small device helpers.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "umma.cuh"

namespace gdn {
namespace tc {

constexpr int D = 128;                  // K = V = 128
constexpr int kImg64x128 = 64 * D * 2;  // 16 KiB
constexpr int kImg64x64 = 64 * 64 * 2;  // 8 KiB
constexpr int RS64 = (64 / 8) * 128;    // image row stride of a 64-column tile
constexpr int kScal = 132;              // per-(head, chunk) scalars: a[64], b[64], gamma, pad
constexpr int kAtom = 64 * 128;         // one 64-row x 128-byte swizzled atom (8 KiB)
constexpr float kLog2e = 1.4426950408889634f;

struct Work {
  const int64_t* coff;  // [N+1] chunk offsets; null: N sequences of cps chunks each (no plan kernel)
  int64_t cps;          // chunks per sequence when coff is null
  int clear_err;        // the WY kernel's first block clears the error word (no plan kernel ran)
  int* err;             // device error word
  uint8_t* wimg;        // [HV][NCU][16 KiB]
  uint8_t* u;           // [HV][NCU][128/vs][64][vs] (rows swizzled; u_off)
  uint8_t* pimg;        // [HV][NCU][8 KiB]
  float* scal;          // [HV][NCU][kScal]: a[64], b[64], gamma, pad
  int64_t ncu;          // chunk capacity
  int vs;               // V-slice width of the state kernel (U layout)
  int* flags;           // [HV][NCU] tile-ready flags of the fused kernel (zeroed by the plan kernel)
  // Test hook (gdn_chunk_fwd_test_stall): block 0 of the state kernel skips
  // the operand fetch of chunk stall_chunk (-1: none) and bounds its waits by
  // stall_limit cycles, so that one wait runs out with nothing in flight.
  int64_t stall_chunk;
  long long stall_limit;
  // The backward's recompute (launch_state_store): the state kernel also
  // stores, per (chunk, v-head), the state at the chunk start and v_new as
  // bf16 operand images (bwd_img_off layouts); null otherwise.
  uint8_t* hs_img;
  uint8_t* vn_img;
  // The backward's recompute (launch_wy_only): the WY kernel also stores the
  // chunk-local cumsum of g ([Ttot][HV] fp32); null otherwise.
  float* gc_out;
};

// The causal conv1d applied by the WY kernel as it loads its tiles
// (causal_conv1d_fn, triton/conv/kernels.py:157-609, vLLM channel-last
// layout; width 4; x, weight, bias and the cache lines in the q/k/v dtype).
// x holds [q heads | k heads | v heads] channels per token.
struct ConvIn {
  const void* x;              // (dim, tokens): element (c, t) at x[t * sx + c]
  const void* weight;         // [dim, 4]
  const void* bias;           // [dim] or null
  const void* states;         // cache lines: (l, c, j) at l * st_seq + j * st_tok + c
  const void* cache_indices;  // [batch] (or [batch, blocks] with prefix caching) or null
  const uint8_t* has_init;    // [batch] or null
  const void* apc_init;       // prefix caching: column of cache_indices holding the initial line
  void* qc;                   // post-conv q [tokens][H][128] for the state kernel
  void* kc;                   // post-conv k [tokens][H][128]
  int64_t sx, st_seq, st_tok, ci_stride, pad_slot, null_block;
  int idx_dtype, apc_dtype, has_null, act;
};

struct Layout {
  size_t err, coff, wimg, u, pimg, scal, flags, qc, kc, total;
};

// conv: room for the post-conv q and k of the fused conv path.
inline Layout plan(const gdn_chunk_args& a, bool conv = false) {
  auto al = [](size_t x) { return (x + 1023) & ~static_cast<size_t>(1023); };
  const int64_t ncu = chunk_upper_bound(a.B * a.T, a.N);
  const size_t hc = static_cast<size_t>(a.HV) * ncu;
  Layout l{};
  size_t o = 0;
  l.err = o; o += al(16);
  l.coff = o; o += al(sizeof(int64_t) * (a.N + 1));
  l.wimg = o; o += al(hc * kImg64x128);
  l.u = o; o += al(hc * 64 * D * 2);
  l.pimg = o; o += al(hc * kImg64x64);
  l.scal = o; o += al(hc * kScal * 4);
  l.flags = o; o += al(hc * 4);
  const size_t qk = conv ? static_cast<size_t>(a.B * a.T) * a.H * D * 2 : 0;
  l.qc = o; o += al(qk);
  l.kc = o; o += al(qk);
  l.total = o;
  return l;
}

__device__ __forceinline__ void record_error(int* err, int code, int site) {
  record_device_error(err, code, site, linear_block_id(), static_cast<int>(threadIdx.x));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* x) {
  uint4 r;
  if constexpr (std::is_same<T, __half>::value) {
    r.x = pack_h2(x[0], x[1]); r.y = pack_h2(x[2], x[3]);
    r.z = pack_h2(x[4], x[5]); r.w = pack_h2(x[6], x[7]);
  } else {
    r.x = pack_bf16x2(x[0], x[1]); r.y = pack_bf16x2(x[2], x[3]);
    r.z = pack_bf16x2(x[4], x[5]); r.w = pack_bf16x2(x[6], x[7]);
  }
  return r;
}
template <typename T>
__device__ __forceinline__ void unpack8(uint4 u, float* x) {
  const T* p = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f<T>(p[i]);
}

// K-major descriptor of k-step ks (16 elements) of a 64-row swizzled tile.
__device__ __forceinline__ uint64_t sw_kmajor(uint32_t base, int ks) {
  return umma::smem_desc_sw128(base + (ks >> 2) * kAtom + (ks & 3) * 32, 16, 1024);
}
// MN-major descriptor (MN = the 128 tile columns, K = the 64 rows) of k-step ks.
__device__ __forceinline__ uint64_t sw_mnmajor(uint32_t base, int ks) {
  return umma::smem_desc_sw128(base + ks * 2048, kAtom, 1024);
}
// Both 64-column boxes of rows [s, s+64) of head hd of a [T, heads, 128] tensor.
__device__ __forceinline__ void tma_tile(uint8_t* dst, const CUtensorMap* map, int hd, int64_t s,
                                         uint32_t bar) {
  umma::tma_load_3d(dst, map, 0, hd, static_cast<int>(s), bar);
  umma::tma_load_3d(dst + kAtom, map, 64, hd, static_cast<int>(s), bar);
}

// Element offset of (row i, column c) in a U tile of S-column slices
// ([128/S][64][S], S = 32 or 64).  The 16-byte chunks of each row are
// XOR-swizzled so that eight consecutive rows touch distinct bank groups.
__device__ __forceinline__ int u_off(int i, int c, int S) {
  const bool s64 = S == 64;
  const int sw = s64 ? (i & 7) : ((i >> 1) & 3);  // (i / (8 / chunks per row)) mod chunks per row
  const int sl = c >> (s64 ? 6 : 5), wc = c & (S - 1);
  return (sl * 64 + i) * S + ((((wc >> 3) ^ sw)) << 3) + (wc & 7);
}

template <int VS_>
struct St3 {
  static constexpr int VS = VS_;
  // stage: W a0 | Q a0 | W a1 | Q a1 | K a0 | K a1 | P | U | scalars
  static constexpr int kWQ = 0;
  static constexpr int kK = 4 * kAtom;
  static constexpr int kP = kK + 2 * kAtom;
  static constexpr int kU = kP + kImg64x64;
  static constexpr int kUBytes = 64 * VS * 2;
  static constexpr int kSc = kU + kUBytes;
  static constexpr int kStage = ((kSc + kScal * 4 + 1023) / 1024) * 1024;
  static constexpr uint32_t kTx = 4 * kAtom + 2 * kAtom + kImg64x64 + kUBytes + kScal * 4;
  static constexpr int kStages = VS == 32 ? 3 : 2;  // a third 65 KB (73 KB) stage does not fit at VS = 64 (128)
  static constexpr int kH = kStages * kStage;    // h image 128 x VS
  static constexpr int kVn = kH + D * VS * 2;    // v image 64 x VS
  static constexpr int kVt = kVn + 64 * VS * 2;  // diag(b) v image 64 x VS
  static constexpr int kBar = kVt + 64 * VS * 2; // full[kStages], mma1, dh, o
  static constexpr int kTmem = kBar + 6 * 8;
  static constexpr int kBytes = kTmem + 8 + 1024;
  // TMEM columns: acc[2], dH, O[2] (VS each; one O buffer at VS = 128)
  static constexpr int kOBufs = VS == 128 ? 1 : 2;
  static constexpr int kAcc = 0, kDH = 2 * VS, kO = 3 * VS, kCols = VS == 32 ? 256 : 512;
  static_assert(kO + kOBufs * VS <= kCols, "TMEM columns");
  // U rows are read through the WY kernel's slices of at most 64 columns
  static constexpr int kUS = VS < 64 ? VS : 64;
  static_assert(kBytes <= 227 * 1024, "shared memory");
};
constexpr int kSt3Threads = 288;  // 8 epilogue warps + 1 load warp

// Operand images of the backward (global memory, one per chunk and v-head):
// a [rows][128] 16-bit matrix as two 128-byte-swizzled atoms of [rows][64]
// (columns 0-63, then 64-127), the layout TMA writes with 128-byte swizzle.
// rows = 128 for the states h and dh' (row = key index), 64 for v_new (row =
// token).  Byte offset of element (r, c):
__host__ __device__ constexpr uint32_t bwd_img_off(int r, int c, int rows) {
  return static_cast<uint32_t>((c >> 6) * rows * 128 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}
constexpr int kStateImg = 128 * 128 * 2;  // 32 KiB
constexpr int kVnImg = 64 * 128 * 2;      // 16 KiB

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry point.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();

// The forward's WY kernel alone (after its chunk plan) into a tensor-core
// workspace of tc_workspace_bytes(a) bytes at `ws`, for the backward's state
// recurrence (its W images and row scales); `w` gets the workspace pointers.
cudaError_t launch_wy_only(const gdn_chunk_args& a, void* ws, cudaStream_t s, Work& w, float* gc_out = nullptr);
// The forward state kernel (32-column slices) after launch_wy_only, for the
// backward's recompute: stores the state at every chunk start and v_new as
// bf16 images (hs_img, vn_img: [chunks][HV] images, bwd_img_off layouts);
// a.o and a.final_state null.
cudaError_t launch_state_store(const gdn_chunk_args& a, const Work& w, uint8_t* hs_img, uint8_t* vn_img,
                               cudaStream_t s);
// dv_local = scale P^T dO per (chunk, v-head) on tcgen05 (gdn_chunk_bwd_tc.cu),
// from the WY kernel's P images, into dvn ([Ttot][HV][V] fp32).
cudaError_t launch_bwd_dvlocal_tc(const gdn_chunk_bwd_args& b, const Work& w, float* dvn, cudaStream_t s);
// The backward's state-gradient recurrence on tcgen05 (gdn_chunk_bwd_tc.cu):
// reads dv_local from dvn ([Ttot][HV][V] fp32), writes dv and dh' of every
// chunk as bf16 images (dv_img: 64 rows, dh_img: 128 rows; [chunks][HV],
// bwd_img_off) and dh0.
cudaError_t launch_bwd_state_tc(const gdn_chunk_bwd_args& b, const Work& w, const float* dvn, uint8_t* dv_img,
                                uint8_t* dh_img, cudaStream_t s);
// dq, dk, dW and dG per (chunk, v-head) on tcgen05 (gdn_chunk_bwd_tc.cu),
// from the images above and G: writes the per-v-head dq, dk ([Ttot][HV][K]
// fp32, w.r.t. the normalised q, k) and dG as the generic bwd_dqkw_kernel
// does, and dW as an image.
struct DqkwOut {
  const uint8_t* dv_img;
  const float* gc;
  const uint8_t* hs_img;
  const uint8_t* dh_img;
  const uint8_t* vn_img;
  float *dqh, *dkh;
  uint8_t* dw_img;  // dW as a bf16 image (64 rows) for the WY-form gradient kernel
  float* dG;
};
cudaError_t launch_bwd_dqkw_tc(const gdn_chunk_bwd_args& b, const Work& w, const DqkwOut& o, cudaStream_t s);
// The WY-form gradients per (chunk, v-head) on tcgen05 (gdn_chunk_bwd_tc.cu):
// dv and dbeta into the call's outputs, dk (per v-head, w.r.t. the normalised
// k) and dG added to what the dq/dk kernel wrote, as the generic bwd_wy_kernel.
struct WyOut {
  const uint8_t* dv_img;  // dv (bf16 image, from the state-gradient kernel)
  const float* gc;        // G
  const uint8_t* dw_img;  // dW (bf16 image, from the dq/dk kernel)
  float *dkh, *dG;
};
cudaError_t launch_bwd_wy_tc(const gdn_chunk_bwd_args& b, const Work& w, const WyOut& o, cudaStream_t s);

// [Ttot, heads, 128] bf16/f16 tensor map with 64 x 64 boxes, 128-byte swizzle.
cudaError_t make_map(CUtensorMap* m, const void* ptr, int heads, int64_t ttot, bool f16, int64_t tstride = 0);

// The fused cluster kernel (gdn_chunk_fused.cu): whether clusters of it can
// be scheduled on the current device, and its launcher (tq, tk, tv as made by
// make_map; the workspace holds only the error word and chunk offsets it uses).
bool fused_launchable(bool f16);
template <typename T>
cudaError_t launch_fused(const gdn_chunk_args& a, const Work& w, float scale, const CUtensorMap& tq,
                         const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t s);

}  // namespace tc
}  // namespace gdn
