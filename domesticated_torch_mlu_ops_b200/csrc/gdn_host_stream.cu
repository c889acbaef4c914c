// gdn_chunk_fwd_host: the chunked prefill for inputs and outputs in host
// memory, with the host link pipelined against the kernels.
//
// The tokens are cut into pieces of about `segment_tokens` tokens: one
// sequence (B = 1, no cu_seqlens) along time at 64-token chunk boundaries,
// its fp32 state handed from piece to piece in device memory and its last
// segment in halving pieces; an
// equal-length batch into groups of sequences; a packed varlen batch into
// groups of consecutive sequences.  Piece p + 1 is copied in on one
// library-owned stream while piece p runs on the caller's stream and piece
// p - 1's output is copied out on a second library-owned stream; two device
// slots alternate, ordered by events.  Every piece is one gdn_chunk_fwd call
// on device copies, so the results are those of the device entry point.

#include <mutex>
#include <string.h>
#include <vector>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace {

constexpr int kMaxDevices = 128;
constexpr int64_t kTailMin = 512;  // tokens: the shortest piece of a time split's tail

struct CopyStreams {
  cudaStream_t in = nullptr, out = nullptr;
};
std::mutex g_stream_mutex;
CopyStreams g_streams[kMaxDevices];

// The two copy streams of the current device, created on first use and kept
// for the life of the process.
cudaError_t copy_streams(CopyStreams& cs) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_stream_mutex);
  CopyStreams& s = g_streams[dev];
  if (!s.in && (e = cudaStreamCreateWithFlags(&s.in, cudaStreamNonBlocking)) != cudaSuccess) return e;
  if (!s.out && (e = cudaStreamCreateWithFlags(&s.out, cudaStreamNonBlocking)) != cudaSuccess) return e;
  cs = s;
  return cudaSuccess;
}

struct Piece {
  int64_t t0, t1;  // flattened token range
  int64_t s0, s1;  // sequence range (time pieces: 0, 1)
  int64_t B, T;    // call shape
};

size_t esize(int dtype) { return dtype == GDN_F32 ? 4 : 2; }
size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct Plan {
  std::vector<Piece> pieces;
  std::vector<int64_t> cu;  // host copy of cu_seqlens (int64), packed inputs only
  bool time_split = false, packed = false;
  int64_t max_tok = 1, max_seq = 1;
  size_t q, k, v, g, b, o, cuo, h0, ht, slot;  // slot layout (offsets within a slot)
  size_t chain, ws, ws_bytes, total;
};

int64_t state_elems(const gdn_chunk_args& a) { return static_cast<int64_t>(a.HV) * a.K * a.V; }

gdn_chunk_args piece_args(const gdn_chunk_args& a, const Piece& p, bool packed) {
  gdn_chunk_args c{};
  c.B = p.B;
  c.T = p.T;
  c.N = p.s1 - p.s0;
  c.H = a.H;
  c.HV = a.HV;
  c.K = a.K;
  c.V = a.V;
  c.qkv_dtype = a.qkv_dtype;
  c.cu_dtype = GDN_I64;
  c.scale = a.scale;
  c.use_qk_l2norm = a.use_qk_l2norm;
  c.state_v_first = a.state_v_first;
  c.force_generic = a.force_generic;
  if (packed) c.cu_seqlens = reinterpret_cast<const void*>(uintptr_t(256));  // sizing only: marks varlen
  return c;
}

int make_plan(const gdn_chunk_args& a, int64_t seg, Plan& P) {
  const int64_t Ttot = a.B * a.T;
  P.packed = a.cu_seqlens != nullptr;
  P.time_split = !P.packed && a.B == 1;
  if (P.packed) {
    P.cu.resize(a.N + 1);
    for (int64_t i = 0; i <= a.N; ++i)
      P.cu[i] = a.cu_dtype == GDN_I64 ? static_cast<const int64_t*>(a.cu_seqlens)[i]
                                      : static_cast<const int32_t*>(a.cu_seqlens)[i];
    if (P.cu[0] != 0 || P.cu[a.N] != Ttot)
      return gdn::set_last_error(GDN_ERR_INVALID, "cu_seqlens must run from 0 to B*T=%lld", (long long)Ttot);
    for (int64_t i = 0; i < a.N; ++i)
      if (P.cu[i + 1] < P.cu[i]) return gdn::set_last_error(GDN_ERR_INVALID, "cu_seqlens must not decrease");
    for (int64_t s0 = 0; s0 < a.N;) {
      int64_t s1 = s0 + 1;
      while (s1 < a.N && P.cu[s1] - P.cu[s0] < seg) ++s1;
      P.pieces.push_back({P.cu[s0], P.cu[s1], s0, s1, 1, P.cu[s1] - P.cu[s0]});
      s0 = s1;
    }
  } else if (P.time_split) {
    // Pieces of `seg` tokens, except that the last `seg` (or fewer) are cut
    // into halving pieces (seg/2, seg/4, ... down to kTailMin, then the rest):
    // nothing overlaps the compute and the copy-out of the last piece, so a
    // short last piece shortens the call by most of a full piece's copy-out.
    const int64_t tail0 = a.T > seg ? ((a.T - seg) / 64) * 64 : 0;  // every piece starts on a chunk boundary
    for (int64_t t0 = 0; t0 < tail0; t0 += seg) {
      const int64_t t1 = t0 + seg < tail0 ? t0 + seg : tail0;
      P.pieces.push_back({t0, t1, 0, 1, 1, t1 - t0});
    }
    for (int64_t t0 = tail0; t0 < a.T;) {
      const int64_t left = a.T - t0;
      int64_t n = ((left / 2) / 64) * 64;
      if (n < kTailMin || left - n < kTailMin) n = left;
      P.pieces.push_back({t0, t0 + n, 0, 1, 1, n});
      t0 += n;
    }
  } else if (a.T > 0) {
    const int64_t per = seg / a.T > 0 ? seg / a.T : 1;
    for (int64_t b0 = 0; b0 < a.B; b0 += per) {
      const int64_t b1 = b0 + per < a.B ? b0 + per : a.B;
      P.pieces.push_back({b0 * a.T, b1 * a.T, b0, b1, b1 - b0, a.T});
    }
  }
  size_t ws = 0;
  for (const Piece& p : P.pieces) {
    P.max_tok = p.t1 - p.t0 > P.max_tok ? p.t1 - p.t0 : P.max_tok;
    P.max_seq = p.s1 - p.s0 > P.max_seq ? p.s1 - p.s0 : P.max_seq;
    gdn_chunk_args c = piece_args(a, p, P.packed);
    const size_t w = gdn_chunk_workspace_size(&c);
    if (w == 0) return GDN_ERR_INVALID;  // message set by the sizing call
    ws = w > ws ? w : ws;
  }
  const size_t es = esize(a.qkv_dtype), se = sizeof(float) * state_elems(a);
  size_t o = 0;
  P.q = o; o += al256(P.max_tok * a.H * a.K * es);
  P.k = o; o += al256(P.max_tok * a.H * a.K * es);
  P.v = o; o += al256(P.max_tok * a.HV * a.V * es);
  P.g = o; o += al256(P.max_tok * a.HV * sizeof(float));
  P.b = o; o += al256(P.max_tok * a.HV * sizeof(float));
  P.o = o; o += al256(P.max_tok * a.HV * a.V * es);
  P.cuo = o; o += al256((P.max_seq + 1) * sizeof(int64_t));
  P.h0 = o; o += al256(P.max_seq * se);
  P.ht = o; o += al256(P.max_seq * se);
  P.slot = o;
  P.chain = 2 * P.slot;
  P.ws = P.chain + 2 * al256(se);
  P.ws_bytes = ws;
  P.total = P.ws + al256(ws);
  return GDN_OK;
}

int check_args(const gdn_chunk_args* a, int64_t seg) {
  if (!a) return gdn::set_last_error(GDN_ERR_INVALID, "null args");
  if (seg <= 0 || seg % 64)
    return gdn::set_last_error(GDN_ERR_INVALID, "segment_tokens=%lld must be a positive multiple of 64",
                               (long long)seg);
  if (a->q_token_stride || a->k_token_stride || a->v_token_stride)
    return gdn::set_last_error(GDN_ERR_UNSUPPORTED, "the host-memory prefill takes packed q/k/v rows");
  gdn_chunk_args c = *a;  // shape and dtype checks of the device entry point
  if (gdn_chunk_workspace_size(&c) == 0) return GDN_ERR_INVALID;
  return GDN_OK;
}

}  // namespace

extern "C" {

size_t gdn_chunk_fwd_host_buffer_size(const gdn_chunk_args* a, int64_t segment_tokens) {
  if (check_args(a, segment_tokens)) return 0;
  Plan P;
  if (make_plan(*a, segment_tokens, P)) return 0;
  return P.total;
}

int gdn_chunk_fwd_host(const gdn_chunk_args* a, int64_t segment_tokens, void* stream) {
  int rc = check_args(a, segment_tokens);
  if (rc) return rc;
  const int64_t Ttot = a->B * a->T;
  if (Ttot > 0 && (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->o))
    return gdn::set_last_error(GDN_ERR_INVALID, "q, k, v, g, beta and o must be non-null");
  Plan P;
  if ((rc = make_plan(*a, segment_tokens, P))) return rc;
  if (!a->workspace || a->workspace_bytes < P.total)
    return gdn::set_last_error(GDN_ERR_WORKSPACE, "device buffer of %zu bytes given, %zu needed",
                               a->workspace_bytes, P.total);
  const size_t es = esize(a->qkv_dtype);
  const int64_t se = state_elems(*a);
  const size_t seb = sizeof(float) * se;
  if (P.pieces.empty()) {  // no tokens: the final state is the initial one
    if (a->final_state) {
      const size_t n = seb * a->N;
      if (a->initial_state) memcpy(a->final_state, a->initial_state, n);
      else memset(a->final_state, 0, n);
    }
    return GDN_OK;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CopyStreams cs;
  cudaError_t e = copy_streams(cs);
  if (e != cudaSuccess) return gdn::set_last_error(GDN_ERR_CUDA, "copy streams: %s", cudaGetErrorString(e));
  cudaEvent_t ev[9] = {};  // in[2], cmp[2], out[2], entry, exit_in, exit_out
  for (int i = 0; i < 9 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  cudaEvent_t *ev_in = ev, *ev_cmp = ev + 2, *ev_out = ev + 4;
  char* dbuf = static_cast<char*>(a->workspace);
  const char* hq = static_cast<const char*>(a->q);
  const char* hk = static_cast<const char*>(a->k);
  const char* hv = static_cast<const char*>(a->v);
  char* ho = static_cast<char*>(a->o);
  const int64_t rq = static_cast<int64_t>(a->H) * a->K, rv = static_cast<int64_t>(a->HV) * a->V;
  float* chain[2] = {reinterpret_cast<float*>(dbuf + P.chain), reinterpret_cast<float*>(dbuf + P.chain + al256(seb))};
  std::vector<int64_t> cu_piece;
  auto cp = [&](void* dst, const void* src, size_t n, cudaMemcpyKind kind, cudaStream_t st) {
    if (e == cudaSuccess && n) e = cudaMemcpyAsync(dst, src, n, kind, st);
  };
  if (e == cudaSuccess) e = cudaEventRecord(ev[6], s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs.in, ev[6], 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs.out, ev[6], 0);
  if (P.time_split && a->initial_state) cp(chain[1], a->initial_state, seb, cudaMemcpyHostToDevice, cs.in);
  for (size_t pi = 0; pi < P.pieces.size() && e == cudaSuccess && rc == GDN_OK; ++pi) {
    const Piece& p = P.pieces[pi];
    const int sl = static_cast<int>(pi & 1);
    char* base = dbuf + sl * P.slot;
    const int64_t nt = p.t1 - p.t0, ns = p.s1 - p.s0;
    // ---- copy in (slot free once the compute of piece pi - 2 is done)
    if (pi >= 2 && e == cudaSuccess) e = cudaStreamWaitEvent(cs.in, ev_cmp[sl], 0);
    cp(base + P.q, hq + p.t0 * rq * es, nt * rq * es, cudaMemcpyHostToDevice, cs.in);
    cp(base + P.k, hk + p.t0 * rq * es, nt * rq * es, cudaMemcpyHostToDevice, cs.in);
    cp(base + P.v, hv + p.t0 * rv * es, nt * rv * es, cudaMemcpyHostToDevice, cs.in);
    cp(base + P.g, a->g + p.t0 * a->HV, nt * a->HV * sizeof(float), cudaMemcpyHostToDevice, cs.in);
    cp(base + P.b, a->beta + p.t0 * a->HV, nt * a->HV * sizeof(float), cudaMemcpyHostToDevice, cs.in);
    if (P.packed) {
      cu_piece.assign(P.cu.begin() + p.s0, P.cu.begin() + p.s1 + 1);
      for (int64_t& c : cu_piece) c -= P.cu[p.s0];
      cp(base + P.cuo, cu_piece.data(), (ns + 1) * sizeof(int64_t), cudaMemcpyHostToDevice, cs.in);
    }
    if (!P.time_split && a->initial_state)
      cp(base + P.h0, a->initial_state + p.s0 * se, ns * seb, cudaMemcpyHostToDevice, cs.in);
    if (e == cudaSuccess) e = cudaEventRecord(ev_in[sl], cs.in);
    // ---- compute on the caller's stream (output slot free once piece pi - 2 is copied out)
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev_in[sl], 0);
    if (pi >= 2 && e == cudaSuccess) e = cudaStreamWaitEvent(s, ev_out[sl], 0);
    if (e != cudaSuccess) break;
    gdn_chunk_args c = piece_args(*a, p, P.packed);
    c.q = base + P.q;
    c.k = base + P.k;
    c.v = base + P.v;
    c.g = reinterpret_cast<const float*>(base + P.g);
    c.beta = reinterpret_cast<const float*>(base + P.b);
    c.o = base + P.o;
    c.cu_seqlens = P.packed ? base + P.cuo : nullptr;
    if (P.time_split) {
      c.initial_state = (pi > 0 || a->initial_state) ? chain[(pi + 1) & 1] : nullptr;
      c.final_state = chain[pi & 1];
    } else {
      c.initial_state = a->initial_state ? reinterpret_cast<const float*>(base + P.h0) : nullptr;
      c.final_state = a->final_state ? reinterpret_cast<float*>(base + P.ht) : nullptr;
    }
    c.workspace = dbuf + P.ws;
    c.workspace_bytes = P.ws_bytes;
    rc = gdn_chunk_fwd(&c, s);
    if (rc != GDN_OK) break;
    e = cudaEventRecord(ev_cmp[sl], s);
    // ---- copy out
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs.out, ev_cmp[sl], 0);
    cp(ho + p.t0 * rv * es, base + P.o, nt * rv * es, cudaMemcpyDeviceToHost, cs.out);
    if (a->final_state && !P.time_split)
      cp(a->final_state + p.s0 * se, base + P.ht, ns * seb, cudaMemcpyDeviceToHost, cs.out);
    if (a->final_state && P.time_split && pi + 1 == P.pieces.size())
      cp(a->final_state, chain[pi & 1], seb, cudaMemcpyDeviceToHost, cs.out);
    if (e == cudaSuccess) e = cudaEventRecord(ev_out[sl], cs.out);
  }
  // the caller's stream waits for both copy streams, on success and on failure
  cudaError_t e2 = cudaEventRecord(ev[7], cs.in);
  if (e2 == cudaSuccess) e2 = cudaEventRecord(ev[8], cs.out);
  if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(s, ev[7], 0);
  if (e2 == cudaSuccess) e2 = cudaStreamWaitEvent(s, ev[8], 0);
  for (cudaEvent_t x : ev)
    if (x) cudaEventDestroy(x);
  if (rc != GDN_OK) return rc;
  if (e == cudaSuccess) e = e2;
  if (e != cudaSuccess) return gdn::set_last_error(GDN_ERR_CUDA, "gdn_chunk_fwd_host: %s", cudaGetErrorString(e));
  return GDN_OK;
}

}  // extern "C"
