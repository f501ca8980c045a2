// Pieces shared by the selective-scan kernels: parameter block, shared-memory
// layout, launch-shape choice, the fused Cayley step and the readout reduction.
#pragma once

#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace scan {

constexpr int kStages = 2;          // bulk-copy ring depth for shared B/C
constexpr int kMaxThreads = 768;    // CTA size cap (G = 4 kernels)
constexpr int kMaxThreadsG8 = 512;  // CTA size cap (G = 8 kernels, more registers per thread)
constexpr int kMaxDxPerThread = 2;  // delta / s elements staged per thread per chunk
constexpr int kMaxTc = 32;          // timesteps per staged chunk
constexpr size_t kSmemBudget = 200 * 1024;
constexpr long long kDefaultPollLimit = 1ll << 22;

struct FwdParams {
  int B, T, D, N;
  float eps;
  const void* delta;
  const float* lam;
  const void* q;
  const void* Bm;
  const void* Cm;
  const void* s;
  const float* dskip;
  int64_t dsb, dst, dsd;
  const float* h0;
  void* y;
  float* hT;
  int* status;
  long long wait_limit;
  float* pout;     // [B, D, N, 4] operator product (state-only pass) or nullptr
  float* ckpt;     // [B, nck, D, N, 4] or nullptr
  int ckpt_every;  // K: checkpoint after steps K-1, 2K-1, ... < T-1
  int nck;         // number of checkpoints = ceil(T / K) - 1
  int nb;   // CTAs per batch row
  int cpb;  // max channels per CTA
  int tc;   // timesteps per chunk
  // Peer outputs of the channel-sharded scan (packed kernel only): with npeer > 0
  // y goes to every ypeer[r] instead of y, each laid out as rows of y_ld elements
  // per (batch, time) step with this shard's channels starting at element y_coff.
  int npeer;
  int64_t y_ld, y_coff;
  void* ypeer[8];
  // With peer_mc set (npeer == 1), ypeer[0] is the multicast address of a
  // buffer bound on every rank (NVLink SHARP): each y quaternion is stored once
  // with multimem.st and the switch writes it to all ranks.
  int peer_mc;
};
constexpr int kMaxPeerOutputs = 8;

struct SmemLayout {
  size_t off_b, off_c, off_delta, off_s, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <typename T, bool S_REAL>
__host__ __device__ inline SmemLayout smem_layout(int tc, int cpb, int N, bool bc_shared) {
  SmemLayout L;
  size_t off = 128;  // mbarriers
  const size_t ring = bc_shared ? size_t(kStages) * tc * N * 4 * sizeof(T) : 0;
  L.off_b = off;
  off = align_up(off + ring, 128);
  L.off_c = off;
  off = align_up(off + ring, 128);
  L.off_delta = off;
  off = align_up(off + size_t(2) * tc * cpb * sizeof(float), 16);
  L.off_s = off;
  off = align_up(off + size_t(2) * tc * cpb * (S_REAL ? 1 : 4) * sizeof(float), 16);
  L.total = off;
  return L;
}

// Per-(d, n) constants of the fused Cayley map, from Lambda = (l_r, l_i, l_j, l_k):
// lr = l_r, (li, lj, lk) = Im Lambda, m = |Lambda|^2 / 4.
struct LamConst {
  float lr, li, lj, lk, m;
};

__device__ __forceinline__ LamConst make_lam_const(float4 lam) {
  return LamConst{lam.x, lam.y, lam.z, lam.w,
                  0.25f * fmaf(lam.x, lam.x, fmaf(lam.y, lam.y, fmaf(lam.z, lam.z, lam.w * lam.w)))};
}

// q = Cayley(delta * Lambda) in closed form, without forming z. With
// w = delta*Lambda/2 = a + v and P = |w|^2 = delta^2 m:
//   |1 - w|^2 = (1-a)^2 + |v|^2 = 1 + P - delta*l_r      (clamped below by eps)
//   conj(1 - w) (x) (1 + w) = (1 - P) + delta * Im Lambda
// so q = ((1 - P), delta * Im Lambda) / max(1 + P - delta l_r, eps).
__device__ __forceinline__ float4 cayley_from_const(float dl, float dl2, const LamConst& c,
                                                    float eps) {
  const float P = dl2 * c.m;
  const float den = fmaxf(fmaf(-dl, c.lr, 1.f + P), eps);
  const float inv = rcp_nr(den);
  const float s = dl * inv;
  return make_float4(fmaf(-P, inv, inv), s * c.li, s * c.lj, s * c.lk);
}

// Stores the G states of one lane as checkpoint k (state after step (k+1)*K - 1).
template <int G, int NG>
__device__ __forceinline__ void store_ckpt(const FwdParams& p, int b, int c, int ng, int k,
                                           const float4 (&h)[G]) {
  float* base = p.ckpt + ((int64_t(b) * p.nck + k) * p.D + c) * int64_t(p.N) * 4;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    if (n < p.N) QIO<float>::st(base + int64_t(n) * 4, h[i]);
  }
}

__device__ __forceinline__ float f4_get(const float4& v, int k) {
  return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

// Sums the per-thread partial readouts `a` over the NG lanes of one channel
// (a reduce-scatter: after it, lane ng holds component ng & 3) and stores
// y = sum + dsk * S. All 32 lanes of the warp must call it.
template <typename T, int NG>
__device__ __forceinline__ void reduce_store_y(float4 a, float4 sv, float dsk, int ng,
                                               bool active, T* yp) {
  constexpr unsigned kFull = 0xffffffffu;
  if constexpr (NG == 1) {
    if (active) {
      a.x = fmaf(dsk, sv.x, a.x);
      a.y = fmaf(dsk, sv.y, a.y);
      a.z = fmaf(dsk, sv.z, a.z);
      a.w = fmaf(dsk, sv.w, a.w);
      QIO<T>::st(yp, a);
    }
  } else {
    const bool odd = ng & 1;
    const float s0 = odd ? a.x : a.y;
    const float s1 = odd ? a.z : a.w;
    const float r0 = __shfl_xor_sync(kFull, s0, 1);
    const float r1 = __shfl_xor_sync(kFull, s1, 1);
    const float k0 = (odd ? a.y : a.x) + r0;  // component (odd)
    const float k1 = (odd ? a.w : a.z) + r1;  // component (odd + 2)
    if constexpr (NG == 2) {
      if (active) {
        const int c0 = odd ? 1 : 0;
        QIO<T>::st1(yp + c0, fmaf(dsk, f4_get(sv, c0), k0));
        QIO<T>::st1(yp + c0 + 2, fmaf(dsk, f4_get(sv, c0 + 2), k1));
      }
    } else {
      const bool hi = (ng >> 1) & 1;
      const float snd = hi ? k0 : k1;
      const float r = __shfl_xor_sync(kFull, snd, 2);
      float v = (hi ? k1 : k0) + r;
#pragma unroll
      for (int m = 4; m < NG; m <<= 1) v += __shfl_xor_sync(kFull, v, m);
      if (active && ng < 4) QIO<T>::st1(yp + ng, fmaf(dsk, f4_get(sv, ng), v));
    }
  }
}

// Lanes per channel: the power of two covering ceil(N / G) with G = 4 (8 above
// N = 128), at most 32.
inline int lanes_per_channel(int N) {
  const int g = N > 128 ? 8 : 4;
  const int need = (N + g - 1) / g;
  int ng = 1;
  while (ng < need) ng <<= 1;
  return ng <= 32 ? ng : 0;
}

struct LaunchShape {
  int nb, cpb, tc, threads;
  size_t smem;
  const char* why;
};

// Balanced partition: each batch row's D channels are split into nb contiguous
// ranges of floor/ceil(D/nb) channels so that B*nb CTAs cover the SMs once.
inline LaunchShape choose_shape(int B, int T, int D, int N, int NG, int esize, bool bc_shared,
                                bool s_real) {
  LaunchShape ls{0, 0, 0, 0, 0, ""};
  const int max_threads = N > 128 ? kMaxThreadsG8 : kMaxThreads;
  const int sms = num_sms();
  int nb = sms / B;  // B * nb <= #SMs: no partial second wave
  if (nb > D) nb = D;
  if (nb < 1) nb = 1;
  int cpb = (D + nb - 1) / nb;
  const int cap = max_threads / NG;
  if (cpb > cap) {
    nb = (D + cap - 1) / cap;
    cpb = (D + nb - 1) / nb;
  }
  const int threads = (cpb * NG + 31) / 32 * 32;
  int tc = kMaxTc;
  while (tc > 1 && tc * cpb > kMaxDxPerThread * threads) tc >>= 1;
  if (tc > T) tc = T < 1 ? 1 : T;
  size_t smem = 0;
  for (;;) {
    smem = s_real ? (esize == 4 ? smem_layout<float, true>(tc, cpb, N, bc_shared).total
                                : smem_layout<__nv_bfloat16, true>(tc, cpb, N, bc_shared).total)
                  : (esize == 4 ? smem_layout<float, false>(tc, cpb, N, bc_shared).total
                                : smem_layout<__nv_bfloat16, false>(tc, cpb, N, bc_shared).total);
    if (smem <= kSmemBudget || tc == 1) break;
    tc >>= 1;
  }
  if (smem > kSmemBudget) {
    ls.why = "shared-memory staging does not fit (d_state too large)";
    return ls;
  }
  ls.nb = nb;
  ls.cpb = cpb;
  ls.tc = tc;
  ls.threads = threads;
  ls.smem = smem;
  return ls;
}

// Warp-specialised kernel for channel-shared B/C without explicit q
// (ssm_scan_fwd_shared.cu).
int dispatch_shared(const FwdParams& p, int dtype, bool s_real, cudaStream_t st);
// The same with packed two-lane FP32 arithmetic over pair-interleaved B/C rows
// (ssm_scan_fwd_packed.cu).
int dispatch_shared_packed(const FwdParams& p, int dtype, bool s_real, cudaStream_t st);
// Rewrites channel-shared B and C [rows, N, 4] (dtype) into fp32 pair-interleaved
// rows of NG*G states, [pair j][lane ng][component][half] with state
// n = ng + NG*(2j + half), zero-padded above N (Cm may be null: C skipped).
int pack_bc_pairs(const void* Bm, const void* Cm, float* Bp, float* Cp, int64_t rows, int N,
                  int NG, int G, int dtype, cudaStream_t st);
// bf16 -> fp32, n elements.
int widen_bf16_to_f32(const void* in, float* out, int64_t n, cudaStream_t st);
// Pass 1 of the time-chunked scan on the packed kernel (channel-shared B/C).
int dispatch_state_only_packed(const FwdParams& p, int dtype, bool s_real, cudaStream_t st);
// Streaming kernel for per-channel B/C and explicit q (ssm_scan_fwd_stream.cu).
int dispatch_stream(const FwdParams& p, int dtype, bool s_real, bool q_given, cudaStream_t st);
// Streaming kernel for channel-shared B/C (short sequences).
int dispatch_stream_shared(const FwdParams& p, int dtype, bool s_real, cudaStream_t st);
// One decode step (T = 1, channel-shared B/C, no checkpoints or operator
// product) on the batch-blocked decode kernel (ssm_scan_decode.cu).
bool decode_serves(const FwdParams& p);
int dispatch_decode(const FwdParams& p, int dtype, bool s_real, cudaStream_t st);
// Sequences up to this length with channel-shared B/C skip the packed kernel's
// pre-pass and producer pipeline and take the streaming kernel.
constexpr int kShortScan = 8;
// Pass 1 of the time-chunked scan: final state + operator product, no readout.
int dispatch_state_only(const FwdParams& p, int dtype, bool s_real, bool bc_shared,
                        cudaStream_t st);

inline int validate_and_fill(const mqc_ssm_scan_args* a, FwdParams* p, const char* name) {
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(dtype_ok(a->dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, a->dtype);
  MQC_REQUIRE((a->flags & ~(MQC_SSM_Q_GIVEN | MQC_SSM_BC_SHARED | MQC_SSM_S_REAL)) == 0,
              MQC_ERR_INVALID_VALUE, "%s: unknown flag bits 0x%x", name, a->flags);
  MQC_REQUIRE(a->batch >= 0 && a->seq_len >= 0 && a->channels >= 0 && a->d_state >= 0,
              MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(a->batch <= 65535 && a->seq_len < (1ll << 31) && a->channels < (1ll << 31),
              MQC_ERR_UNSUPPORTED, "%s: size out of range (batch <= 65535)", name);
  MQC_REQUIRE(a->d_state <= 256, MQC_ERR_UNSUPPORTED, "%s: d_state=%lld > 256", name,
              (long long)a->d_state);
  p->B = int(a->batch);
  p->T = int(a->seq_len);
  p->D = int(a->channels);
  p->N = int(a->d_state);
  if (p->B == 0 || p->T == 0 || p->D == 0) return MQC_OK;
  MQC_REQUIRE(p->N >= 1, MQC_ERR_INVALID_VALUE, "%s: d_state must be >= 1", name);
  const bool qg = a->flags & MQC_SSM_Q_GIVEN;
  const bool sh = a->flags & MQC_SSM_BC_SHARED;
  const bool sr = a->flags & MQC_SSM_S_REAL;
  MQC_REQUIRE(a->y && a->s && a->Bm && a->Cm, MQC_ERR_INVALID_VALUE,
              "%s: y, s, Bm and Cm are required", name);
  if (qg) {
    MQC_REQUIRE(a->q != nullptr, MQC_ERR_INVALID_VALUE, "%s: q required with Q_GIVEN", name);
  } else {
    MQC_REQUIRE(a->delta && a->lambda_, MQC_ERR_INVALID_VALUE,
                "%s: delta and lambda_ are required without Q_GIVEN", name);
    MQC_REQUIRE(!(a->eps < 0.f), MQC_ERR_INVALID_VALUE, "%s: eps must be >= 0", name);
  }
  const uintptr_t qa = a->dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(a->y, qa) && (qg ? aligned(a->q, qa) : true) && (sr || aligned(a->s, qa)),
              MQC_ERR_MISALIGNED, "%s: quaternion tensors must be %d-byte aligned", name,
              int(qa));
  if (sh) {
    MQC_REQUIRE(aligned(a->Bm, 16) && aligned(a->Cm, 16), MQC_ERR_MISALIGNED,
                "%s: shared B/C must be 16-byte aligned (bulk copies)", name);
    MQC_REQUIRE(a->dtype == MQC_DTYPE_F32 || (p->N % 2) == 0, MQC_ERR_UNSUPPORTED,
                "%s: bf16 shared B/C needs an even d_state", name);
  } else {
    MQC_REQUIRE(aligned(a->Bm, qa) && aligned(a->Cm, qa), MQC_ERR_MISALIGNED,
                "%s: B/C must be %d-byte aligned", name, int(qa));
  }
  MQC_REQUIRE((a->lambda_ == nullptr || aligned(a->lambda_, 16)) &&
                  (a->h0 == nullptr || aligned(a->h0, 16)) &&
                  (a->hT == nullptr || aligned(a->hT, 16)),
              MQC_ERR_MISALIGNED, "%s: Lambda, h0, hT must be 16-byte aligned", name);
  MQC_REQUIRE(a->dskip != nullptr, MQC_ERR_INVALID_VALUE, "%s: dskip is required", name);
  p->eps = a->eps;
  p->delta = a->delta;
  p->lam = a->lambda_;
  p->q = a->q;
  p->Bm = a->Bm;
  p->Cm = a->Cm;
  p->s = a->s;
  p->dskip = a->dskip;
  p->dsb = a->dskip_sb;
  p->dst = a->dskip_st;
  p->dsd = a->dskip_sd;
  p->h0 = a->h0;
  p->y = a->y;
  p->hT = a->hT;
  p->status = a->status;
  p->wait_limit = a->wait_poll_limit < 0 ? kDefaultPollLimit : a->wait_poll_limit;
  p->ckpt = a->ckpt;
  p->ckpt_every = 0;
  p->nck = 0;
  if (a->ckpt != nullptr) {
    MQC_REQUIRE(a->ckpt_every == MQC_SSM_CKPT_EVERY, MQC_ERR_UNSUPPORTED,
                "%s: ckpt_every must be %d", name, MQC_SSM_CKPT_EVERY);
    MQC_REQUIRE(aligned(a->ckpt, 16), MQC_ERR_MISALIGNED, "%s: ckpt must be 16-byte aligned", name);
    p->ckpt_every = int(a->ckpt_every);
    p->nck = (p->T + p->ckpt_every - 1) / p->ckpt_every - 1;
  }
  if (lanes_per_channel(p->N) == 0)
    return fail(MQC_ERR_UNSUPPORTED, "%s: d_state=%d unsupported", name, p->N);
  return MQC_OK;
}

}  // namespace scan
}  // namespace mqc
