// Selective scan forward for per-channel B/C ([B,T,D,N,4], the reference block's
// layout) and for explicit operators q (ssm_forward_fused,
// mambaqc/kernels/ssm_fused.py:340-401): the streaming kernel.
//
// These modes move 32 B (B, C) or 48 B (with q) per (b, t, d, n) element that no
// other lane reuses, so the kernel is an HBM stream: per step a lane loads its
// G states' B_t/C_t (and q_t) for the NEXT step into registers while it computes
// the current one (one-step software pipeline), so every warp keeps
// 2 x G x 16 B (x 32 lanes) of reads in flight without any block barrier. Lanes
// of a channel read consecutive 16-byte quaternions (n = ng + NG*i), so each
// warp-wide load is fully coalesced. delta / x (or S) of the next step are
// prefetched the same way. Same per-element math as the fused kernels.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "packed_math.cuh"
#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {

constexpr int kStreamThreads = 256;

// BC_SHARED: B/C are [B,T,N,4] (stride 0 over channels) instead of [B,T,D,N,4].
// STATE_ONLY: no readout; the kernel returns the final state (p.hT) and the
// product of the step operators P = q_{T-1} (x) ... (x) q_0 (p.pout) -- pass 1
// of the time-chunked scan.
template <typename T, int G, int NG, bool S_REAL, bool Q_GIVEN, bool BC_SHARED = false,
          bool STATE_ONLY = false>
__global__ void __launch_bounds__(kStreamThreads)
    scan_fwd_stream_kernel(const FwdParams p) {
  constexpr int CPW = 32 / NG;
  constexpr int CPB = kStreamThreads / 32 * CPW;  // channels per CTA
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ng = lane % NG;
  const int b = blockIdx.y;
  const int c_raw = blockIdx.x * CPB + warp * CPW + lane / NG;
  const bool active = c_raw < p.D;
  const int c = active ? c_raw : 0;
  const int T_ = p.T, D = p.D, N = p.N;

  const T* __restrict__ gdelta = static_cast<const T*>(p.delta);
  const T* __restrict__ gs = static_cast<const T*>(p.s);
  const T* __restrict__ gB = static_cast<const T*>(p.Bm);
  const T* __restrict__ gC = static_cast<const T*>(p.Cm);
  const T* __restrict__ gq = static_cast<const T*>(p.q);

  float4 h[G];
  LamConst lc[G];
  bool nok[G];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    nok[i] = active && n < N;
    h[i] = f4_zero();
    lc[i] = LamConst{0.f, 0.f, 0.f, 0.f, 0.f};
    if (nok[i]) {
      if (p.h0 != nullptr) h[i] = QIO<float>::ld(p.h0 + ((int64_t(b) * D + c) * N + n) * 4);
      if (!Q_GIVEN) lc[i] = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n) * 4));
    }
  }
  const bool d_const = p.dst == 0;
  const float dsk0 = active ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(c) * p.dsd) : 0.f;

  // per-step strides (elements) and this lane's offsets
  const int64_t row_stride = int64_t(D);                   // [B,T,D]
  const int64_t q_stride = int64_t(D) * N * 4;             // [B,T,D,N,4] per step
  const int64_t row0 = int64_t(b) * T_ * D + c;            // (b, 0, c)
  const int64_t e0 = (int64_t(b) * T_ * D + c) * N * 4 + int64_t(ng) * 4;  // (b, 0, c, ng)
  const int64_t bc_stride = BC_SHARED ? int64_t(N) * 4 : q_stride;
  const int64_t bc0 = BC_SHARED ? int64_t(b) * T_ * N * 4 + int64_t(ng) * 4 : e0;
  float4 P[STATE_ONLY ? G : 1];
#pragma unroll
  for (int i = 0; i < (STATE_ONLY ? G : 1); ++i) P[i] = make_float4(1.f, 0.f, 0.f, 0.f);

  struct Step {
    float dl;
    float4 sv;
    float4 Bv[G], Cv[G], qv[G];
  };
  auto load_step = [&](int t, Step& s) {
    const int64_t row = row0 + int64_t(t) * row_stride;
    const int64_t e = e0 + int64_t(t) * q_stride;
    const int64_t ebc = bc0 + int64_t(t) * bc_stride;
    s.dl = (!Q_GIVEN && active) ? to_f(gdelta[row]) : 0.f;
    s.sv = f4_zero();
    if (active) {
      if (S_REAL) s.sv.x = to_f(gs[row]);
      else s.sv = QIO<T>::ld(gs + row * 4);
    }
#pragma unroll
    for (int i = 0; i < G; ++i) {
      s.Bv[i] = s.Cv[i] = f4_zero();
      s.qv[i] = make_float4(1.f, 0.f, 0.f, 0.f);
      if (nok[i]) {
        if (BC_SHARED) {
          s.Bv[i] = QIO<T>::ld(gB + ebc + NG * i * 4);
          if (!STATE_ONLY) s.Cv[i] = QIO<T>::ld(gC + ebc + NG * i * 4);
        } else {
          s.Bv[i] = QIO<T>::ld_stream(gB + ebc + NG * i * 4);
          if (!STATE_ONLY) s.Cv[i] = QIO<T>::ld_stream(gC + ebc + NG * i * 4);
        }
        if (Q_GIVEN) s.qv[i] = QIO<T>::ld_stream(gq + e + NG * i * 4);
      }
    }
  };

  Step cur, nxt;
  load_step(0, cur);
  const float eps = p.eps;
  T* yb = static_cast<T*>(p.y) + (int64_t(b) * T_ * D + c) * 4;
  // two states per lane with the Cayley map formed here: run them as one packed
  // pair (n0, n1) through two-lane FP32 instructions, with the rounding and order
  // of the scalar formulas below (packed_math.cuh), so the results are the same
  if constexpr (G == 2 && !Q_GIVEN && !STATE_ONLY) {
    const pk::LamPair lp{make_float2(lc[0].lr, lc[1].lr), make_float2(lc[0].li, lc[1].li),
                         make_float2(lc[0].lj, lc[1].lj), make_float2(lc[0].lk, lc[1].lk),
                         make_float2(lc[0].m, lc[1].m)};
    pk::QPair hq = pk::qp_from(h[0], h[1]);
    // B and C of the next step are held as loaded (bf16: 8 bytes a quaternion)
    // and unpacked straight into the pair registers when used
    using Raw = typename std::conditional<sizeof(T) == 2, uint2, float4>::type;
    struct RStep {
      float dl;
      float4 sv;
      Raw B[2], C[2];
    };
    auto ld_raw = [&](const T* ptr) -> Raw {
      if constexpr (sizeof(T) == 2) return __ldcs(reinterpret_cast<const uint2*>(ptr));
      else return __ldcs(reinterpret_cast<const float4*>(ptr));
    };
    auto load_raw = [&](int t, RStep& s) {
      const int64_t row = row0 + int64_t(t) * row_stride;
      const int64_t ebc = bc0 + int64_t(t) * bc_stride;
      s.dl = active ? to_f(gdelta[row]) : 0.f;
      s.sv = f4_zero();
      if (active) {
        if (S_REAL) s.sv.x = to_f(gs[row]);
        else s.sv = QIO<T>::ld(gs + row * 4);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        s.B[i] = s.C[i] = Raw{};
        if (nok[i]) {
          s.B[i] = ld_raw(gB + ebc + NG * i * 4);
          s.C[i] = ld_raw(gC + ebc + NG * i * 4);
        }
      }
    };
    auto to_pair = [&](const Raw& a, const Raw& b) -> pk::QPair {
      if constexpr (sizeof(T) == 2) {
        return pk::QPair{make_float2(__uint_as_float(a.x << 16), __uint_as_float(b.x << 16)),
                         make_float2(__uint_as_float(a.x & 0xffff0000u),
                                     __uint_as_float(b.x & 0xffff0000u)),
                         make_float2(__uint_as_float(a.y << 16), __uint_as_float(b.y << 16)),
                         make_float2(__uint_as_float(a.y & 0xffff0000u),
                                     __uint_as_float(b.y & 0xffff0000u))};
      } else {
        return pk::qp_from(a, b);
      }
    };
    RStep rc, rn;
    load_raw(0, rc);
    for (int t = 0; t < T_; ++t) {
      if (t + 1 < T_) load_raw(t + 1, rn);
      const float dl = rc.dl;
      const float4 sv = rc.sv;
      const pk::QPair qv = pk::cayley_pair(dl, dl * dl, lp, eps);
      const pk::QPair Bq = to_pair(rc.B[0], rc.B[1]);
      pk::QPair inj;
      if (S_REAL) {
        const float2 s2 = pk::bc2(sv.x);
        inj = pk::QPair{pk::mul2(s2, Bq.x), pk::mul2(s2, Bq.y), pk::mul2(s2, Bq.z),
                        pk::mul2(s2, Bq.w)};
      } else {
        inj = pk::qp_mul_bcast(Bq, sv);
      }
      hq = pk::qp_mul_acc(qv, hq, inj);
      const pk::QPair y2 = pk::qp_mul_acc(to_pair(rc.C[0], rc.C[1]), hq, pk::qp_zero());
      const float4 ya =
          make_float4(y2.x.x + y2.x.y, y2.y.x + y2.y.y, y2.z.x + y2.z.y, y2.w.x + y2.w.y);
      float dsk = dsk0;
      if (!d_const)
        dsk = (active && ng < 4)
                  ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst + int64_t(c) * p.dsd)
                  : 0.f;
      reduce_store_y<T, NG>(ya, sv, dsk, ng, active, yb + int64_t(t) * D * 4);
      if (p.ckpt != nullptr && active && (t + 1) % p.ckpt_every == 0 && t + 1 < T_) {
        const float4 hh[2] = {pk::qp_half(hq, 0), pk::qp_half(hq, 1)};
        store_ckpt<G, NG>(p, b, c, ng, (t + 1) / p.ckpt_every - 1, hh);
      }
      rc = rn;
    }
    h[0] = pk::qp_half(hq, 0);
    h[1] = pk::qp_half(hq, 1);
  } else
  for (int t = 0; t < T_; ++t) {
    if (t + 1 < T_) load_step(t + 1, nxt);
    const float dl = cur.dl, dl2 = dl * dl;
    const float4 sv = cur.sv;
    float4 ya = f4_zero(), yb2 = f4_zero();
#pragma unroll
    for (int i = 0; i < G; ++i) {
      float4 qv;
      if (Q_GIVEN) qv = cur.qv[i];
      else qv = cayley_from_const(dl, dl2, lc[i], eps);
      const float4 Bv = cur.Bv[i];
      float4 inj;
      if (S_REAL) inj = make_float4(sv.x * Bv.x, sv.x * Bv.y, sv.x * Bv.z, sv.x * Bv.w);
      else inj = qmul(Bv, sv);
      h[i] = qmul_acc(qv, h[i], inj);
      if constexpr (STATE_ONLY) {
        P[i] = qmul(qv, P[i]);
      } else {
        if (i & 1) yb2 = qmul_acc(cur.Cv[i], h[i], yb2);
        else ya = qmul_acc(cur.Cv[i], h[i], ya);
      }
    }
    if constexpr (STATE_ONLY) {
      cur = nxt;
      continue;
    }
    ya.x += yb2.x;
    ya.y += yb2.y;
    ya.z += yb2.z;
    ya.w += yb2.w;
    float dsk = dsk0;
    if (!d_const)
      dsk = (active && ng < 4)
                ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst + int64_t(c) * p.dsd)
                : 0.f;
    reduce_store_y<T, NG>(ya, sv, dsk, ng, active, yb + int64_t(t) * D * 4);
    if (p.ckpt != nullptr && active && (t + 1) % p.ckpt_every == 0 && t + 1 < T_)
      store_ckpt<G, NG>(p, b, c, ng, (t + 1) / p.ckpt_every - 1, h);
    cur = nxt;
  }

  if (p.hT != nullptr) {
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      if (nok[i]) QIO<float>::st(p.hT + ((int64_t(b) * D + c) * N + n) * 4, h[i]);
    }
  }
  if constexpr (STATE_ONLY) {
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      if (nok[i]) QIO<float>::st(p.pout + ((int64_t(b) * D + c) * N + n) * 4, P[i]);
    }
  }
}

template <typename T, int G, int NG, bool S_REAL, bool Q_GIVEN, bool BC_SHARED, bool STATE_ONLY>
int launch_stream(const FwdParams& p, cudaStream_t st) {
  constexpr int CPB = kStreamThreads / 32 * (32 / NG);
  dim3 grid{unsigned((p.D + CPB - 1) / CPB), unsigned(p.B), 1u};
  scan_fwd_stream_kernel<T, G, NG, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>
      <<<grid, kStreamThreads, 0, st>>>(p);
  return check_launch("mqc_ssm_scan_fwd(stream)");
}

template <typename T, bool S_REAL, bool Q_GIVEN, bool BC_SHARED, bool STATE_ONLY>
int dispatch_stream_t(const FwdParams& p, cudaStream_t st) {
  // G = 2 states per lane up to N = 64 (NG = next power of two of N/2), then G = 4 / 8
  if (p.N <= 64) {
    const int need = (p.N + 1) / 2;
    int ng = 1;
    while (ng < need) ng <<= 1;
    switch (ng) {
      case 1: return launch_stream<T, 2, 1, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
      case 2: return launch_stream<T, 2, 2, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
      case 4: return launch_stream<T, 2, 4, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
      case 8: return launch_stream<T, 2, 8, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
      case 16: return launch_stream<T, 2, 16, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
      default: return launch_stream<T, 2, 32, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
    }
  }
  if (p.N <= 128) return launch_stream<T, 4, 32, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
  return launch_stream<T, 8, 32, S_REAL, Q_GIVEN, BC_SHARED, STATE_ONLY>(p, st);
}

int dispatch_stream(const FwdParams& p, int dtype, bool s_real, bool q_given, cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32) {
    if (q_given)
      return s_real ? dispatch_stream_t<float, true, true, false, false>(p, st)
                    : dispatch_stream_t<float, false, true, false, false>(p, st);
    return s_real ? dispatch_stream_t<float, true, false, false, false>(p, st)
                  : dispatch_stream_t<float, false, false, false, false>(p, st);
  }
  if (q_given)
    return s_real ? dispatch_stream_t<__nv_bfloat16, true, true, false, false>(p, st)
                  : dispatch_stream_t<__nv_bfloat16, false, true, false, false>(p, st);
  return s_real ? dispatch_stream_t<__nv_bfloat16, true, false, false, false>(p, st)
                : dispatch_stream_t<__nv_bfloat16, false, false, false, false>(p, st);
}

int dispatch_stream_shared(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32)
    return s_real ? dispatch_stream_t<float, true, false, true, false>(p, st)
                  : dispatch_stream_t<float, false, false, true, false>(p, st);
  return s_real ? dispatch_stream_t<__nv_bfloat16, true, false, true, false>(p, st)
                : dispatch_stream_t<__nv_bfloat16, false, false, true, false>(p, st);
}

int dispatch_state_only(const FwdParams& p, int dtype, bool s_real, bool bc_shared,
                        cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32) {
    if (bc_shared)
      return s_real ? dispatch_stream_t<float, true, false, true, true>(p, st)
                    : dispatch_stream_t<float, false, false, true, true>(p, st);
    return s_real ? dispatch_stream_t<float, true, false, false, true>(p, st)
                  : dispatch_stream_t<float, false, false, false, true>(p, st);
  }
  if (bc_shared)
    return s_real ? dispatch_stream_t<__nv_bfloat16, true, false, true, true>(p, st)
                  : dispatch_stream_t<__nv_bfloat16, false, false, true, true>(p, st);
  return s_real ? dispatch_stream_t<__nv_bfloat16, true, false, false, true>(p, st)
                : dispatch_stream_t<__nv_bfloat16, false, false, false, true>(p, st);
}

}  // namespace scan
}  // namespace mqc
