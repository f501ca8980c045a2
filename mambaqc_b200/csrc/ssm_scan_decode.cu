// One decode step of the fused Cayley + quaternion scan (seq_len 1, channel-
// shared B/C): the block's recurrent `step` / `generate(use_cache=True)` path,
// h <- q (x) h + B (x) S and y = sum_n C (x) h + D S with the fp32 state cache
// updated in place (mambaqc/kernels/ssm_fused.py:258-337 is the reference's
// single step, with q formed here from delta and Lambda as in
// models/quaternion_mamba2_block.py:214-228).
//
// The step is bound by the state cache, read and written once: 32 bytes per
// (b, d, n) state. The per-(d, n) Cayley constants (Lambda, 16 bytes per state)
// are shared by every batch row, so a warp owns CPW channels for kRows batch
// rows: it loads Lambda once, then issues the loads of all its rows' states
// and B/C up front (no dependency between rows), so each warp keeps
// kRows x 32 lanes x 96 bytes in flight, and computes the rows in turn.
#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {
namespace {

constexpr int kDecWarps = 4;
constexpr int kRows = 4;  // batch rows per warp

template <typename T, int NG, bool S_REAL>
__global__ void __launch_bounds__(32 * kDecWarps) scan_decode_kernel(const FwdParams p) {
  constexpr int CPW = 32 / NG;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ng = lane % NG;
  const int c_raw = (blockIdx.x * kDecWarps + warp) * CPW + lane / NG;
  const bool active = c_raw < p.D;
  const int c = active ? c_raw : 0;
  const int b0 = blockIdx.y * kRows;
  const int D = p.D, N = p.N;
  const int n0 = ng, n1 = ng + NG;
  const bool ok0 = active && n0 < N, ok1 = active && n1 < N;

  LamConst l0{0.f, 0.f, 0.f, 0.f, 0.f}, l1{0.f, 0.f, 0.f, 0.f, 0.f};
  if (ok0) l0 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n0) * 4));
  if (ok1) l1 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n1) * 4));

  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  const T* gB = static_cast<const T*>(p.Bm);
  const T* gC = static_cast<const T*>(p.Cm);
  // all rows' operands first: every load of the warp is in flight at once
  float4 h[kRows][2], Bv[kRows][2], Cv[kRows][2], sv[kRows];
  float dl[kRows], dsk[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int b = b0 + r;
    const bool rv = b < p.B;
    h[r][0] = h[r][1] = Bv[r][0] = Bv[r][1] = Cv[r][0] = Cv[r][1] = sv[r] = f4_zero();
    dl[r] = dsk[r] = 0.f;
    if (rv) {
      const int64_t hs = (int64_t(b) * D + c) * N;
      if (p.h0 != nullptr) {
        if (ok0) h[r][0] = QIO<float>::ld(p.h0 + (hs + n0) * 4);
        if (ok1) h[r][1] = QIO<float>::ld(p.h0 + (hs + n1) * 4);
      }
      const int64_t bc = int64_t(b) * N;
      if (ok0) {
        Bv[r][0] = QIO<T>::ld(gB + (bc + n0) * 4);
        Cv[r][0] = QIO<T>::ld(gC + (bc + n0) * 4);
      }
      if (ok1) {
        Bv[r][1] = QIO<T>::ld(gB + (bc + n1) * 4);
        Cv[r][1] = QIO<T>::ld(gC + (bc + n1) * 4);
      }
      if (active) {
        const int64_t row = int64_t(b) * D + c;
        dl[r] = to_f(gdelta[row]);
        if (S_REAL) sv[r].x = to_f(gs[row]);
        else sv[r] = QIO<T>::ld(gs + row * 4);
        dsk[r] = __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(c) * p.dsd);
      }
    }
  }
  const float eps = p.eps;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int b = b0 + r;
    if (b >= p.B) break;  // uniform over the CTA
    const float d2 = dl[r] * dl[r];
    float4 hn[2];
    // one readout accumulator per state of the pair, summed at the end: the
    // streaming kernel's order, so a step equals a one-step scan bit for bit
    float4 ya = f4_zero(), yb = f4_zero();
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float4 qv = cayley_from_const(dl[r], d2, e ? l1 : l0, eps);
      float4 inj;
      if (S_REAL)
        inj = make_float4(sv[r].x * Bv[r][e].x, sv[r].x * Bv[r][e].y, sv[r].x * Bv[r][e].z,
                          sv[r].x * Bv[r][e].w);
      else
        inj = qmul(Bv[r][e], sv[r]);
      hn[e] = qmul_acc(qv, h[r][e], inj);
      if (e) yb = qmul_acc(Cv[r][e], hn[e], yb);
      else ya = qmul_acc(Cv[r][e], hn[e], ya);
    }
    ya.x += yb.x;
    ya.y += yb.y;
    ya.z += yb.z;
    ya.w += yb.w;
    reduce_store_y<T, NG>(ya, sv[r], dsk[r], ng, active, static_cast<T*>(p.y) +
                                                            (int64_t(b) * D + c) * 4);
    const int64_t hs = (int64_t(b) * D + c) * N;
    if (ok0) QIO<float>::st(p.hT + (hs + n0) * 4, hn[0]);
    if (ok1) QIO<float>::st(p.hT + (hs + n1) * 4, hn[1]);
  }
}

template <typename T, int NG, bool S_REAL>
int launch_decode(const FwdParams& p, cudaStream_t st) {
  constexpr int CPB = kDecWarps * (32 / NG);
  dim3 grid{unsigned((p.D + CPB - 1) / CPB), unsigned((p.B + kRows - 1) / kRows), 1u};
  scan_decode_kernel<T, NG, S_REAL><<<grid, 32 * kDecWarps, 0, st>>>(p);
  return check_launch("mqc_ssm_scan_fwd(decode)");
}

template <typename T, bool S_REAL>
int dispatch_decode_t(const FwdParams& p, cudaStream_t st) {
  const int need = (p.N + 1) / 2;
  int ng = 1;
  while (ng < need) ng <<= 1;
  switch (ng) {
    case 1: return launch_decode<T, 1, S_REAL>(p, st);
    case 2: return launch_decode<T, 2, S_REAL>(p, st);
    case 4: return launch_decode<T, 4, S_REAL>(p, st);
    case 8: return launch_decode<T, 8, S_REAL>(p, st);
    case 16: return launch_decode<T, 16, S_REAL>(p, st);
    default: return launch_decode<T, 32, S_REAL>(p, st);
  }
}

}  // namespace

// Up to 32 batch rows: measured at config-3 channel and state sizes, this
// kernel takes 4.0 / 13.2 us per step at 4 / 16 rows against 4.4 / 13.8 us on
// the streaming kernel, and 63.5 / 250 us at 64 / 256 rows against 62 / 242 us
// (there the state stream, not Lambda, limits both).
bool decode_serves(const FwdParams& p) {
  return p.T == 1 && p.B <= 32 && p.N <= 64 && p.hT != nullptr && p.ckpt == nullptr &&
         p.pout == nullptr;
}

int dispatch_decode(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32)
    return s_real ? dispatch_decode_t<float, true>(p, st) : dispatch_decode_t<float, false>(p, st);
  return s_real ? dispatch_decode_t<__nv_bfloat16, true>(p, st)
                : dispatch_decode_t<__nv_bfloat16, false>(p, st);
}

}  // namespace scan
}  // namespace mqc
