// Backward of the fused Cayley + quaternion selective scan (sm_100a).
//
// The reference has no GPU backward (its Triton kernels carry no autograd); the
// gradients here are those torch autograd takes through the reference's CPU
// composition, QuaternionMamba2Block._ssm_forward lines 214-228
// (mambaqc/models/quaternion_mamba2_block.py) with cayley_discretization_reference
// (mambaqc/kernels/cayley_transform.py:199-223) and the ssm_step_reference loop
// (mambaqc/kernels/ssm_fused.py:363-379, 405-430).
//
// Lane layout as in the forward: a lane owns G states n = ng + NG*i of one
// channel, NG lanes cover the channel's N states. Time is walked backwards in
// sub-blocks of K = MQC_SSM_CKPT_EVERY steps. For each sub-block the lane
//   1. reloads the state before the sub-block (forward checkpoint, h0 or zero),
//   2. recomputes the K states forward into its slots of a per-warp shared
//      buffer (only the lane itself reads them back),
//   3. runs the adjoint recursion backwards over the K steps.
// Per-(t, channel) results (ddelta, dS) are summed over the NG lanes with
// shuffles; dLambda accumulates in registers over t; channel-shared dB/dC are
// summed over the CTA's channels in a shared-memory tile with shared atomics,
// then added to global fp32 accumulators with vector atomics once per sub-block.
#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {

constexpr int kSub = MQC_SSM_CKPT_EVERY;
// Warps per CTA: the recomputed-state buffer is kSub * G * 32 lanes * 16 B per
// warp, so the CTA shrinks as G grows (G=2: 8 warps, 64 KiB; G=8: 2 warps).
__host__ __device__ constexpr int bwd_warps(int g) { return 16 / g; }

struct BwdParams {
  int B, T, D, N;
  float eps;
  const void* delta;
  const float* lam;
  const void* Bm;
  const void* Cm;
  const void* s;
  const float* dskip;
  int64_t dsb, dst, dsd;
  const float* h0;
  const float* ckpt;
  const void* dy;
  const float* dhT;
  void* ddelta;
  float* dlam_part;
  void* dB;
  void* dC;
  void* ds;
  float* dh0;
  int nck;
  int cpb;  // channels per CTA
};

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

__device__ __forceinline__ float4 axpy4(float a, float4 x, float4 y) {
  return make_float4(fmaf(a, x.x, y.x), fmaf(a, x.y, y.y), fmaf(a, x.z, y.z), fmaf(a, x.w, y.w));
}

// Sum of v over the NG lanes of a channel (butterfly; every lane gets the total).
template <int NG>
__device__ __forceinline__ float lane_sum(float v) {
#pragma unroll
  for (int m = 1; m < NG; m <<= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

template <typename T, int G, int NG, bool BC_SHARED, bool S_REAL>
__global__ void __launch_bounds__(32 * bwd_warps(G))
    ssm_scan_bwd_kernel(const BwdParams p) {
  constexpr int kBwdWarps = bwd_warps(G);
  constexpr int CPW = 32 / NG;
  constexpr int NP = NG * G;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // per warp: [kSub][G][32 lanes] float4 recomputed states; then (shared B/C)
  // the dB/dC tile [kSub][NP][8] floats
  float4* hs_all = reinterpret_cast<float4*>(smem_raw);
  float* acc = reinterpret_cast<float*>(smem_raw + size_t(kBwdWarps) * kSub * G * 32 * 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = lane % NG;
  const int cl = warp * CPW + lane / NG;
  const int b = blockIdx.y;
  const int c_raw = blockIdx.x * p.cpb + cl;
  const bool active = cl < p.cpb && c_raw < p.D;
  const int c = active ? c_raw : 0;
  const int T_ = p.T, D = p.D, N = p.N;
  float4* hs = hs_all + size_t(warp) * kSub * G * 32;

  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  const T* gB = static_cast<const T*>(p.Bm);
  const T* gC = static_cast<const T*>(p.Cm);
  const T* gdy = static_cast<const T*>(p.dy);

  LamConst lc[G];
  float4 lamq[G];   // Lambda as a quaternion (for z = delta * Lambda)
  float4 carry[G];  // conj(q_{t+1}) (x) lambda_{t+1}
  float4 dlam[G];
  float4 hstart[G];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    lamq[i] = f4_zero();
    carry[i] = f4_zero();
    dlam[i] = f4_zero();
    lc[i] = LamConst{0.f, 0.f, 0.f, 0.f, 0.f};
    if (active && n < N) {
      lamq[i] = QIO<float>::ld(p.lam + (int64_t(c) * N + n) * 4);
      lc[i] = make_lam_const(lamq[i]);
      if (p.dhT != nullptr) carry[i] = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n) * 4);
    }
  }

  auto bc_index = [&](int t, int n) -> int64_t {  // element offset of B/C at (b, t, c, n)
    if (BC_SHARED) return ((int64_t(b) * T_ + t) * N + n) * 4;
    return (((int64_t(b) * T_ + t) * D + c) * N + n) * 4;
  };
  auto load_s = [&](int t) -> float4 {
    if (!active) return f4_zero();
    const int64_t row = (int64_t(b) * T_ + t) * D + c;
    if (S_REAL) return make_float4(to_f(gs[row]), 0.f, 0.f, 0.f);
    return QIO<T>::ld(gs + row * 4);
  };

  const int nsub = (T_ + kSub - 1) / kSub;
  for (int sb = nsub - 1; sb >= 0; --sb) {
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    // ---- state before the sub-block
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      hstart[i] = f4_zero();
      if (active && n < N) {
        if (sb > 0)
          hstart[i] = QIO<float>::ld(p.ckpt + ((int64_t(b) * p.nck + (sb - 1)) * D + c) * int64_t(N) * 4 +
                                     int64_t(n) * 4);
        else if (p.h0 != nullptr)
          hstart[i] = QIO<float>::ld(p.h0 + ((int64_t(b) * D + c) * N + n) * 4);
      }
    }
    // ---- recompute the sub-block's states forward
    {
      float4 h[G];
#pragma unroll
      for (int i = 0; i < G; ++i) h[i] = hstart[i];
      for (int tt = 0; tt < len; ++tt) {
        const int t = t0 + tt;
        const float dl = active ? to_f(gdelta[(int64_t(b) * T_ + t) * D + c]) : 0.f;
        const float dl2 = dl * dl;
        const float4 sv = load_s(t);
#pragma unroll
        for (int i = 0; i < G; ++i) {
          const int n = ng + NG * i;
          float4 Bv = f4_zero();
          if (active && n < N) Bv = QIO<T>::ld(gB + bc_index(t, n));
          const float4 qv = cayley_from_const(dl, dl2, lc[i], p.eps);
          float4 inj;
          if (S_REAL) inj = make_float4(sv.x * Bv.x, sv.x * Bv.y, sv.x * Bv.z, sv.x * Bv.w);
          else inj = qmul(Bv, sv);
          h[i] = qmul_acc(qv, h[i], inj);
          hs[(tt * G + i) * 32 + lane] = h[i];
        }
      }
    }
    if (BC_SHARED) {
      // zero this sub-block's dB/dC tile
      for (int e = threadIdx.x; e < kSub * NP * 8; e += blockDim.x) acc[e] = 0.f;
      __syncthreads();
    }
    // ---- adjoint, backwards over the sub-block
    for (int tt = len - 1; tt >= 0; --tt) {
      const int t = t0 + tt;
      const int64_t row = (int64_t(b) * T_ + t) * D + c;
      const float dl = active ? to_f(gdelta[row]) : 0.f;
      const float dl2 = dl * dl;
      const float4 sv = load_s(t);
      const float4 gy = active ? QIO<T>::ld(gdy + row * 4) : f4_zero();
      float pd = 0.f;        // sum_n <dz, Lambda>
      float4 psum = f4_zero();  // sum_n conj(B) (x) lambda (x component only for a real S)
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const int n = ng + NG * i;
        const bool ok = active && n < N;
        float4 Bv = f4_zero(), Cv = f4_zero();
        if (ok) {
          Bv = QIO<T>::ld(gB + bc_index(t, n));
          Cv = QIO<T>::ld(gC + bc_index(t, n));
        }
        const float4 hcur = hs[(tt * G + i) * 32 + lane];
        const float4 hprev = tt > 0 ? hs[((tt - 1) * G + i) * 32 + lane] : hstart[i];
        // lambda_t = conj(C_t) (x) dy_t + conj(q_{t+1}) (x) lambda_{t+1}
        const float4 lam = qmul_acc(qconj(Cv), gy, carry[i]);
        const float4 qv = cayley_from_const(dl, dl2, lc[i], p.eps);
        const float4 dq = qmul(lam, qconj(hprev));
        const float4 z = make_float4(dl * lamq[i].x, dl * lamq[i].y, dl * lamq[i].z, dl * lamq[i].w);
        const float4 dz = cayley_vjp(z, dq, p.eps);
        pd = fmaf(1.f, dot4(dz, lamq[i]), pd);
        dlam[i] = axpy4(dl, dz, dlam[i]);
        float4 dBv, dCv;
        if (S_REAL) {
          dBv = make_float4(sv.x * lam.x, sv.x * lam.y, sv.x * lam.z, sv.x * lam.w);
          psum.x += dot4(Bv, lam);
        } else {
          dBv = qmul(lam, qconj(sv));
          psum = qmul_acc(qconj(Bv), lam, psum);
        }
        dCv = qmul(gy, qconj(hcur));
        if (ok) {
          if (BC_SHARED) {
            float* slot = acc + (tt * NP + n) * 8;
            atomicAdd(slot + 0, dBv.x);
            atomicAdd(slot + 1, dBv.y);
            atomicAdd(slot + 2, dBv.z);
            atomicAdd(slot + 3, dBv.w);
            atomicAdd(slot + 4, dCv.x);
            atomicAdd(slot + 5, dCv.y);
            atomicAdd(slot + 6, dCv.z);
            atomicAdd(slot + 7, dCv.w);
          } else {
            QIO<T>::st(static_cast<T*>(p.dB) + bc_index(t, n), dBv);
            QIO<T>::st(static_cast<T*>(p.dC) + bc_index(t, n), dCv);
          }
        }
        carry[i] = qmul(qconj(qv), lam);
      }
      // per-(t, channel) sums over the NG lanes of the channel
      pd = lane_sum<NG>(pd);
      psum.x = lane_sum<NG>(psum.x);
      if (!S_REAL) {
        psum.y = lane_sum<NG>(psum.y);
        psum.z = lane_sum<NG>(psum.z);
        psum.w = lane_sum<NG>(psum.w);
      }
      if (active && ng == 0) {
        const float dsk = __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst + int64_t(c) * p.dsd);
        QIO<T>::st1(static_cast<T*>(p.ddelta) + row, pd);
        if (S_REAL) {
          QIO<T>::st1(static_cast<T*>(p.ds) + row, fmaf(dsk, gy.x, psum.x));
        } else {
          QIO<T>::st(static_cast<T*>(p.ds) + row * 4, axpy4(dsk, gy, psum));
        }
      }
    }
    if (BC_SHARED) {
      __syncthreads();
      float* dB = static_cast<float*>(p.dB);
      float* dC = static_cast<float*>(p.dC);
      for (int e = threadIdx.x; e < len * N * 2; e += blockDim.x) {
        const int which = e & 1, tn = e >> 1;
        const int tt = tn / N, n = tn % N;
        const float* slot = acc + (tt * NP + n) * 8 + which * 4;
        const float4 v = make_float4(slot[0], slot[1], slot[2], slot[3]);
        float* dst = (which ? dC : dB) + ((int64_t(b) * T_ + t0 + tt) * N + n) * 4;
        atomicAdd(reinterpret_cast<float4*>(dst), v);
      }
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    if (active && n < N) {
      const int64_t off = ((int64_t(b) * D + c) * N + n) * 4;
      QIO<float>::st(p.dlam_part + off, dlam[i]);
      if (p.dh0 != nullptr) QIO<float>::st(p.dh0 + off, carry[i]);  // conj(q_0) (x) lambda_0
    }
  }
}

template <typename T, int G, int NG, bool BC_SHARED, bool S_REAL>
int launch_bwd(BwdParams p, cudaStream_t st) {
  constexpr int kBwdWarps = bwd_warps(G);
  constexpr int CPW = 32 / NG;
  p.cpb = kBwdWarps * CPW;
  const size_t smem = size_t(kBwdWarps) * kSub * G * 32 * 16 +
                      (BC_SHARED ? size_t(kSub) * NG * G * 8 * sizeof(float) : 0);
  auto kern = ssm_scan_bwd_kernel<T, G, NG, BC_SHARED, S_REAL>;
  if (smem > 48 * 1024) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_ssm_scan_bwd: smem attribute: %s", cudaGetErrorString(e));
  }
  dim3 grid{unsigned((p.D + p.cpb - 1) / p.cpb), unsigned(p.B), 1u};
  kern<<<grid, 32 * kBwdWarps, smem, st>>>(p);
  return check_launch("mqc_ssm_scan_bwd");
}

template <typename T, bool BC_SHARED, bool S_REAL>
int dispatch_bwd_ng(const BwdParams& p, cudaStream_t st) {
  // G = 2 states per lane up to N = 64 (NG <= 32), then G = 4 / 8
  if (p.N <= 64) {
    const int need = (p.N + 1) / 2;
    int ng = 1;
    while (ng < need) ng <<= 1;
    switch (ng) {
      case 1: return launch_bwd<T, 2, 1, BC_SHARED, S_REAL>(p, st);
      case 2: return launch_bwd<T, 2, 2, BC_SHARED, S_REAL>(p, st);
      case 4: return launch_bwd<T, 2, 4, BC_SHARED, S_REAL>(p, st);
      case 8: return launch_bwd<T, 2, 8, BC_SHARED, S_REAL>(p, st);
      case 16: return launch_bwd<T, 2, 16, BC_SHARED, S_REAL>(p, st);
      default: return launch_bwd<T, 2, 32, BC_SHARED, S_REAL>(p, st);
    }
  }
  if (p.N <= 128) return launch_bwd<T, 4, 32, BC_SHARED, S_REAL>(p, st);
  return launch_bwd<T, 8, 32, BC_SHARED, S_REAL>(p, st);
}

template <typename T>
int dispatch_bwd(const BwdParams& p, int flags, cudaStream_t st) {
  const bool sh = flags & MQC_SSM_BC_SHARED;
  const bool sr = flags & MQC_SSM_S_REAL;
  if (sh) return sr ? dispatch_bwd_ng<T, true, true>(p, st) : dispatch_bwd_ng<T, true, false>(p, st);
  return sr ? dispatch_bwd_ng<T, false, true>(p, st) : dispatch_bwd_ng<T, false, false>(p, st);
}

}  // namespace scan
}  // namespace mqc

using namespace mqc;
using namespace mqc::scan;

extern "C" int mqc_ssm_scan_bwd(const mqc_ssm_scan_bwd_args* a, void* stream) {
  clear_error();
  const char* name = "mqc_ssm_scan_bwd";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(dtype_ok(a->dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, a->dtype);
  MQC_REQUIRE((a->flags & ~(MQC_SSM_BC_SHARED | MQC_SSM_S_REAL)) == 0, MQC_ERR_INVALID_VALUE,
              "%s: unsupported flags 0x%x (explicit q has no backward here)", name, a->flags);
  MQC_REQUIRE(a->batch >= 0 && a->seq_len >= 0 && a->channels >= 0 && a->d_state >= 0,
              MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(a->batch <= 65535 && a->seq_len < (1ll << 31) && a->channels < (1ll << 31),
              MQC_ERR_UNSUPPORTED, "%s: size out of range", name);
  MQC_REQUIRE(a->d_state <= 256, MQC_ERR_UNSUPPORTED, "%s: d_state > 256", name);
  if (a->batch == 0 || a->seq_len == 0 || a->channels == 0) return MQC_OK;
  MQC_REQUIRE(a->d_state >= 1, MQC_ERR_INVALID_VALUE, "%s: d_state must be >= 1", name);
  MQC_REQUIRE(a->ckpt_every == MQC_SSM_CKPT_EVERY, MQC_ERR_UNSUPPORTED, "%s: ckpt_every must be %d",
              name, MQC_SSM_CKPT_EVERY);
  const int64_t nck = (a->seq_len + a->ckpt_every - 1) / a->ckpt_every - 1;
  MQC_REQUIRE(a->delta && a->lambda_ && a->Bm && a->Cm && a->s && a->dskip && a->dy && a->ddelta &&
                  a->dlambda_part && a->dBm && a->dCm && a->ds && (nck == 0 || a->ckpt),
              MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  const uintptr_t qa = a->dtype == MQC_DTYPE_F32 ? 16 : 8;
  const bool sh = a->flags & MQC_SSM_BC_SHARED;
  const bool sr = a->flags & MQC_SSM_S_REAL;
  MQC_REQUIRE(aligned(a->dy, qa) && (sr || (aligned(a->s, qa) && aligned(a->ds, qa))) &&
                  aligned(a->lambda_, 16) && aligned(a->dlambda_part, 16) &&
                  (a->ckpt == nullptr || aligned(a->ckpt, 16)) &&
                  (a->h0 == nullptr || aligned(a->h0, 16)) &&
                  (a->dhT == nullptr || aligned(a->dhT, 16)) &&
                  (a->dh0 == nullptr || aligned(a->dh0, 16)),
              MQC_ERR_MISALIGNED, "%s: misaligned tensor", name);
  if (sh) {
    MQC_REQUIRE(aligned(a->Bm, qa) && aligned(a->Cm, qa) && aligned(a->dBm, 16) &&
                    aligned(a->dCm, 16),
                MQC_ERR_MISALIGNED, "%s: misaligned B/C or dB/dC", name);
  } else {
    MQC_REQUIRE(aligned(a->Bm, qa) && aligned(a->Cm, qa) && aligned(a->dBm, qa) &&
                    aligned(a->dCm, qa),
                MQC_ERR_MISALIGNED, "%s: misaligned B/C or dB/dC", name);
  }
  BwdParams p{};
  p.B = int(a->batch);
  p.T = int(a->seq_len);
  p.D = int(a->channels);
  p.N = int(a->d_state);
  p.eps = a->eps;
  p.delta = a->delta;
  p.lam = a->lambda_;
  p.Bm = a->Bm;
  p.Cm = a->Cm;
  p.s = a->s;
  p.dskip = a->dskip;
  p.dsb = a->dskip_sb;
  p.dst = a->dskip_st;
  p.dsd = a->dskip_sd;
  p.h0 = a->h0;
  p.ckpt = a->ckpt;
  p.dy = a->dy;
  p.dhT = a->dhT;
  p.ddelta = a->ddelta;
  p.dlam_part = a->dlambda_part;
  p.dB = a->dBm;
  p.dC = a->dCm;
  p.ds = a->ds;
  p.dh0 = a->dh0;
  p.nck = int(nck);
  if (a->dtype == MQC_DTYPE_F32) return dispatch_bwd<float>(p, a->flags, as_stream(stream));
  return dispatch_bwd<__nv_bfloat16>(p, a->flags, as_stream(stream));
}
