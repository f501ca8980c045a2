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
// shuffles; dLambda accumulates in registers over t; channel-shared dB/dC go to
// a per-warp shared-memory slice, the slices are summed over the CTA's warps in a
// fixed order at the end of each sub-block, and the CTA's sum is added to global
// fp32 accumulators with one vector atomic per (t, n, tensor).
#include <cstdlib>
#include <type_traits>

#include "packed_math.cuh"
#include "ssm_scan_bwd_common.cuh"

namespace mqc {
namespace scan {

// Double-buffered shared-memory stage of one sub-block's inputs (fp32,
// channel-shared B/C): B and C rows [kSub][2][N] float4, delta and x (or S) and
// dy of the CTA's channels [kSub][cpb], and the lanes' start states
// [warps][G][32] float4. Filled with cp.async one sub-block ahead.
struct StageLayout {
  size_t bc, dl, sx, gy, hst, bytes;
};

__host__ __device__ inline StageLayout stage_layout(int N, int cpb, int warps, int G, bool s_real) {
  StageLayout L;
  size_t off = 0;
  L.bc = off;
  off += size_t(kSub) * 2 * N * 16;
  L.dl = off;
  off = align_up(off + size_t(kSub) * cpb * 4, 16);
  L.sx = off;
  off = align_up(off + size_t(kSub) * cpb * (s_real ? 4 : 16), 16);
  L.gy = off;
  off += size_t(kSub) * cpb * 16;
  L.hst = off;
  off += size_t(warps) * G * 32 * 16;
  L.bytes = off;
  return L;
}

template <typename T, int G, int NG, bool BC_SHARED, bool S_REAL, bool STAGE>
__global__ void __launch_bounds__(32 * bwd_warps(G, BC_SHARED))
    ssm_scan_bwd_kernel(const BwdParams p) {
  constexpr int kBwdWarps = bwd_warps(G, BC_SHARED);
  constexpr int CPW = 32 / NG;
  constexpr int NP = NG * G;
  // fp32 with channel-shared B/C (when the stage fits): inputs staged in shared
  // memory by cp.async
  constexpr bool STAGED = STAGE && BC_SHARED && std::is_same<T, float>::value;
  constexpr bool HS_REG = G == 2;      // recomputed states in registers (else shared)
  constexpr int NV = S_REAL ? 2 : 8;   // per-(t, channel) sums: ddelta, dS (padded)
  constexpr int V = kSub * NV;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // [per warp: kSub x G x 32 lanes float4 states, when not in registers]
  // [per warp: private dB/dC slice kSub x 2 x NP float4, for channel-shared B/C]
  const size_t hs_bytes = HS_REG ? 0 : size_t(kBwdWarps) * kSub * G * 32 * 16;
  float4* hs_all = reinterpret_cast<float4*>(smem_raw);
  float4* slices = reinterpret_cast<float4*>(smem_raw + hs_bytes);
  const size_t slice_bytes = BC_SHARED ? size_t(kBwdWarps) * kSub * 2 * NP * 16 : 0;
  const StageLayout SL = stage_layout(p.N, p.cpb, kBwdWarps, G, S_REAL);
  unsigned char* stage_base = smem_raw + hs_bytes + slice_bytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = lane % NG;
  const int cl = warp * CPW + lane / NG;
  const int b = blockIdx.y;
  const int c_raw = blockIdx.x * p.cpb + cl;
  const bool active = cl < p.cpb && c_raw < p.D;
  const int c = active ? c_raw : 0;
  const int T_ = p.T, D = p.D, N = p.N;
  float4* hs_smem = hs_all + size_t(warp) * kSub * G * 32;
  float4* slice = slices + size_t(warp) * kSub * 2 * NP;

  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  const T* gB = static_cast<const T*>(p.Bm);
  const T* gC = static_cast<const T*>(p.Cm);
  const T* gdy = static_cast<const T*>(p.dy);

  LamConst lc[G];
  float4 carry[G];  // conj(q_{t+1}) (x) lambda_{t+1}
  float4 dlam[G];
  float4 hstart[G];
  bool nok[G];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    nok[i] = active && n < N;
    carry[i] = f4_zero();
    dlam[i] = f4_zero();
    lc[i] = LamConst{0.f, 0.f, 0.f, 0.f, 0.f};
    if (nok[i]) {
      lc[i] = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n) * 4));
      if (p.dhT != nullptr) carry[i] = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n) * 4);
    }
  }
  const float eps = p.eps;
  const int64_t bc_row = BC_SHARED ? int64_t(N) * 4 : int64_t(D) * N * 4;  // per-step stride
  const int64_t bc_lane = BC_SHARED ? int64_t(ng) * 4 : (int64_t(c) * N + ng) * 4;
  float4 hsr[HS_REG ? kSub : 1][G];

  // issue the cp.async copies of sub-block `sb`'s inputs into stage buffer `buf`
  auto issue_stage = [&](int sb, int buf) {
    unsigned char* st = stage_base + size_t(buf) * SL.bytes;
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    const float* fB = reinterpret_cast<const float*>(gB);
    const float* fC = reinterpret_cast<const float*>(gC);
    float4* sbc = reinterpret_cast<float4*>(st + SL.bc);
    for (int e = threadIdx.x; e < len * 2 * N; e += blockDim.x) {
      const int tt = e / (2 * N), r = e % (2 * N), which = r / N, n = r % N;
      const float* src = (which ? fC : fB) + ((int64_t(b) * T_ + t0 + tt) * N + n) * 4;
      cp_async16(sbc + (tt * 2 + which) * N + n, src, true);
    }
    float* sdl = reinterpret_cast<float*>(st + SL.dl);
    float* ssx = reinterpret_cast<float*>(st + SL.sx);
    float4* sgy = reinterpret_cast<float4*>(st + SL.gy);
    const float* fdelta = reinterpret_cast<const float*>(gdelta);
    const float* fs = reinterpret_cast<const float*>(gs);
    const float* fdy = reinterpret_cast<const float*>(gdy);
    for (int e = threadIdx.x; e < len * p.cpb; e += blockDim.x) {
      const int tt = e / p.cpb, cc = e % p.cpb;
      const int ch = blockIdx.x * p.cpb + cc;
      const bool v = ch < D;
      const int64_t row = v ? (int64_t(b) * T_ + t0 + tt) * D + ch : 0;
      cp_async4(sdl + e, fdelta + row, v);
      if (S_REAL) cp_async4(ssx + e, fs + row, v);
      else cp_async16(reinterpret_cast<float4*>(ssx) + e, fs + row * 4, v);
      cp_async16(sgy + e, fdy + row * 4, v);
    }
    float4* shst = reinterpret_cast<float4*>(st + SL.hst);
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      const bool from_ckpt = sb > 0;
      const bool v = nok[i] && (from_ckpt || p.h0 != nullptr);
      const float* src = p.ckpt;
      if (v) {
        src = from_ckpt ? p.ckpt + ((int64_t(b) * p.nck + (sb - 1)) * D + c) * int64_t(N) * 4 +
                              int64_t(n) * 4
                        : p.h0 + ((int64_t(b) * D + c) * N + n) * 4;
      }
      cp_async16(shst + (warp * G + i) * 32 + lane, v ? src : p.lam, v);
    }
    cp_async_commit();
  };

  const int nsub = (T_ + kSub - 1) / kSub;
  if constexpr (STAGED) {
    issue_stage(nsub - 1, 0);
    cp_async_wait_all();
    __syncthreads();
  }
  for (int sb = nsub - 1; sb >= 0; --sb) {
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    const int64_t row0 = (int64_t(b) * T_ + t0) * D + c;  // (b, t0, c) in [B,T,D]
    const T* B0 = gB + (int64_t(b) * T_ + t0) * bc_row + bc_lane;
    const T* C0 = gC + (int64_t(b) * T_ + t0) * bc_row + bc_lane;
    const int buf = (nsub - 1 - sb) & 1;
    const unsigned char* stg = stage_base + size_t(buf) * SL.bytes;
    const float4* sbc = reinterpret_cast<const float4*>(stg + SL.bc) + ng;
    const float* sdl = reinterpret_cast<const float*>(stg + SL.dl) + cl;
    const float* ssx = reinterpret_cast<const float*>(stg + SL.sx);
    const float4* sgy = reinterpret_cast<const float4*>(stg + SL.gy) + cl;
    if constexpr (STAGED) {
      if (sb > 0) issue_stage(sb - 1, buf ^ 1);
    }
    // inputs of step tt of this sub-block (staged or straight from global)
    auto in_delta = [&](int tt) -> float {
      if constexpr (STAGED) return sdl[tt * p.cpb];
      else return active ? to_f(gdelta[row0 + int64_t(tt) * D]) : 0.f;
    };
    auto in_s = [&](int tt) -> float4 {
      if constexpr (STAGED) {
        if (S_REAL) return make_float4(ssx[tt * p.cpb + cl], 0.f, 0.f, 0.f);
        return reinterpret_cast<const float4*>(ssx)[tt * p.cpb + cl];
      } else {
        if (!active) return f4_zero();
        const int64_t row = row0 + int64_t(tt) * D;
        if (S_REAL) return make_float4(to_f(gs[row]), 0.f, 0.f, 0.f);
        return QIO<T>::ld(gs + row * 4);
      }
    };
    auto in_dy = [&](int tt) -> float4 {
      if constexpr (STAGED) return sgy[tt * p.cpb];
      else return active ? QIO<T>::ld(gdy + (row0 + int64_t(tt) * D) * 4) : f4_zero();
    };
    auto in_bc = [&](int tt, int i, int which) -> float4 {
      if constexpr (STAGED) return sbc[(tt * 2 + which) * N + NG * i];
      else return QIO<T>::ld((which ? C0 : B0) + tt * bc_row + NG * i * 4);
    };
    // ---- state before the sub-block
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      hstart[i] = f4_zero();
      if constexpr (STAGED) {
        hstart[i] = reinterpret_cast<const float4*>(stg + SL.hst)[(warp * G + i) * 32 + lane];
      } else if (nok[i]) {
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
#pragma unroll
      for (int tt = 0; tt < kSub; ++tt) {
        if (tt < len) {
          const float dl = in_delta(tt);
          const float dl2 = dl * dl;
          const float4 sv = in_s(tt);
#pragma unroll
          for (int i = 0; i < G; ++i) {
            const float4 Bv = nok[i] ? in_bc(tt, i, 0) : f4_zero();
            const float4 qv = cayley_from_const(dl, dl2, lc[i], eps);
            float4 inj;
            if (S_REAL) inj = make_float4(sv.x * Bv.x, sv.x * Bv.y, sv.x * Bv.z, sv.x * Bv.w);
            else inj = qmul(Bv, sv);
            h[i] = qmul_acc(qv, h[i], inj);
            if constexpr (HS_REG) hsr[tt][i] = h[i];
            else hs_smem[(tt * G + i) * 32 + lane] = h[i];
          }
        }
      }
    }
    // ---- adjoint, backwards over the sub-block
    float part[V];  // per (tt, k): k = 0 ddelta, k >= 1 dS components; summed over n later
#pragma unroll
    for (int e = 0; e < V; ++e) part[e] = 0.f;
#pragma unroll
    for (int tt = kSub - 1; tt >= 0; --tt) {
      if (tt < len) {
        const int t = t0 + tt;
        const float dl = in_delta(tt);
        const float dl2 = dl * dl;
        const float4 sv = in_s(tt);
        const float4 gy = in_dy(tt);
        float pd = 0.f;
        float4 psum = f4_zero();
        if (ng == 0 && active) {  // skip term D * dy, counted once per channel
          const float dsk = __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst +
                                  int64_t(c) * p.dsd);
          psum = make_float4(dsk * gy.x, dsk * gy.y, dsk * gy.z, dsk * gy.w);
        }
#pragma unroll
        for (int i = 0; i < G; ++i) {
          float4 Bv = f4_zero(), Cv = f4_zero();
          if (nok[i]) {
            Bv = in_bc(tt, i, 0);
            Cv = in_bc(tt, i, 1);
          }
          float4 hcur, hprev;
          if constexpr (HS_REG) {
            hcur = hsr[tt][i];
            hprev = tt > 0 ? hsr[tt > 0 ? tt - 1 : 0][i] : hstart[i];
          } else {
            hcur = hs_smem[(tt * G + i) * 32 + lane];
            hprev = tt > 0 ? hs_smem[((tt > 0 ? tt - 1 : 0) * G + i) * 32 + lane] : hstart[i];
          }
          // lambda_t = conj(C_t) (x) dy_t + conj(q_{t+1}) (x) lambda_{t+1}
          const float4 lam = qmul_acc(qconj(Cv), gy, carry[i]);
          const float4 qv = cayley_from_const(dl, dl2, lc[i], eps);
          const float4 dq = qmul(lam, qconj(hprev));
          const float4 lq = make_float4(lc[i].lr, lc[i].li, lc[i].lj, lc[i].lk);
          const float4 z = make_float4(dl * lq.x, dl * lq.y, dl * lq.z, dl * lq.w);
          const float4 dz = cayley_vjp(z, dq, eps);
          pd += dot4(dz, lq);
          dlam[i] = axpy4(dl, dz, dlam[i]);
          float4 dBv;
          if (S_REAL) {
            dBv = make_float4(sv.x * lam.x, sv.x * lam.y, sv.x * lam.z, sv.x * lam.w);
            psum.x += dot4(Bv, lam);
          } else {
            dBv = qmul(lam, qconj(sv));
            psum = qmul_acc(qconj(Bv), lam, psum);
          }
          float4 dCv = qmul(gy, qconj(hcur));
          if (BC_SHARED) {
            if (!nok[i]) {
              dBv = f4_zero();
              dCv = f4_zero();
            }
            // sum over the CPW channels this warp holds (lanes ng + NG*k share n)
#pragma unroll
            for (int m = NG; m < 32; m <<= 1) {
              dBv.x += __shfl_xor_sync(0xffffffffu, dBv.x, m);
              dBv.y += __shfl_xor_sync(0xffffffffu, dBv.y, m);
              dBv.z += __shfl_xor_sync(0xffffffffu, dBv.z, m);
              dBv.w += __shfl_xor_sync(0xffffffffu, dBv.w, m);
              dCv.x += __shfl_xor_sync(0xffffffffu, dCv.x, m);
              dCv.y += __shfl_xor_sync(0xffffffffu, dCv.y, m);
              dCv.z += __shfl_xor_sync(0xffffffffu, dCv.z, m);
              dCv.w += __shfl_xor_sync(0xffffffffu, dCv.w, m);
            }
            // the warp's first channel lanes write every (tt, n < NP) slot, so the
            // slice needs no clearing; consecutive n per lane: conflict-free
            if (lane < NG) {
              const int n = ng + NG * i;
              slice[(tt * 2 + 0) * NP + n] = dBv;
              slice[(tt * 2 + 1) * NP + n] = dCv;
            }
          } else if (nok[i]) {
            T* dBp = static_cast<T*>(p.dB) + (B0 - gB) + tt * bc_row + NG * i * 4;
            T* dCp = static_cast<T*>(p.dC) + (C0 - gC) + tt * bc_row + NG * i * 4;
            QIO<T>::st(dBp, dBv);
            QIO<T>::st(dCp, dCv);
          }
          carry[i] = qmul(qconj(qv), lam);
        }
        part[tt * NV + 0] = pd;
        part[tt * NV + 1] = psum.x;
        if (!S_REAL) {
          part[tt * NV + 2] = psum.y;
          part[tt * NV + 3] = psum.z;
          part[tt * NV + 4] = psum.w;
        }
      }
    }
    // ---- per-(t, channel) sums over the NG lanes of the channel, then stores
    {
      const int base = reduce_scatter<V, NG>(part, ng);
      constexpr int W = (V / NG) > 0 ? (V / NG) : 1;
      constexpr int kLogV = (V >= 64) ? 6 : (V >= 32 ? 5 : (V >= 16 ? 4 : (V >= 8 ? 3 : 1)));
      const bool writer = active && (NG <= V || (ng >> kLogV) == 0);
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int idx = base + j;
        const int tt = idx / NV, k = idx % NV;
        if (writer && tt < len) {
          const int64_t row = row0 + int64_t(tt) * D;
          if (k == 0) {
            QIO<T>::st1(static_cast<T*>(p.ddelta) + row, part[j]);
          } else if (S_REAL) {
            QIO<T>::st1(static_cast<T*>(p.ds) + row, part[j]);
          } else if (k <= 4) {
            QIO<T>::st1(static_cast<T*>(p.ds) + row * 4 + (k - 1), part[j]);
          }
        }
      }
    }
    if (BC_SHARED) {
      // sum the warps' slices (fixed order) and add the CTA's share to global
      __syncthreads();
      float* dB = static_cast<float*>(p.dB);
      float* dC = static_cast<float*>(p.dC);
      for (int e = threadIdx.x; e < len * 2 * N; e += blockDim.x) {
        const int n = e % N, tw = e / N;  // tw = tt * 2 + which
        float4 v = slices[tw * NP + n];
        for (int w = 1; w < kBwdWarps; ++w) {
          const float4 u = slices[size_t(w) * kSub * 2 * NP + tw * NP + n];
          v.x += u.x;
          v.y += u.y;
          v.z += u.z;
          v.w += u.w;
        }
        const int tt = tw >> 1;
        float* dst = ((tw & 1) ? dC : dB) + ((int64_t(b) * T_ + t0 + tt) * N + n) * 4;
        atomicAdd(reinterpret_cast<float4*>(dst), v);
      }
    }
    if constexpr (STAGED) cp_async_wait_all();
    if (BC_SHARED) __syncthreads();  // slices free; next stage (if any) visible
  }

#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    if (nok[i]) {
      const int64_t off = ((int64_t(b) * D + c) * N + n) * 4;
      QIO<float>::st(p.dlam_part + off, dlam[i]);
      if (p.dh0 != nullptr) QIO<float>::st(p.dh0 + off, carry[i]);  // conj(q_0) (x) lambda_0
    }
  }
}

// ---------------------------------------------------------------------------
// Packed backward: channel-shared B/C with d_state <= 2*NG, G = 2 states per lane
// forming one pair (ng, ng + NG), on packed two-lane FP32 (packed_math.cuh).
// Same algorithm as ssm_scan_bwd_kernel:
//  * B/C come from the pair-interleaved pre-pass (pack_bc_pairs), whose rows
//    keep the two 16-byte parts of a pair NG*16 bytes apart, so a warp's loads
//    are contiguous;
//  * delta, x (or S) and dy are fp32 (bf16 inputs widened first);
//  * all inputs of a sub-block are staged one sub-block ahead with cp.async;
//  * the per-warp dB/dC slices are pair-interleaved, stored component-major
//    ([t][tensor][component][pair] float2: contiguous 8-byte stores across the
//    lanes), and are un-interleaved only
//    in the per-CTA summation.
constexpr int kPbWarps = 8;

struct PbLayout {
  size_t slices, bc, dl, sx, gy, hst, stage, total;
};

// [slices: warps x kSub x 2 tensors x 4 components x NG pairs x 2 f32] then 2 stages of
// [bc: kSub x 2 x NG x 8 f32 | dl: kSub x cpb f32 | sx: kSub x cpb x sw f32 |
//  gy: kSub x cpb x 4 f32 | hst: warps x 32 lanes x 8 f32]; stage offsets are
// relative to the stage.
__host__ __device__ inline PbLayout pb_layout(int NG, int cpb, bool s_real) {
  PbLayout L;
  L.slices = size_t(kPbWarps) * kSub * 2 * NG * 32;
  L.bc = 0;
  size_t o = size_t(kSub) * 2 * NG * 32;
  L.dl = o;
  o = align_up(o + size_t(kSub) * cpb * 4, 16);
  L.sx = o;
  o = align_up(o + size_t(kSub) * cpb * (s_real ? 4 : 16), 16);
  L.gy = o;
  o += size_t(kSub) * cpb * 16;
  L.hst = o;
  o += size_t(kPbWarps) * 32 * 32;
  L.stage = o;
  L.total = L.slices + 2 * o;
  return L;
}

template <typename T, int NG, bool S_REAL>
__global__ void __launch_bounds__(32 * kPbWarps)
    ssm_scan_bwd_packed_kernel(const BwdParams p, const float* __restrict__ Bp,
                               const float* __restrict__ Cp, const float* __restrict__ dlf,
                               const float* __restrict__ sf, const float* __restrict__ dyf) {
  using namespace ::mqc::pk;
  constexpr int CPW = 32 / NG;
  constexpr int NV = S_REAL ? 2 : 8;  // per-(t, channel) sums: ddelta, dS (padded)
  constexpr int V = kSub * NV;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int cpb = p.cpb;
  const PbLayout L = pb_layout(NG, cpb, S_REAL);
  float* slices = reinterpret_cast<float*>(smem_raw);
  unsigned char* stage_base = smem_raw + L.slices;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = lane % NG;
  const int cl = warp * CPW + lane / NG;
  const int b = blockIdx.y;
  const int c_raw = blockIdx.x * cpb + cl;
  const bool active = cl < cpb && c_raw < p.D;
  const int c = active ? c_raw : 0;
  const int T_ = p.T, D = p.D, N = p.N;
  const int n0 = ng, n1 = ng + NG;
  const bool ok0 = active && n0 < N, ok1 = active && n1 < N;
  float* slice = slices + size_t(warp) * kSub * 2 * NG * 8;

  LamPair lc;
  QPair carry, dlam = qp_zero();
  {
    LamConst k0{0.f, 0.f, 0.f, 0.f, 0.f}, k1{0.f, 0.f, 0.f, 0.f, 0.f};
    float4 c0 = f4_zero(), c1 = f4_zero();
    if (ok0) {
      k0 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n0) * 4));
      if (p.dhT != nullptr) c0 = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n0) * 4);
    }
    if (ok1) {
      k1 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n1) * 4));
      if (p.dhT != nullptr) c1 = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n1) * 4);
    }
    lc = LamPair{make_float2(k0.lr, k1.lr), make_float2(k0.li, k1.li),
                 make_float2(k0.lj, k1.lj), make_float2(k0.lk, k1.lk), make_float2(k0.m, k1.m)};
    carry = qp_from(c0, c1);  // conj(q_{t+1}) (x) lambda_{t+1}
  }
  const QPair lq{lc.lr, lc.li, lc.lj, lc.lk};
  const float eps = p.eps;

  auto issue_stage = [&](int sb, int buf) {
    unsigned char* st = stage_base + size_t(buf) * L.stage;
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    float* sbc = reinterpret_cast<float*>(st + L.bc);
    // packed rows: per step and matrix NG pairs x 8 floats = 2*NG chunks of 16 B
    for (int e = threadIdx.x; e < len * 4 * NG; e += blockDim.x) {
      const int tt = e / (4 * NG), r = e % (4 * NG), which = r / (2 * NG), k = r % (2 * NG);
      const float* src = (which ? Cp : Bp) + (int64_t(b) * T_ + t0 + tt) * NG * 8 + k * 4;
      cp_async16(sbc + (tt * 2 + which) * NG * 8 + k * 4, src, true);
    }
    float* sdl = reinterpret_cast<float*>(st + L.dl);
    float* ssx = reinterpret_cast<float*>(st + L.sx);
    float* sgy = reinterpret_cast<float*>(st + L.gy);
    for (int e = threadIdx.x; e < len * cpb; e += blockDim.x) {
      const int tt = e / cpb, cc = e % cpb;
      const int ch = blockIdx.x * cpb + cc;
      const bool v = ch < D;
      const int64_t row = v ? (int64_t(b) * T_ + t0 + tt) * D + ch : 0;
      cp_async4(sdl + e, dlf + row, v);
      if (S_REAL) cp_async4(ssx + e, sf + row, v);
      else cp_async16(ssx + e * 4, sf + row * 4, v);
      cp_async16(sgy + e * 4, dyf + row * 4, v);
    }
    // the lane's two start states (checkpoint, h0 or zero), state-wise
    float* shst = reinterpret_cast<float*>(st + L.hst) + (warp * 32 + lane) * 8;
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int n = e2 ? n1 : n0;
      const bool ok = e2 ? ok1 : ok0;
      const bool v = ok && (sb > 0 || p.h0 != nullptr);
      const float* src = p.lam;
      if (v)
        src = sb > 0 ? p.ckpt + ((int64_t(b) * p.nck + (sb - 1)) * D + c) * int64_t(N) * 4 +
                           int64_t(n) * 4
                     : p.h0 + ((int64_t(b) * D + c) * N + n) * 4;
      cp_async16(shst + e2 * 4, src, v);
    }
    cp_async_commit();
  };

  const int nsub = (T_ + kSub - 1) / kSub;
  issue_stage(nsub - 1, 0);
  cp_async_wait_all();
  __syncthreads();
  for (int sb = nsub - 1; sb >= 0; --sb) {
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    const int64_t row0 = (int64_t(b) * T_ + t0) * D + c;  // (b, t0, c) in [B,T,D]
    const int buf = (nsub - 1 - sb) & 1;
    const unsigned char* stg = stage_base + size_t(buf) * L.stage;
    const float* sbc = reinterpret_cast<const float*>(stg + L.bc) + ng * 4;
    const float* sdl = reinterpret_cast<const float*>(stg + L.dl) + cl;
    const float* ssx = reinterpret_cast<const float*>(stg + L.sx);
    const float4* sgy = reinterpret_cast<const float4*>(stg + L.gy) + cl;
    if (sb > 0) issue_stage(sb - 1, buf ^ 1);
    auto ld_pair = [&](int tt, int which) -> QPair {
      const float* q = sbc + (tt * 2 + which) * NG * 8;
      const float4 u = *reinterpret_cast<const float4*>(q);
      const float4 w = *reinterpret_cast<const float4*>(q + NG * 4);
      return QPair{make_float2(u.x, u.y), make_float2(u.z, u.w), make_float2(w.x, w.y),
                   make_float2(w.z, w.w)};
    };
    auto in_s = [&](int tt) -> float4 {
      if (S_REAL) return make_float4(ssx[tt * cpb + cl], 0.f, 0.f, 0.f);
      return reinterpret_cast<const float4*>(ssx)[tt * cpb + cl];
    };
    const float* shst = reinterpret_cast<const float*>(stg + L.hst) + (warp * 32 + lane) * 8;
    const QPair hstart = qp_from(*reinterpret_cast<const float4*>(shst),
                                 *reinterpret_cast<const float4*>(shst + 4));
    // ---- recompute + adjoint of the sub-block; FULL (len == kSub, every
    // sub-block but possibly the last) compiles without per-step guards, so the
    // loop-carried values need no conditional merges
    float part[V];
    auto run_sub = [&](auto full_tag) {
    constexpr bool FULL = decltype(full_tag)::value;
    QPair hs[kSub];
    {
      QPair h = hstart;
#pragma unroll
      for (int tt = 0; tt < kSub; ++tt) {
        if (FULL || tt < len) {
          const float dl = sdl[tt * cpb];
          const float4 sv = in_s(tt);
          const QPair Bq = ld_pair(tt, 0);
          const QPair qv = cayley_pair(dl, dl * dl, lc, eps);
          QPair inj;
          if (S_REAL) {
            const float2 s2 = bc2(sv.x);
            inj = QPair{mul2(s2, Bq.x), mul2(s2, Bq.y), mul2(s2, Bq.z), mul2(s2, Bq.w)};
          } else {
            inj = qp_mul_bcast(Bq, sv);
          }
          h = qp_mul_acc(qv, h, inj);
        }
        hs[tt] = h;
      }
    }
    // ---- adjoint, backwards over the sub-block
#pragma unroll
    for (int e = 0; e < V; ++e) part[e] = 0.f;
#pragma unroll
    for (int tt = kSub - 1; tt >= 0; --tt) {
      if (FULL || tt < len) {
        const int t = t0 + tt;
        const float dl = sdl[tt * cpb];
        const float4 sv = in_s(tt);
        const float4 gy = sgy[tt * cpb];
        float4 psum = f4_zero();
        if (ng == 0 && active) {  // skip term D * dy, counted once per channel
          const float dsk = __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst +
                                  int64_t(c) * p.dsd);
          psum = make_float4(dsk * gy.x, dsk * gy.y, dsk * gy.z, dsk * gy.w);
        }
        const QPair Bq = ld_pair(tt, 0), Cq = ld_pair(tt, 1);
        const QPair hcur = hs[tt];
        const QPair hprev = tt > 0 ? hs[tt > 0 ? tt - 1 : 0] : hstart;
        // lambda_t = conj(C_t) (x) dy_t + conj(q_{t+1}) (x) lambda_{t+1}
        const QPair cg = qp_mul_bcast(qp_conj(Cq), gy);
        const QPair lam{add2(cg.x, carry.x), add2(cg.y, carry.y), add2(cg.z, carry.z),
                        add2(cg.w, carry.w)};
        float2 cinv, cden;
        const QPair qv = cayley_pair_keep(dl, dl * dl, lc, eps, &cinv, &cden);
        const QPair dq = qp_mul_acc(lam, qp_conj(hprev), qp_zero());
        const float2 d2 = bc2(dl);
        const QPair dz = cayley_vjp_pair_shared(dl, lc, cinv, cden, dq, eps);
        const float2 pdp = qp_dot(dz, lq);
        dlam = QPair{fma2(d2, dz.x, dlam.x), fma2(d2, dz.y, dlam.y), fma2(d2, dz.z, dlam.z),
                     fma2(d2, dz.w, dlam.w)};
        QPair dB;
        if (S_REAL) {
          const float2 s2 = bc2(sv.x);
          dB = QPair{mul2(s2, lam.x), mul2(s2, lam.y), mul2(s2, lam.z), mul2(s2, lam.w)};
          const float2 bl = qp_dot(Bq, lam);
          psum.x += bl.x + bl.y;
        } else {
          dB = qp_mul_bcast(lam, qconj(sv));
          const QPair pl = qp_mul_acc(qp_conj(Bq), lam, qp_zero());
          psum.x += pl.x.x + pl.x.y;
          psum.y += pl.y.x + pl.y.y;
          psum.z += pl.z.x + pl.z.y;
          psum.w += pl.w.x + pl.w.y;
        }
        QPair dC = qp_bmul(gy, qp_conj(hcur));
        // sum over the CPW channels of this warp (lanes ng + NG*k hold the same states)
#pragma unroll
        for (int m = NG; m < 32; m <<= 1) {
          float* fb = reinterpret_cast<float*>(&dB);
          float* fc = reinterpret_cast<float*>(&dC);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            fb[k] += __shfl_xor_sync(0xffffffffu, fb[k], m);
            fc[k] += __shfl_xor_sync(0xffffffffu, fc[k], m);
          }
        }
        // the warp's first channel lanes write every (tt, pair) slot, so the slice
        // needs no clearing
        if (lane < NG) {  // one 8-byte store per pair component: no register assembly
          float2* sbw = reinterpret_cast<float2*>(slice + (tt * 2) * NG * 8) + ng;
          sbw[0] = dB.x;
          sbw[NG] = dB.y;
          sbw[2 * NG] = dB.z;
          sbw[3 * NG] = dB.w;
          float2* scw = reinterpret_cast<float2*>(slice + (tt * 2 + 1) * NG * 8) + ng;
          scw[0] = dC.x;
          scw[NG] = dC.y;
          scw[2 * NG] = dC.z;
          scw[3 * NG] = dC.w;
        }
        carry = qp_mul_acc(qp_conj(qv), lam, qp_zero());
        part[tt * NV + 0] = pdp.x + pdp.y;
        part[tt * NV + 1] = psum.x;
        if (!S_REAL) {
          part[tt * NV + 2] = psum.y;
          part[tt * NV + 3] = psum.z;
          part[tt * NV + 4] = psum.w;
        }
      }
    }
    };
    if (len == kSub) run_sub(std::true_type{});
    else run_sub(std::false_type{});
    // ---- per-(t, channel) sums over the NG lanes of the channel, then stores
    {
      const int base = reduce_scatter<V, NG>(part, ng);
      constexpr int W = (V / NG) > 0 ? (V / NG) : 1;
      constexpr int kLogV = (V >= 64) ? 6 : (V >= 32 ? 5 : (V >= 16 ? 4 : (V >= 8 ? 3 : 1)));
      const bool writer = active && (NG <= V || (ng >> kLogV) == 0);
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int idx = base + j;
        const int tt = idx / NV, k = idx % NV;
        if (writer && tt < len) {
          const int64_t row = row0 + int64_t(tt) * D;
          if (k == 0) {
            QIO<T>::st1(static_cast<T*>(p.ddelta) + row, part[j]);
          } else if (S_REAL) {
            QIO<T>::st1(static_cast<T*>(p.ds) + row, part[j]);
          } else if (k <= 4) {
            QIO<T>::st1(static_cast<T*>(p.ds) + row * 4 + (k - 1), part[j]);
          }
        }
      }
    }
    // ---- sum the warps' slices (fixed order) and add the CTA's share to global
    __syncthreads();
    float* dBg = static_cast<float*>(p.dB);
    float* dCg = static_cast<float*>(p.dC);
    for (int e = threadIdx.x; e < len * 2 * NG; e += blockDim.x) {
      const int pg = e % NG, tw = e / NG;  // tw = tt * 2 + which
      const float2* p0 = reinterpret_cast<const float2*>(slices + size_t(tw) * NG * 8) + pg;
      float2 px = p0[0], py = p0[NG], pz = p0[2 * NG], pw = p0[3 * NG];
#pragma unroll
      for (int k = 1; k < kPbWarps; ++k) {
        const float2* pk2 = p0 + size_t(k) * kSub * 2 * NG * 4;
        px = add2(px, pk2[0]);
        py = add2(py, pk2[NG]);
        pz = add2(pz, pk2[2 * NG]);
        pw = add2(pw, pk2[3 * NG]);
      }
      const float4 u = make_float4(px.x, px.y, py.x, py.y);
      const float4 w = make_float4(pz.x, pz.y, pw.x, pw.y);
      // u = (x0, x1, y0, y1), w = (z0, z1, w0, w1): states pg and pg + NG
      float* dst = ((tw & 1) ? dCg : dBg) + (int64_t(b) * T_ + t0 + (tw >> 1)) * N * 4;
      if (pg < N) atomicAdd(reinterpret_cast<float4*>(dst + pg * 4), make_float4(u.x, u.z, w.x, w.z));
      if (pg + NG < N)
        atomicAdd(reinterpret_cast<float4*>(dst + (pg + NG) * 4), make_float4(u.y, u.w, w.y, w.w));
    }
    cp_async_wait_all();
    __syncthreads();  // slices free; next stage visible
  }

  if (ok0) {
    const int64_t off = ((int64_t(b) * D + c) * N + n0) * 4;
    QIO<float>::st(p.dlam_part + off, qp_half(dlam, 0));
    if (p.dh0 != nullptr) QIO<float>::st(p.dh0 + off, qp_half(carry, 0));
  }
  if (ok1) {
    const int64_t off = ((int64_t(b) * D + c) * N + n1) * 4;
    QIO<float>::st(p.dlam_part + off, qp_half(dlam, 1));
    if (p.dh0 != nullptr) QIO<float>::st(p.dh0 + off, qp_half(carry, 1));
  }
}

template <typename T, int NG, bool S_REAL>
int launch_bwd_packed(BwdParams p, cudaStream_t st) {
  constexpr int CPW = 32 / NG;
  constexpr int SW = S_REAL ? 1 : 4;
  p.cpb = kPbWarps * CPW;
  const PbLayout L = pb_layout(NG, p.cpb, S_REAL);
  if (L.total > size_t(kMaxBwdSmem))
    return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_bwd: packed staging does not fit");
  constexpr bool kWiden = !std::is_same<T, float>::value;
  const int64_t rows = int64_t(p.B) * p.T;
  const size_t plane = size_t(rows) * NG * 8 * sizeof(float);
  const int64_t n_delta = rows * p.D;
  const size_t bytes = 2 * plane + (kWiden ? size_t(n_delta) * (1 + SW + 4) * sizeof(float) : 0);
  float* ws = nullptr;
  cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&ws), bytes, st);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_ssm_scan_bwd: scratch allocation of %zu bytes: %s", bytes,
                cudaGetErrorString(e));
  float* Bp = ws;
  float* Cp = ws + plane / sizeof(float);
  const float* dlf = static_cast<const float*>(p.delta);
  const float* sf = static_cast<const float*>(p.s);
  const float* dyf = static_cast<const float*>(p.dy);
  int rc = pack_bc_pairs(p.Bm, p.Cm, Bp, Cp, rows, p.N, NG, 2,
                         kWiden ? MQC_DTYPE_BF16 : MQC_DTYPE_F32, st);
  if (kWiden && rc == MQC_OK) {
    float* w0 = Cp + plane / sizeof(float);
    float* w1 = w0 + n_delta;
    float* w2 = w1 + n_delta * SW;
    rc = widen_bf16_to_f32(p.delta, w0, n_delta, st);
    if (rc == MQC_OK) rc = widen_bf16_to_f32(p.s, w1, n_delta * SW, st);
    if (rc == MQC_OK) rc = widen_bf16_to_f32(p.dy, w2, n_delta * 4, st);
    dlf = w0;
    sf = w1;
    dyf = w2;
  }
  if (rc == MQC_OK) {
    auto kern = ssm_scan_bwd_packed_kernel<T, NG, S_REAL>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L.total));
    if (e != cudaSuccess) {
      rc = fail(MQC_ERR_CUDA, "mqc_ssm_scan_bwd: smem attribute (%zu B): %s", L.total,
                cudaGetErrorString(e));
    } else {
      dim3 grid{unsigned((p.D + p.cpb - 1) / p.cpb), unsigned(p.B), 1u};
      kern<<<grid, 32 * kPbWarps, L.total, st>>>(p, Bp, Cp, dlf, sf, dyf);
      rc = check_launch("mqc_ssm_scan_bwd(packed)");
    }
  }
  scratch_free(ws, st);
  return rc;
}

template <typename T, int G, int NG, bool BC_SHARED, bool S_REAL>
int launch_bwd(BwdParams p, cudaStream_t st) {
  constexpr int kBwdWarps = bwd_warps(G, BC_SHARED);
  constexpr int CPW = 32 / NG;
  p.cpb = kBwdWarps * CPW;
  const size_t base = (G == 2 ? 0 : size_t(kBwdWarps) * kSub * G * 32 * 16) +
                      (BC_SHARED ? size_t(kBwdWarps) * kSub * 2 * NG * G * 16 : 0);
  const size_t staged = base + 2 * stage_layout(p.N, p.cpb, kBwdWarps, G, S_REAL).bytes;
  const bool can_stage =
      BC_SHARED && std::is_same<T, float>::value && staged <= size_t(kMaxBwdSmem);
  const size_t smem = can_stage ? staged : base;
  auto kern = can_stage ? ssm_scan_bwd_kernel<T, G, NG, BC_SHARED, S_REAL, true>
                        : ssm_scan_bwd_kernel<T, G, NG, BC_SHARED, S_REAL, false>;
  if (smem > 48 * 1024) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_ssm_scan_bwd: smem attribute (%zu B): %s", smem,
                  cudaGetErrorString(e));
  }
  dim3 grid{unsigned((p.D + p.cpb - 1) / p.cpb), unsigned(p.B), 1u};
  kern<<<grid, 32 * kBwdWarps, smem, st>>>(p);
  return check_launch("mqc_ssm_scan_bwd");
}

// The packed kernels serve channel-shared B/C up to N = 64 and per-channel B/C
// with 16 < N <= 64 unless MQC_SCAN_IMPL selects another implementation (the
// unpacked kernel is then used).
inline bool use_packed_bwd() {
  static const bool packed = [] {
    const char* v = getenv("MQC_SCAN_IMPL");
    return v == nullptr || v[0] == '\0';
  }();
  return packed;
}

template <typename T, bool BC_SHARED, bool S_REAL>
int dispatch_bwd_ng(const BwdParams& p, cudaStream_t st) {
  // G = 2 states per lane up to N = 64 (NG <= 32), then G = 4 / 8
  if (p.N <= 64) {
    const int need = (p.N + 1) / 2;
    int ng = 1;
    while (ng < need) ng <<= 1;
    if (BC_SHARED && use_packed_bwd()) {
      switch (ng) {
        case 1: return launch_bwd_packed<T, 1, S_REAL>(p, st);
        case 2: return launch_bwd_packed<T, 2, S_REAL>(p, st);
        case 4: return launch_bwd_packed<T, 4, S_REAL>(p, st);
        case 8: return launch_bwd_packed<T, 8, S_REAL>(p, st);
        case 16: return launch_bwd_packed<T, 16, S_REAL>(p, st);
        default: return launch_bwd_packed<T, 32, S_REAL>(p, st);
      }
    }
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
  // per-channel B/C (the block's layout): the packed kernel with per-warp
  // cp.async staging, where its 16-byte row copies apply
  const int dtype = std::is_same<T, float>::value ? MQC_DTYPE_F32 : MQC_DTYPE_BF16;
  if (!sh && use_packed_bwd() && perchannel_bwd_serves(p.N, dtype) && aligned(p.Bm, 16) &&
      aligned(p.Cm, 16))
    return launch_bwd_perchannel(p, dtype, sr, st);
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
