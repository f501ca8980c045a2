// Backward of the fused Cayley + quaternion scan for per-channel B/C
// [B,T,D,N,4] -- the layout QuaternionMamba2Block._ssm_forward feeds the scan
// (mambaqc/models/quaternion_mamba2_block.py:186-191, B_proj/C_proj outputs
// viewed per channel) -- on packed two-lane FP32 (packed_math.cuh).
//
// Same algorithm and gradients as ssm_scan_bwd_kernel (ssm_scan_bwd.cu): time
// is walked backwards in sub-blocks of kSub = MQC_SSM_CKPT_EVERY steps; each
// sub-block recomputes its states from the forward's checkpoint and then runs
// the adjoint lambda_t = conj(C_t) (x) dy_t + conj(q_{t+1}) (x) lambda_{t+1}.
// This layout moves B, C, dB and dC (4 x B*T*D*N quaternions) through HBM once
// each and is bound by that traffic, so the kernel is built to keep HBM busy:
//  * every warp is independent and owns CPW = 32/NG whole channels of one batch
//    row; a lane holds the state pair (ng, ng + NG) of its channel;
//  * the B and C rows of a sub-block (contiguous per time step and channel
//    group) and its start states are staged into a per-warp, double-buffered
//    shared-memory stage with cp.async one sub-block ahead, so each warp always
//    has a sub-block of loads in flight and holds no staging registers;
//  * the per-(t, channel) inputs delta, x (or S), dy and the skip weight of the
//    next sub-block are fetched one per lane and broadcast with shuffles;
//  * dB and dC are the lane's own pairs and go straight to global memory (no
//    reduction, no atomics);
//  * all state arithmetic is packed (fma/mul/add .rn.f32x2): a bf16 quaternion
//    unpacks directly into the pair registers, so no register shuffling is
//    needed to form the pairs.
// No CTA-wide barrier is used: a warp waits only on its own copies
// (cp.async.wait_group, a hardware wait with no polling loop) and __syncwarp.
#include <type_traits>

#include "packed_math.cuh"
#include "ssm_scan_bwd_common.cuh"

namespace mqc {
namespace scan {
namespace {

template <typename T, int NG>
struct PcGeom {
  static constexpr int CPW = 32 / NG;                     // channels per warp
  static constexpr int NP = 2 * NG;                       // padded states per channel
  static constexpr int ROW = CPW * NP * 4;                // smem row stride, elements of T
  static constexpr int BC_BYTES = kSub * 2 * ROW * int(sizeof(T));
  static constexpr int HST_BYTES = CPW * NP * 16;         // start states, fp32
  // per-(t, channel) items, 48 bytes each: [0,4) the 32-bit word holding delta,
  // [4,8) the skip weight, [8,12) the word holding a real x, [16,32) a
  // quaternion S, [32,48) dy (bf16 quaternions use the first 8 bytes)
  static constexpr int ITEM_BYTES = 48;
  static constexpr int ITEMS_BYTES = kSub * CPW * ITEM_BYTES;
  static constexpr int STAGE_BYTES = BC_BYTES + HST_BYTES + ITEMS_BYTES;
  static constexpr int EPC = 16 / int(sizeof(T));         // elements per 16-byte chunk
  // 16-byte chunks of one (t, matrix) row of the warp's channels, at most
  static constexpr int MAX_CHUNKS = CPW * NP * 4 * int(sizeof(T)) / 16;
  static constexpr int J = (MAX_CHUNKS + 31) / 32;         // chunks per lane per row
  static_assert(STAGE_BYTES % 16 == 0, "stage alignment");
};

// The aligned 32-bit word holding element *e (cp.async moves 4, 8 or 16 bytes,
// so a bf16 scalar is fetched together with its neighbour), and which half of
// the word holds it.
template <typename T>
__device__ __forceinline__ const void* word_of(const T* e) {
  return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(e) & ~uintptr_t(3));
}
template <typename T>
__device__ __forceinline__ int half_of(const T* e) {
  return int((reinterpret_cast<uintptr_t>(e) >> 1) & 1);
}
template <typename T>
__device__ __forceinline__ float word_value(uint32_t w, int half) {
  if constexpr (std::is_same<T, float>::value) {
    (void)half;
    return __uint_as_float(w);
  } else {
    return __uint_as_float(half ? (w & 0xffff0000u) : (w << 16));
  }
}
// Shared-memory loads issued in program order (ld.volatile.shared) from a
// 32-bit shared address plus a compile-time byte offset. In order, because the
// straight-line sub-block code would otherwise let the compiler hoist the loads
// of later steps, each holding registers until its step runs; with an
// immediate offset, because every step's operands sit at fixed offsets from a
// per-lane base, so no address arithmetic is issued per load.
template <int OFF>
__device__ __forceinline__ uint32_t ldsi_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ float4 ldsi_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4+%5];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a), "n"(OFF));
  return v;
}
// One quaternion in the storage type.
template <typename T, int OFF>
__device__ __forceinline__ float4 ldsi_q(uint32_t a) {
  if constexpr (std::is_same<T, float>::value) {
    return ldsi_f4<OFF>(a);
  } else {
    uint32_t x, y;
    asm volatile("ld.volatile.shared.v2.u32 {%0, %1}, [%2+%3];"
                 : "=r"(x), "=r"(y)
                 : "r"(a), "n"(OFF));
    return QIO<__nv_bfloat16>::unpack(make_uint2(x, y));
  }
}

// f(std::integral_constant<int, I>) for I = B, B+1, ..., E-1 (unrolled at compile time)
template <int B, int E, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (B < E) {
    f(std::integral_constant<int, B>{});
    static_for<B + 1, E>(f);
  }
}
// f(std::integral_constant<int, I>) for I = B, B-1, ..., E
template <int B, int E, typename F>
__device__ __forceinline__ void static_for_down(F&& f) {
  if constexpr (B >= E) {
    f(std::integral_constant<int, B>{});
    static_for_down<B - 1, E>(f);
  }
}

// One quaternion (16 bytes fp32, 8 bytes bf16), global -> shared.
template <typename T>
__device__ __forceinline__ void cp_async_q(void* dst, const T* src) {
  if constexpr (std::is_same<T, float>::value) {
    cp_async16(dst, src, true);
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
  }
}

// fp32 stages are twice as large, so their CTAs have fewer warps to keep three
// CTAs per SM.
template <typename T>
constexpr int pc_warps() {
  return std::is_same<T, float>::value ? 2 : 4;
}
// Three resident CTAs per SM (12 warps for bf16, 6 for fp32, whose larger stages
// fill the shared memory first): at most 168 registers per thread.
template <typename T>
constexpr int pc_min_ctas() {
  return 3;
}

// EXACT: N == 2 * NG and every warp has CPW channels, so no lane is padding and
// no state guard is compiled.
template <typename T, int NG, bool S_REAL, bool EXACT>
__global__ void __launch_bounds__(32 * pc_warps<T>(), pc_min_ctas<T>())
    ssm_scan_bwd_pc_kernel(const BwdParams p) {
  using namespace ::mqc::pk;
  using G = PcGeom<T, NG>;
  constexpr int CPW = G::CPW, NP = G::NP, ROW = G::ROW, EPC = G::EPC, J = G::J;
  constexpr int WARPS = pc_warps<T>();
  extern __shared__ __align__(16) unsigned char smem_raw[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = lane % NG, chl = lane / NG;
  const int b = blockIdx.y;
  const int c0 = (blockIdx.x * WARPS + warp) * CPW;  // first channel of this warp
  if (c0 >= p.D) return;                             // warp-uniform; no CTA barriers follow
  const int T_ = p.T, D = p.D, N = p.N;
  const int nch = EXACT ? CPW : min(CPW, D - c0);
  const bool active = EXACT || chl < nch;
  const int c = active ? c0 + chl : c0;
  const int n0 = ng, n1 = ng + NG;
  const bool ok0 = EXACT || (active && n0 < N), ok1 = EXACT || (active && n1 < N);
  unsigned char* wbase = smem_raw + size_t(warp) * 2 * G::STAGE_BYTES;

  // Zero the padding of both stages once (states N..NP of every channel slot and
  // the slots of absent channels); the copies never write there, so padded
  // lanes read zeros and contribute nothing to the per-channel sums.
  if (!EXACT && (N < NP || nch < CPW)) {
    for (int st = 0; st < 2; ++st) {
      T* sbc = reinterpret_cast<T*>(wbase + size_t(st) * G::STAGE_BYTES);
      float* shs = reinterpret_cast<float*>(wbase + size_t(st) * G::STAGE_BYTES + G::BC_BYTES);
      for (int e = lane; e < kSub * 2 * CPW * NP; e += 32) {
        const int slot = e % (CPW * NP), cc = slot / NP, n = slot % NP;
        if (cc >= nch || n >= N) {
          const int row = e / (CPW * NP);
#pragma unroll
          for (int k = 0; k < 4; ++k) sbc[row * ROW + slot * 4 + k] = T(0.f);
          if (row == 0) *reinterpret_cast<float4*>(shs + slot * 4) = f4_zero();
        }
      }
    }
    __syncwarp();
  }

  // Per-lane chunk assignment of one (t, matrix) row (the same for every row):
  // chunk e = lane + 32 j is chunk k of channel cc.
  const int cpc = N * 4 / EPC;  // chunks per channel (N * 4 * sizeof(T) is a multiple of 16)
  int src_off[J], dst_off[J];
  bool cvalid[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = lane + 32 * j;
    const int cc = e / cpc, k = e - cc * cpc;
    cvalid[j] = cc < nch;
    src_off[j] = cc * N * 4 + k * EPC;
    dst_off[j] = cc * NP * 4 + k * EPC;
  }
  const int64_t bc_step = int64_t(D) * N * 4;  // elements per time step of B/C
  const int64_t bc_base = (int64_t(b) * T_ * D + c0) * int64_t(N) * 4;
  const T* gB = static_cast<const T*>(p.Bm) + bc_base;
  const T* gC = static_cast<const T*>(p.Cm) + bc_base;
  T* gdB = static_cast<T*>(p.dB) + bc_base;
  T* gdC = static_cast<T*>(p.dC) + bc_base;
  const int hchunks = nch * N;  // 16-byte chunks of the start states
  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  const T* gdy = static_cast<const T*>(p.dy);

  // stage sub-block sb (B, C rows and start states) into buffer buf; one commit group
  auto issue = [&](int sb, int buf) {
    unsigned char* st = wbase + size_t(buf) * G::STAGE_BYTES;
    T* sbc = reinterpret_cast<T*>(st);
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    for (int row = 0; row < 2 * len; ++row) {
      const int tt = row >> 1;
      const T* src = ((row & 1) ? gC : gB) + int64_t(t0 + tt) * bc_step;
      T* dst = sbc + row * ROW;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (cvalid[j]) cp_async16(dst + dst_off[j], src + src_off[j], true);
    }
    const float* hsrc = nullptr;
    if (sb > 0)
      hsrc = p.ckpt + ((int64_t(b) * p.nck + (sb - 1)) * D + c0) * int64_t(N) * 4;
    else if (p.h0 != nullptr)
      hsrc = p.h0 + (int64_t(b) * D + c0) * int64_t(N) * 4;
    if (hsrc != nullptr) {
      float* shs = reinterpret_cast<float*>(st + G::BC_BYTES);
      for (int e = lane; e < hchunks; e += 32) {
        const int cc = e / N, n = e - cc * N;
        cp_async16(shs + (cc * NP + n) * 4, hsrc + int64_t(e) * 4, true);
      }
    }
    // lane l < kSub * CPW copies the item of step l / CPW, channel c0 + l % CPW
    {
      const int tt = lane / CPW, cc = lane % CPW;
      if (lane < kSub * CPW && tt < len && cc < nch) {
        unsigned char* it = st + G::BC_BYTES + G::HST_BYTES + lane * G::ITEM_BYTES;
        const int t = t0 + tt, ch = c0 + cc;
        const int64_t row = (int64_t(b) * T_ + t) * D + ch;
        cp_async4(it + 0, word_of(gdelta + row), true);
        cp_async4(it + 4, p.dskip + int64_t(b) * p.dsb + int64_t(t) * p.dst + int64_t(ch) * p.dsd,
                  true);
        if constexpr (S_REAL) cp_async4(it + 8, word_of(gs + row), true);
        else cp_async_q<T>(it + 16, gs + row * 4);
        cp_async_q<T>(it + 32, gdy + row * 4);
      }
    }
    cp_async_commit();
  };

  LamPair lc;
  QPair carry, dlam = qp_zero();
  {
    LamConst k0{0.f, 0.f, 0.f, 0.f, 0.f}, k1{0.f, 0.f, 0.f, 0.f, 0.f};
    float4 h0v = f4_zero(), h1v = f4_zero();
    if (ok0) {
      k0 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n0) * 4));
      if (p.dhT != nullptr) h0v = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n0) * 4);
    }
    if (ok1) {
      k1 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n1) * 4));
      if (p.dhT != nullptr) h1v = QIO<float>::ld(p.dhT + ((int64_t(b) * D + c) * N + n1) * 4);
    }
    lc = LamPair{make_float2(k0.lr, k1.lr), make_float2(k0.li, k1.li),
                 make_float2(k0.lj, k1.lj), make_float2(k0.lk, k1.lk), make_float2(k0.m, k1.m)};
    carry = qp_from(h0v, h1v);  // conj(q_{t+1}) (x) lambda_{t+1}, = dL/dh_T at the end
  }
  const QPair lq{lc.lr, lc.li, lc.lj, lc.lk};
  const float eps = p.eps;

  const int nsub = (T_ + kSub - 1) / kSub;
  issue(nsub - 1, 0);
  for (int sb = nsub - 1; sb >= 0; --sb) {
    const int t0 = sb * kSub;
    const int len = min(kSub, T_ - t0);
    const int buf = (nsub - 1 - sb) & 1;
    if (sb > 0) {
      issue(sb - 1, buf ^ 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncwarp();
    const unsigned char* stg = wbase + size_t(buf) * G::STAGE_BYTES;
    // per-lane 32-bit shared addresses; every operand below is at a
    // compile-time offset from one of them
    constexpr int ES = int(sizeof(T));
    const uint32_t sbase = smem_addr(stg);
    const uint32_t bcl = sbase + uint32_t((chl * NP + n0) * 4 * ES);
    const uint32_t hsl = sbase + uint32_t(G::BC_BYTES + (chl * NP + n0) * 16);
    const uint32_t itl = sbase + uint32_t(G::BC_BYTES + G::HST_BYTES + chl * G::ITEM_BYTES);
    const bool zero_start = sb == 0 && p.h0 == nullptr;
    const QPair hstart = zero_start ? qp_zero()
                                    : qp_from(ldsi_f4<0>(hsl), ldsi_f4<NG * 16>(hsl));
    // B (which = 0) or C (1) of step TT: the lane's states n0 and n0 + NG
    auto ld_pair = [&](auto tt_c, auto which_c) -> QPair {
      constexpr int TT = decltype(tt_c)::value, WH = decltype(which_c)::value;
      constexpr int OFF = (TT * 2 + WH) * ROW * ES;
      return qp_from(ldsi_q<T, OFF>(bcl), ldsi_q<T, OFF + NG * 4 * ES>(bcl));
    };
    // per-(t, channel) items of step TT, broadcast to the channel's NG lanes;
    // a bf16 delta / x sits in one half of its fetched word: the element index
    // advances by D per step, so with D odd the half alternates with the step
    const int dhalf = half_of(gdelta + ((int64_t(b) * T_ + t0) * D + c));
    const int shalf = half_of(gs + ((int64_t(b) * T_ + t0) * D + c));
    const int dodd = D & 1;
    auto it_delta = [&](auto tt_c) -> float {
      constexpr int TT = decltype(tt_c)::value;
      return word_value<T>(ldsi_u32<TT * CPW * G::ITEM_BYTES>(itl), dhalf ^ (TT & dodd));
    };
    auto it_dsk = [&](auto tt_c) -> float {
      constexpr int TT = decltype(tt_c)::value;
      return __uint_as_float(ldsi_u32<TT * CPW * G::ITEM_BYTES + 4>(itl));
    };
    auto it_s = [&](auto tt_c) -> float4 {
      constexpr int TT = decltype(tt_c)::value;
      constexpr int OFF = TT * CPW * G::ITEM_BYTES;
      if constexpr (S_REAL)
        return make_float4(word_value<T>(ldsi_u32<OFF + 8>(itl), shalf ^ (TT & dodd)), 0.f, 0.f,
                           0.f);
      else
        return ldsi_q<T, OFF + 16>(itl);
    };
    auto it_dy = [&](auto tt_c) -> float4 {
      constexpr int TT = decltype(tt_c)::value;
      return ldsi_q<T, TT * CPW * G::ITEM_BYTES + 32>(itl);
    };
    // output pointers at the step the adjoint is on; it walks 7, 6, ..., 0, so
    // they move back one step per adjoint step
    T* dBp = gdB + int64_t(t0 + kSub - 1) * bc_step + (chl * N + n0) * 4;
    T* dCp = gdC + int64_t(t0 + kSub - 1) * bc_step + (chl * N + n0) * 4;
    T* ddp = static_cast<T*>(p.ddelta) + ((int64_t(b) * T_ + t0 + kSub - 1) * D + c);
    T* dsp = static_cast<T*>(p.ds) + ((int64_t(b) * T_ + t0 + kSub - 1) * D + c) * (S_REAL ? 1 : 4);

    // one recompute step: h_t = q_t (x) h_{t-1} + B_t (x) S_t
    auto fwd_step = [&](const QPair& h, auto tt_c) -> QPair {
      const float dl = it_delta(tt_c);
      const QPair Bq = ld_pair(tt_c, std::integral_constant<int, 0>{});
      const QPair qv = cayley_pair(dl, dl * dl, lc, eps);
      QPair inj;
      if constexpr (S_REAL) {
        const float2 s2 = bc2(it_s(tt_c).x);
        inj = QPair{mul2(s2, Bq.x), mul2(s2, Bq.y), mul2(s2, Bq.z), mul2(s2, Bq.w)};
      } else {
        inj = qp_mul_bcast(Bq, it_s(tt_c));
      }
      return qp_mul_acc(qv, h, inj);
    };
    // one adjoint step at TT, given the states after steps TT and TT - 1; runs
    // for TT < len only, but moves the output pointers back in every case
    auto adj_step = [&](auto tt_c, bool run, const QPair& hcur, const QPair& hprev) {
      if (run) {
        const float dl = it_delta(tt_c);
        const float4 sv = it_s(tt_c);
        const float4 gy = it_dy(tt_c);
        const float dsk = it_dsk(tt_c);
        const QPair Bq = ld_pair(tt_c, std::integral_constant<int, 0>{});
        const QPair Cq = ld_pair(tt_c, std::integral_constant<int, 1>{});
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
        float4 psum = make_float4(ng == 0 ? dsk * gy.x : 0.f, ng == 0 ? dsk * gy.y : 0.f,
                                  ng == 0 ? dsk * gy.z : 0.f, ng == 0 ? dsk * gy.w : 0.f);
        if constexpr (S_REAL) {
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
        const QPair dC = qp_bmul(gy, qp_conj(hcur));
        if (ok0) {
          QIO<T>::st(dBp, qp_half(dB, 0));
          QIO<T>::st(dCp, qp_half(dC, 0));
        }
        if (ok1) {
          QIO<T>::st(dBp + NG * 4, qp_half(dB, 1));
          QIO<T>::st(dCp + NG * 4, qp_half(dC, 1));
        }
        carry = qp_mul_acc(qp_conj(qv), lam, qp_zero());
        // sum ddelta and dS over the channel's lanes at once (no partials are
        // held across steps, which keeps the sub-block's register set small)
        if constexpr (S_REAL) {
          float v[2] = {pdp.x + pdp.y, psum.x};
          const int k = reduce_scatter<2, NG>(v, ng);  // lanes with ng & 1 == k hold sum k
          if (active && (ng >> 1) == 0) QIO<T>::st1(k == 0 ? ddp : dsp, v[0]);
        } else {
          float v[8] = {pdp.x + pdp.y, psum.x, psum.y, psum.z, psum.w, 0.f, 0.f, 0.f};
          const int k = reduce_scatter<8, NG>(v, ng);  // one sum per lane (8 <= NG)
          if (active && (ng >> 3) == 0 && k <= 4) QIO<T>::st1(k == 0 ? ddp : dsp + (k - 1), v[0]);
        }
      }
      dBp -= bc_step;
      dCp -= bc_step;
      ddp -= D;
      dsp -= int64_t(D) * (S_REAL ? 1 : 4);
    };
    // The sub-block runs in two halves so that at most five recomputed states are
    // live (instead of kSub): pass A recomputes steps 0..7 and keeps the states
    // after steps 3..7 for the adjoint of steps 7..4; pass B recomputes steps
    // 0..2 again (same operations, same bits) for the adjoint of steps 3..0.
    static_assert(kSub == 8, "the two-half schedule assumes 8-step sub-blocks");
    auto run_sub = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
      QPair hk[5];  // states after steps 3..7
      {
        QPair h = hstart;
        static_for<0, kSub>([&](auto tt_c) {
          constexpr int TT = decltype(tt_c)::value;
          if (FULL || TT < len) h = fwd_step(h, tt_c);
          if constexpr (TT >= 3) hk[TT - 3] = h;
        });
      }
      static_for_down<kSub - 1, 4>([&](auto tt_c) {
        constexpr int TT = decltype(tt_c)::value;
        adj_step(tt_c, FULL || TT < len, hk[TT - 3], hk[TT - 4]);
      });
      QPair hl[3];  // states after steps 0..2
      {
        QPair h = hstart;
        static_for<0, 3>([&](auto tt_c) {
          constexpr int TT = decltype(tt_c)::value;
          if (FULL || TT < len) h = fwd_step(h, tt_c);
          hl[TT] = h;
        });
      }
      static_for_down<3, 0>([&](auto tt_c) {
        constexpr int TT = decltype(tt_c)::value;
        if constexpr (TT == 3) adj_step(tt_c, FULL || TT < len, hk[0], hl[2]);
        else if constexpr (TT == 0) adj_step(tt_c, FULL || TT < len, hl[0], hstart);
        else adj_step(tt_c, FULL || TT < len, hl[TT], hl[TT - 1]);
      });
    };
    if (len == kSub) run_sub(std::true_type{});
    else run_sub(std::false_type{});
    __syncwarp();  // every lane is done with this stage before it is refilled
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
int launch_pc(const BwdParams& p, cudaStream_t st) {
  using G = PcGeom<T, NG>;
  constexpr int WARPS = pc_warps<T>();
  const size_t smem = size_t(WARPS) * 2 * G::STAGE_BYTES;
  const bool exact = p.N == 2 * NG && p.D % G::CPW == 0;
  auto kern = exact ? ssm_scan_bwd_pc_kernel<T, NG, S_REAL, true>
                    : ssm_scan_bwd_pc_kernel<T, NG, S_REAL, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_ssm_scan_bwd: smem attribute (%zu B): %s", smem,
                cudaGetErrorString(e));
  const int per_cta = WARPS * G::CPW;
  dim3 grid{unsigned((p.D + per_cta - 1) / per_cta), unsigned(p.B), 1u};
  kern<<<grid, 32 * WARPS, smem, st>>>(p);
  return check_launch("mqc_ssm_scan_bwd(per-channel packed)");
}

template <typename T>
int launch_pc_t(const BwdParams& p, bool s_real, cudaStream_t st) {
  const bool ng32 = p.N > 32;
  if (s_real) return ng32 ? launch_pc<T, 32, true>(p, st) : launch_pc<T, 16, true>(p, st);
  return ng32 ? launch_pc<T, 32, false>(p, st) : launch_pc<T, 16, false>(p, st);
}

}  // namespace

bool perchannel_bwd_serves(int N, int dtype) {
  // lanes hold pairs (ng, ng + NG) with NG in {16, 32}; a channel's row of N
  // quaternions must be whole 16-byte chunks for cp.async
  if (N <= 16 || N > 64) return false;
  return dtype == MQC_DTYPE_F32 || (N % 2) == 0;
}

int launch_bwd_perchannel(const BwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  if (!perchannel_bwd_serves(p.N, dtype))
    return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_bwd: per-channel packed path needs "
                                     "16 < d_state <= 64 (even for bf16)");
  if (dtype == MQC_DTYPE_F32) return launch_pc_t<float>(p, s_real, st);
  return launch_pc_t<__nv_bfloat16>(p, s_real, st);
}

}  // namespace scan
}  // namespace mqc
