// Fused Cayley + quaternion selective scan, forward, for B/C shared by all
// channels ([B,T,N,4]; the layout of the hot-path configuration) -- the
// warp-specialised kernel.
//
// Same math as ssm_scan_fwd.cu (QuaternionMamba2Block._ssm_forward,
// mambaqc/models/quaternion_mamba2_block.py:214-228, without materialising z or
// q), organised so that no block-wide barrier sits in the time loop:
//
//  * warp 0 is the producer: one lane streams the B_t/C_t tiles of each chunk of
//    tc timesteps into a kRing-deep shared-memory ring with bulk copies (TMA
//    engine), signalling `full[stage]` by transaction bytes and waiting on
//    `empty[stage]` before it reuses a stage;
//  * every other warp is a consumer that owns 32/NG channels x N states
//    (G states per lane, n = ng + NG*i); it stages its own channels' delta and
//    x (or S) one chunk ahead through registers into a warp-private buffer,
//    waits on `full`, runs the chunk, and releases the stage with one arrive on
//    `empty` -- warps drift freely and only meet in the ring;
//  * B/C rows in shared memory are padded to NP = NG*G states with zeros, so
//    the inner loop has no lane guards;
//  * the per-step readout sum over n is in registers over G states (two
//    accumulators) and a shuffle reduce-scatter over the NG lanes of a channel.
//
// All waits are bounded (poll limit); on timeout the kernel reports
// MQC_DEVICE_STATUS_TIMEOUT, raises a shared abort flag so the other warps stop
// at their next chunk, and the producer drains its copies in flight before it
// exits.
#include <cstdlib>
#include <type_traits>

#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {

constexpr int kRing = 3;
// CTA size cap: 8 states per lane need ~128 registers per thread (512 threads);
// 4 states per lane fit in ~80 (768 threads).
__host__ __device__ constexpr int v2_max_threads(int g) { return g == 4 ? 768 : 512; }
constexpr int kV2MaxDx = 8;   // staged delta/x elements per lane per chunk (real signal)
constexpr int kV2MaxDxQ = 2;  // the same for a quaternion signal S (4x the registers)
constexpr size_t kV2SmemBudget = 220 * 1024;

struct V2Layout {
  size_t off_b, off_c, off_dx, off_sx, total;
};

// [full x kRing][empty x kRing][abort flag] | sB [kRing][tc][np][4] | sC |
// per consumer warp: delta [2][tc][cpw] f32 | s [2][tc][cpw][sw] f32
template <typename T>
__host__ __device__ inline V2Layout v2_layout(int tc, int np, int warps, int cpw, int sw) {
  V2Layout L;
  size_t off = 128;
  const size_t ring = size_t(kRing) * tc * np * 4 * sizeof(T);
  L.off_b = off;
  off = align_up(off + ring, 128);
  L.off_c = off;
  off = align_up(off + ring, 128);
  L.off_dx = off;
  off = align_up(off + size_t(warps) * 2 * tc * cpw * sizeof(float), 16);
  L.off_sx = off;
  off = align_up(off + size_t(warps) * 2 * tc * cpw * sw * sizeof(float), 16);
  L.total = off;
  return L;
}

template <typename T, int G, int NG, bool S_REAL>
__global__ void __launch_bounds__(v2_max_threads(G), 1)
    scan_fwd_shared_kernel(const FwdParams p, const int np) {
  constexpr int CPW = 32 / NG;  // channels per consumer warp
  constexpr int SW = S_REAL ? 1 : 4;
  constexpr unsigned kFull = 0xffffffffu;
  extern __shared__ __align__(128) unsigned char smem_raw[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps_c = (blockDim.x >> 5) - 1;
  const int T_ = p.T, D = p.D, N = p.N, tc = p.tc;
  const int b = blockIdx.y;
  const int c0 = int((int64_t(D) * blockIdx.x) / p.nb);
  const int c1 = int((int64_t(D) * (blockIdx.x + 1)) / p.nb);
  const int nch = c1 - c0;
  const int busy_warps = (nch + CPW - 1) / CPW;
  const int nchunks = (T_ + tc - 1) / tc;

  const V2Layout L = v2_layout<T>(tc, np, nwarps_c, CPW, SW);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kRing;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kRing);
  T* sB = reinterpret_cast<T*>(smem_raw + L.off_b);
  T* sC = reinterpret_cast<T*>(smem_raw + L.off_c);

  // zero the padding states n in [N, np) of every ring row once; copies never touch them
  if (np != N) {
    const int pad = np - N;
    for (int i = threadIdx.x; i < kRing * tc * pad; i += blockDim.x) {
      const int row = i / pad, n = N + i % pad;
      QIO<T>::st(sB + (int64_t(row) * np + n) * 4, f4_zero());
      QIO<T>::st(sC + (int64_t(row) * np + n) * 4, f4_zero());
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], uint32_t(busy_warps));
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // ------------------------------------------------------------- producer
  if (warp == 0) {
    if (lane == 0) {
      const T* gB = static_cast<const T*>(p.Bm);
      const T* gC = static_cast<const T*>(p.Cm);
      const uint32_t row_bytes = uint32_t(N) * 4 * sizeof(T);
      int issued = 0;
      bool ok = true;
      for (int k = 0; k < nchunks; ++k) {
        const int st = k % kRing;
        if (k >= kRing) {
          ok = mbar_wait_bounded(&empty[st], uint32_t(((k / kRing) - 1) & 1), p.wait_limit);
          if (!ok) break;
        }
        if (*abort_flag) break;
        const int t0 = k * tc;
        const int len = min(tc, T_ - t0);
        mbar_arrive_expect_tx(&full[st], 2u * uint32_t(len) * row_bytes);
        const int64_t g0 = (int64_t(b) * T_ + t0) * N * 4;
        T* dB = sB + int64_t(st) * tc * np * 4;
        T* dC = sC + int64_t(st) * tc * np * 4;
        if (np == N) {
          bulk_g2s(dB, gB + g0, uint32_t(len) * row_bytes, &full[st]);
          bulk_g2s(dC, gC + g0, uint32_t(len) * row_bytes, &full[st]);
        } else {
          for (int tt = 0; tt < len; ++tt) {
            bulk_g2s(dB + int64_t(tt) * np * 4, gB + g0 + int64_t(tt) * N * 4, row_bytes, &full[st]);
            bulk_g2s(dC + int64_t(tt) * np * 4, gC + g0 + int64_t(tt) * N * 4, row_bytes, &full[st]);
          }
        }
        issued = k + 1;
      }
      if (!ok) {
        *abort_flag = 1;
        report_status(p.status, MQC_DEVICE_STATUS_TIMEOUT);
      }
      // the CTA must outlive its copies: wait (bounded) for the last ones issued
      for (int k = issued > kRing ? issued - kRing : 0; k < issued; ++k)
        mbar_wait_bounded(&full[k % kRing], uint32_t((k / kRing) & 1), kDrainPollLimit);
    }
    return;
  }

  // ------------------------------------------------------------- consumers
  const int cw = warp - 1;
  if (cw >= busy_warps) return;
  const int lc_ch = lane / NG;  // channel slot within the warp
  const int ng = lane % NG;
  const int cl = cw * CPW + lc_ch;
  const bool active = cl < nch;
  const int c = active ? c0 + cl : c0;

  float4 h[G];
  LamConst lc[G];
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int n = ng + NG * i;
    h[i] = f4_zero();
    lc[i] = LamConst{0.f, 0.f, 0.f, 0.f, 0.f};
    if (active && n < N) {
      if (p.h0 != nullptr) h[i] = QIO<float>::ld(p.h0 + ((int64_t(b) * D + c) * N + n) * 4);
      lc[i] = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n) * 4));
    }
  }
  const bool d_const = p.dst == 0;
  const float dsk0 = active ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(c) * p.dsd) : 0.f;

  // warp-private staging of delta and s: [2][tc][CPW] (+ [SW] for s)
  float* wdel = reinterpret_cast<float*>(smem_raw + L.off_dx) + int64_t(cw) * 2 * tc * CPW;
  float* wsig = reinterpret_cast<float*>(smem_raw + L.off_sx) + int64_t(cw) * 2 * tc * CPW * SW;
  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  const int per_chunk = tc * CPW;
  // fp32 inputs: delta / s go global -> shared with cp.async (no registers held
  // across the chunk); bf16 inputs (2-byte elements) go through registers.
  constexpr bool kAsync = std::is_same<T, float>::value;
  constexpr int MD = kAsync ? 1 : (S_REAL ? kV2MaxDx : kV2MaxDxQ);
  float rd[MD];
  float4 rs[MD];
  auto issue_dx_async = [&](int k, int buf) {
    const int t0 = k * tc;
    for (int e = lane; e < per_chunk; e += 32) {
      const int tt = e / CPW, cc = cw * CPW + e % CPW;
      const bool v = (t0 + tt < T_) && (cc < nch);
      const int64_t idx = v ? (int64_t(b) * T_ + t0 + tt) * D + c0 + cc : 0;
      cp_async4(wdel + buf * per_chunk + e, gdelta + idx, v);
      if (S_REAL) cp_async4(wsig + buf * per_chunk + e, gs + idx, v);
      else cp_async16(wsig + (buf * per_chunk + e) * 4, gs + idx * 4, v);
    }
    cp_async_commit();
  };
  auto load_dx = [&](int k) {
    const int t0 = k * tc;
#pragma unroll
    for (int j = 0; j < MD; ++j) {
      const int e = lane + 32 * j;
      rd[j] = 0.f;
      rs[j] = f4_zero();
      if (e < per_chunk) {
        const int tt = e / CPW, cc = cw * CPW + e % CPW;
        if (t0 + tt < T_ && cc < nch) {
          const int64_t idx = (int64_t(b) * T_ + t0 + tt) * D + c0 + cc;
          rd[j] = to_f(gdelta[idx]);
          if (S_REAL) rs[j].x = to_f(gs[idx]);
          else rs[j] = QIO<T>::ld(gs + idx * 4);
        }
      }
    }
  };
  auto store_dx = [&](int buf) {
#pragma unroll
    for (int j = 0; j < MD; ++j) {
      const int e = lane + 32 * j;
      if (e < per_chunk) {
        wdel[buf * per_chunk + e] = rd[j];
        if (S_REAL) wsig[buf * per_chunk + e] = rs[j].x;
        else reinterpret_cast<float4*>(wsig)[buf * per_chunk + e] = rs[j];
      }
    }
  };

  if constexpr (kAsync) {
    issue_dx_async(0, 0);
    cp_async_wait_all();
  } else {
    load_dx(0);
    store_dx(0);
  }
  __syncwarp();

  const float eps = p.eps;
  T* yb = static_cast<T*>(p.y) + (int64_t(b) * T_ * D + c) * 4;
  for (int k = 0; k < nchunks; ++k) {
    const int st = k % kRing;
    const int buf = k & 1;
    bool ok = *abort_flag == 0;
    if (ok) ok = mbar_wait_bounded(&full[st], uint32_t((k / kRing) & 1), p.wait_limit);
    if (!__all_sync(kFull, ok)) {
      if (lane == 0) {
        *abort_flag = 1;
        report_status(p.status, MQC_DEVICE_STATUS_TIMEOUT);
      }
      return;
    }
    if (k + 1 < nchunks) {
      if constexpr (kAsync) issue_dx_async(k + 1, buf ^ 1);
      else load_dx(k + 1);
    }

    const int t0 = k * tc;
    const int len = min(tc, T_ - t0);
    const float* cdel = wdel + buf * per_chunk;
    const float* csig = wsig + buf * per_chunk * SW;
    const T* rowB = sB + int64_t(st) * tc * np * 4 + ng * 4;
    const T* rowC = sC + int64_t(st) * tc * np * 4 + ng * 4;
    for (int tt = 0; tt < len; ++tt) {
      const int t = t0 + tt;
      const float dl = cdel[tt * CPW + lc_ch];
      const float dl2 = dl * dl;
      float4 sv;
      if (S_REAL) sv = make_float4(csig[tt * CPW + lc_ch], 0.f, 0.f, 0.f);
      else sv = reinterpret_cast<const float4*>(csig)[tt * CPW + lc_ch];
      float4 ya = f4_zero(), yb2 = f4_zero();
#pragma unroll
      for (int i = 0; i < G; ++i) {
        const float4 Bv = QIO<T>::lds(rowB + (tt * np + NG * i) * 4);
        const float4 Cv = QIO<T>::lds(rowC + (tt * np + NG * i) * 4);
        const float4 qv = cayley_from_const(dl, dl2, lc[i], eps);
        float4 inj;
        if (S_REAL) inj = make_float4(sv.x * Bv.x, sv.x * Bv.y, sv.x * Bv.z, sv.x * Bv.w);
        else inj = qmul(Bv, sv);
        h[i] = qmul_acc(qv, h[i], inj);
        if (i & 1) yb2 = qmul_acc(Cv, h[i], yb2);
        else ya = qmul_acc(Cv, h[i], ya);
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
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (k + 1 < nchunks) {
      if constexpr (kAsync) cp_async_wait_all();
      else store_dx(buf ^ 1);
      __syncwarp();
    }
  }

  if (p.hT != nullptr && active) {
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const int n = ng + NG * i;
      if (n < N) QIO<float>::st(p.hT + ((int64_t(b) * D + c) * N + n) * 4, h[i]);
    }
  }
}

template <typename T, int G, int NG, bool S_REAL>
int launch_shared(FwdParams p, cudaStream_t st) {
  constexpr int CPW = 32 / NG;
  const int np = NG * G;
  const int sw = S_REAL ? 1 : 4;
  // one CTA per SM: nb CTAs per batch row with B * nb <= #SMs (never a partial
  // second wave); rows beyond #SMs simply queue
  const int sms = num_sms();
  int nb = sms / p.B;
  if (nb > p.D) nb = p.D;
  if (nb < 1) nb = 1;
  int cpb = (p.D + nb - 1) / nb;
  const int cap = (v2_max_threads(G) / 32 - 1) * CPW;
  if (cpb > cap) {
    nb = (p.D + cap - 1) / cap;
    cpb = (p.D + nb - 1) / nb;
  }
  const int warps = (cpb + CPW - 1) / CPW;
  int tc = kMaxTc;
  const int max_dx = S_REAL ? kV2MaxDx : kV2MaxDxQ;
  while (tc > 1 && tc * CPW > 32 * max_dx) tc >>= 1;
  if (tc > p.T) tc = p.T;
  size_t smem = v2_layout<T>(tc, np, warps, CPW, sw).total;
  while (smem > kV2SmemBudget && tc > 1) {
    tc >>= 1;
    smem = v2_layout<T>(tc, np, warps, CPW, sw).total;
  }
  if (smem > kV2SmemBudget)
    return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_fwd: shared staging does not fit (N=%d)", p.N);
  p.nb = nb;
  p.cpb = cpb;
  p.tc = tc;
  auto kern = scan_fwd_shared_kernel<T, G, NG, S_REAL>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd: smem attribute (%zu B): %s", smem,
                cudaGetErrorString(e));
  dim3 grid{unsigned(nb), unsigned(p.B), 1u};
  kern<<<grid, 32 * (warps + 1), smem, st>>>(p, np);
  return check_launch("mqc_ssm_scan_fwd(shared)");
}

template <typename T, int G, bool S_REAL>
int dispatch_shared_g(const FwdParams& p, cudaStream_t st) {
  // NG = lanes per channel: the power of two covering ceil(N / G), at most 32
  const int need = (p.N + G - 1) / G;
  int ng = 1;
  while (ng < need) ng <<= 1;
  switch (ng) {
    case 1: return launch_shared<T, G, 1, S_REAL>(p, st);
    case 2: return launch_shared<T, G, 2, S_REAL>(p, st);
    case 4: return launch_shared<T, G, 4, S_REAL>(p, st);
    case 8: return launch_shared<T, G, 8, S_REAL>(p, st);
    case 16: return launch_shared<T, G, 16, S_REAL>(p, st);
    case 32: return launch_shared<T, G, 32, S_REAL>(p, st);
    default:
      return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_fwd: d_state=%d (supported 1..%d)", p.N,
                  32 * G);
  }
}

// States per lane: 8 by default; MQC_SCAN_G=4 selects 4 (twice the warps, half
// the registers per thread) for tuning comparisons.
int states_per_lane() {
  static const int g = [] {
    const char* v = getenv("MQC_SCAN_G");
    return (v != nullptr && v[0] == '4' && v[1] == '\0') ? 4 : 8;
  }();
  return g;
}

template <typename T, bool S_REAL>
int dispatch_shared_t(const FwdParams& p, cudaStream_t st) {
  if (states_per_lane() == 4 && p.N <= 128) return dispatch_shared_g<T, 4, S_REAL>(p, st);
  return dispatch_shared_g<T, 8, S_REAL>(p, st);
}

int dispatch_shared(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32)
    return s_real ? dispatch_shared_t<float, true>(p, st) : dispatch_shared_t<float, false>(p, st);
  return s_real ? dispatch_shared_t<__nv_bfloat16, true>(p, st)
                : dispatch_shared_t<__nv_bfloat16, false>(p, st);
}

}  // namespace scan
}  // namespace mqc
