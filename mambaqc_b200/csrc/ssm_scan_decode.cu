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

// ------------------------------------------------ large decode batches
// For many batch rows the step is a pure stream of the state cache (read once,
// written once). A CTA owns a block of CB channels -- its Lambda constants stay
// in registers -- and walks a range of batch rows; for each row a producer warp
// bulk-copies the block's contiguous state slab (CB x N x 16 bytes, 8 KB at
// N = 64) and the row's B and C into a kStrStages-deep shared-memory ring, so
// every SM keeps tens of KB of reads in flight without holding registers for
// them. The consumer warps (a channel per NG lanes, two states per lane) compute
// the step, store the new state straight to the cache and y, and release the
// stage. Arithmetic and readout order are those of the streaming kernel.
constexpr int kStrWarps = 8;   // consumer warps
constexpr int kStrStages = 5;  // ring depth (rows in flight per CTA)

__host__ __device__ inline uint32_t str_stage_bytes(int cb, int N, int tsize) {
  return uint32_t(cb) * N * 16 + 2u * uint32_t(N) * 4 * tsize;
}

// Four CTAs per SM (56 registers per thread, 5 x 10 KB stages each): about
// 200 KB of state reads in flight per SM.
template <typename T, int NG, bool S_REAL>
__global__ void __launch_bounds__(32 * (kStrWarps + 1), 4)
    scan_decode_stream_kernel(const FwdParams p, int rows_per_cta) {
  constexpr int CPW = 32 / NG;
  constexpr int CB = kStrWarps * CPW;
  constexpr unsigned kFull = 0xffffffffu;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kStrStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStrStages);
  unsigned char* ring = smem + 128;
  const int N = p.N, D = p.D;
  const int c0 = blockIdx.x * CB;
  const int nch = min(CB, D - c0);
  const int b0 = blockIdx.y * rows_per_cta;
  const int nrows = min(rows_per_cta, p.B - b0);
  const uint32_t hbytes = p.h0 != nullptr ? uint32_t(nch) * N * 16 : 0u;
  const uint32_t bcbytes = uint32_t(N) * 4 * sizeof(T);
  const uint32_t stage_bytes = str_stage_bytes(CB, N, sizeof(T));
  const uint32_t off_b = uint32_t(CB) * N * 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStrStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStrWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kStrWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int r = 0; r < nrows; ++r) {
        const int s = r % kStrStages;
        if (r >= kStrStages) {
          ok = mbar_wait_bounded(&empty[s], uint32_t(((r / kStrStages) - 1) & 1), p.wait_limit);
          if (!ok) break;
        }
        if (*abort_flag) break;
        const int64_t b = b0 + r;
        unsigned char* st = ring + size_t(s) * stage_bytes;
        mbar_arrive_expect_tx(&full[s], hbytes + 2 * bcbytes);
        if (hbytes != 0) bulk_g2s(st, p.h0 + (b * D + c0) * int64_t(N) * 4, hbytes, &full[s]);
        bulk_g2s(st + off_b, static_cast<const T*>(p.Bm) + b * N * 4, bcbytes, &full[s]);
        bulk_g2s(st + off_b + bcbytes, static_cast<const T*>(p.Cm) + b * N * 4, bcbytes,
                 &full[s]);
        issued = r + 1;
      }
      if (!ok) {
        *abort_flag = 1;
        report_status(p.status, MQC_DEVICE_STATUS_TIMEOUT);
      }
      // the CTA must outlive its copies: wait (bounded) for the last ones issued
      for (int r = issued > kStrStages ? issued - kStrStages : 0; r < issued; ++r)
        mbar_wait_bounded(&full[r % kStrStages], uint32_t((r / kStrStages) & 1), kDrainPollLimit);
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int ng = lane % NG;
  const int cl = warp * CPW + lane / NG;
  const bool active = cl < nch;
  const int c = active ? c0 + cl : c0;
  const int n0 = ng, n1 = ng + NG;
  const bool ok0 = active && n0 < N, ok1 = active && n1 < N;
  LamConst l0{0.f, 0.f, 0.f, 0.f, 0.f}, l1{0.f, 0.f, 0.f, 0.f, 0.f};
  if (ok0) l0 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n0) * 4));
  if (ok1) l1 = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n1) * 4));
  const T* gdelta = static_cast<const T*>(p.delta);
  const T* gs = static_cast<const T*>(p.s);
  // Delta and the signal of the next row, loaded one row ahead
  auto load_row = [&](int r, float& dl, float4& sv) {
    dl = 0.f;
    sv = f4_zero();
    if (active && r < nrows) {
      const int64_t row = int64_t(b0 + r) * D + c;
      dl = to_f(gdelta[row]);
      if (S_REAL) sv.x = to_f(gs[row]);
      else sv = QIO<T>::ld(gs + row * 4);
    }
  };
  float dl_n;
  float4 sv_n;
  load_row(0, dl_n, sv_n);
  const float eps = p.eps;
  for (int r = 0; r < nrows; ++r) {
    const int s = r % kStrStages;
    bool ok = *abort_flag == 0 &&
              mbar_wait_bounded(&full[s], uint32_t((r / kStrStages) & 1), p.wait_limit);
    if (!__all_sync(kFull, ok)) {
      if (lane == 0) {
        *abort_flag = 1;
        report_status(p.status, MQC_DEVICE_STATUS_TIMEOUT);
      }
      return;
    }
    const float dl = dl_n;
    const float4 sv = sv_n;
    load_row(r + 1, dl_n, sv_n);
    const int b = b0 + r;
    const unsigned char* st = ring + size_t(s) * stage_bytes;
    const float* sh = reinterpret_cast<const float*>(st) + int64_t(cl) * N * 4;
    const T* sB = reinterpret_cast<const T*>(st + off_b);
    const T* sC = reinterpret_cast<const T*>(st + off_b + bcbytes);
    float4 h[2], Bv[2], Cv[2];
    h[0] = h[1] = Bv[0] = Bv[1] = Cv[0] = Cv[1] = f4_zero();
    if (ok0) {
      if (hbytes != 0) h[0] = QIO<float>::lds(sh + n0 * 4);
      Bv[0] = QIO<T>::lds(sB + n0 * 4);
      Cv[0] = QIO<T>::lds(sC + n0 * 4);
    }
    if (ok1) {
      if (hbytes != 0) h[1] = QIO<float>::lds(sh + n1 * 4);
      Bv[1] = QIO<T>::lds(sB + n1 * 4);
      Cv[1] = QIO<T>::lds(sC + n1 * 4);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage is read: free for the producer
    const float d2 = dl * dl;
    float4 hn[2];
    float4 ya = f4_zero(), yb = f4_zero();
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float4 qv = cayley_from_const(dl, d2, e ? l1 : l0, eps);
      float4 inj;
      if (S_REAL)
        inj = make_float4(sv.x * Bv[e].x, sv.x * Bv[e].y, sv.x * Bv[e].z, sv.x * Bv[e].w);
      else
        inj = qmul(Bv[e], sv);
      hn[e] = qmul_acc(qv, h[e], inj);
      if (e) yb = qmul_acc(Cv[e], hn[e], yb);
      else ya = qmul_acc(Cv[e], hn[e], ya);
    }
    ya.x += yb.x;
    ya.y += yb.y;
    ya.z += yb.z;
    ya.w += yb.w;
    const float dsk = active ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(c) * p.dsd) : 0.f;
    reduce_store_y<T, NG>(ya, sv, dsk, ng, active,
                          static_cast<T*>(p.y) + (int64_t(b) * D + c) * 4);
    const int64_t hs = (int64_t(b) * D + c) * N;
    if (ok0) QIO<float>::st(p.hT + (hs + n0) * 4, hn[0]);
    if (ok1) QIO<float>::st(p.hT + (hs + n1) * 4, hn[1]);
  }
}

template <typename T, int NG, bool S_REAL>
int launch_decode_stream(const FwdParams& p, cudaStream_t st) {
  constexpr int CB = kStrWarps * (32 / NG);
  const int nblk = (p.D + CB - 1) / CB;
  // one resident wave (four CTAs per SM): as many row ranges per channel block
  // as fit beside the blocks, so no SM waits on a partial second wave
  const int64_t slots = int64_t(num_sms()) * 4;
  int64_t ranges = slots / nblk;
  if (ranges < 1) ranges = 1;
  if (ranges > p.B) ranges = p.B;
  const int rpc = int((p.B + ranges - 1) / ranges);
  const unsigned gy = unsigned((p.B + rpc - 1) / rpc);
  const size_t smem = 128 + size_t(kStrStages) * str_stage_bytes(CB, p.N, sizeof(T));
  auto kern = scan_decode_stream_kernel<T, NG, S_REAL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd(decode): smem attribute: %s",
                  cudaGetErrorString(e));
  }
  dim3 grid{unsigned(nblk), gy, 1u};
  kern<<<grid, 32 * (kStrWarps + 1), smem, st>>>(p, rpc);
  return check_launch("mqc_ssm_scan_fwd(decode stream)");
}

template <typename T, bool S_REAL>
int dispatch_decode_stream_t(const FwdParams& p, cudaStream_t st) {
  const int need = (p.N + 1) / 2;
  int ng = 1;
  while (ng < need) ng <<= 1;
  switch (ng) {
    case 1: return launch_decode_stream<T, 1, S_REAL>(p, st);
    case 2: return launch_decode_stream<T, 2, S_REAL>(p, st);
    case 4: return launch_decode_stream<T, 4, S_REAL>(p, st);
    case 8: return launch_decode_stream<T, 8, S_REAL>(p, st);
    case 16: return launch_decode_stream<T, 16, S_REAL>(p, st);
    default: return launch_decode_stream<T, 32, S_REAL>(p, st);
  }
}

}  // namespace

// Up to 32 batch rows: the row-blocked kernel (measured at config-3 channel and
// state sizes: 4.0 / 13.2 us per step at 4 / 16 rows, against 4.4 / 13.8 us on
// the general streaming kernel); more rows: the state-streaming kernel.
bool decode_serves(const FwdParams& p) {
  return p.T == 1 && p.N <= 64 && p.hT != nullptr && p.ckpt == nullptr && p.pout == nullptr;
}

int dispatch_decode(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  if (p.B > 32) {  // the state-streaming kernel
    if (dtype == MQC_DTYPE_F32)
      return s_real ? dispatch_decode_stream_t<float, true>(p, st)
                    : dispatch_decode_stream_t<float, false>(p, st);
    return s_real ? dispatch_decode_stream_t<__nv_bfloat16, true>(p, st)
                  : dispatch_decode_stream_t<__nv_bfloat16, false>(p, st);
  }
  if (dtype == MQC_DTYPE_F32)
    return s_real ? dispatch_decode_t<float, true>(p, st) : dispatch_decode_t<float, false>(p, st);
  return s_real ? dispatch_decode_t<__nv_bfloat16, true>(p, st)
                : dispatch_decode_t<__nv_bfloat16, false>(p, st);
}

}  // namespace scan
}  // namespace mqc
