// The B/C projections of the block fused into its per-channel scan, forward.
//
// The reference block (mambaqc/models/quaternion_mamba2_block.py:186-191 and
// 214-228) computes B = B_proj(x) and C = C_proj(x) -- two real -> quaternion
// projections, F.linear with d_inner * d_state * 4 outputs
// (mambaqc/layers/quaternion_linear.py:145-161) -- views them per channel as
// [B, T, d_inner, d_state, 4] and scans
//   h_t = q_t (x) h_{t-1} + B_t s_t,  y_t = sum_n C_t (x) h_t + D s_t,
//   q_t = cayley(delta_t Lambda).
// B and C are the widest tensors of the block (2 x 6.4 GB in bf16 at B=4,
// T=2048, d_inner 1536, d_state 64): the GEMMs write them and the scan reads
// them back. Here they never leave the SM: a CTA owns one recurrence (batch row
// b, channel d), and for every tile of BM = 128 time steps
//   1. the tensor cores compute the channel's B and C tile,
//        B[t, f] = sum_k x[b, t, k] W_B[d*4N + f, k]   (f = 4n + component),
//      as two 128 x 4N fp32 accumulators in tensor memory (tcgen05.mma, bf16
//      operands staged by TMA through a shared-memory ring);
//   2. four copy warps -- one per 32-lane quarter of tensor memory, i.e. per
//      32-step slab of the tile -- read the accumulators (tcgen05.ld), round
//      them to bf16 (the projection's output type in the reference's bf16
//      autocast) and store the slab's rows [t][f] in shared memory;
//   3. the scan warps (a state per lane) run the 32 steps of the slab from
//      those rows, four steps at a time, reduce the four steps' readouts over
//      the states with one reduce-scatter, add D s and store y.
// There are three slab buffers, so the tensor memory is released once the
// fourth slab is copied, which waits only for the scan of the tile's first
// slab: the next tile's MMAs overlap the scan of the other three.
//
// Warp roles (256 threads, one CTA per SM):
//   warp 0      TMA producer (one thread): x tile + W_B tile + W_C tile per stage
//   warp 1      tensor-memory allocation and the MMA issuer (one thread)
//   warps 2..5  copy warps (warp w reads tensor-memory lanes 32 (w % 4) ...)
//   warps 6..7  scan warps (states 32 (w - 6) + lane)
// Every mbarrier wait is bounded: on timeout the CTA raises its abort flag and
// the status word, the other roles stop at their next wait, what was issued is
// drained (bounded), the tensor memory is freed and the kernel returns. Plain
// TMA loads only (no multicast); every tensor map covers this GPU's memory.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "ssm_scan_common.cuh"
#include "tc_common.cuh"

namespace mqc {
namespace bcscan {
namespace {

using scan::cayley_from_const;
using scan::LamConst;
using scan::make_lam_const;

constexpr int BM = 128;        // time steps of one batch row per tile (tensor-memory lanes)
constexpr int kSlab = 32;      // time steps per slab (one lane quarter)
constexpr int kThreads = 256;  // 8 warps
constexpr unsigned kFull = 0xffffffffu;

constexpr size_t kSmemMax = 232448;  // dynamic shared memory of one CTA (227 KB)

template <int N, int BK>
struct Cfg {
  static constexpr int BN = 4 * N;          // projection outputs per channel (B or C), MMA N
  static constexpr int kRowBytes = BK * 2;  // one swizzle row of a K block
  static constexpr uint32_t kXBytes = BM * BK * 2;
  static constexpr uint32_t kWBytes = BN * BK * 2;
  static constexpr uint32_t kStageBytes = kXBytes + 2 * kWBytes;
  static constexpr int kRowPad = BN + 8;  // bf16 per slab row (16 bytes of padding)
  // three slab buffers: the tensor memory is free once the scan has finished
  // the first slab of a tile (the other three are copied out at once)
  static constexpr int kSlabBufs = 3;
  static constexpr uint32_t kSlabBytes = 2u * kSlab * kRowPad * 2;  // B rows, then C rows
  static constexpr uint32_t kTmemCols = 2 * BN;                     // B accumulator, then C
  static constexpr int kScanWarps = (N + 31) / 32;
  // y partials of a slab per scan warp, double-buffered by slab parity
  static constexpr size_t kSyBytes = size_t(2) * kScanWarps * kSlab * 16;
  static constexpr size_t kFixed = 1024 + size_t(kSlabBufs) * kSlabBytes + kSyBytes + 256;
  // as many ring stages as fit, at most 4
  static constexpr int kStages =
      (kSmemMax - kFixed) / kStageBytes >= 4 ? 4 : int((kSmemMax - kFixed) / kStageBytes);
  static constexpr uint32_t kIdesc = tc::idesc_bf16(BM, BN);
  static_assert(kXBytes % 1024 == 0 && kWBytes % 1024 == 0, "swizzle atoms stay aligned");
  static_assert(kStages >= 2, "shared memory holds two ring stages at least");
};

template <int S>
struct Ctl {
  uint64_t full[S], empty[S];
  uint64_t accum_full, accum_empty;
  uint64_t slab_full[3];
  uint64_t ydone;  // scan warp 1 has written its y partials of a slab
  uint64_t yread;  // scan warp 0 has combined them
  uint32_t tmem_base;
  int abort;
  int scan_done[2];  // slabs finished by each scan warp
};

// Bounded wait that sleeps between polls: for the copy warps, whose waits are
// long (a whole tile of MMAs) and share sub-partitions with the scan warps, so
// that their polling does not take the scan's issue slots.
__device__ __forceinline__ bool wait_sleepy(uint64_t* bar, uint32_t parity,
                                            volatile int* abort_flag, int* status,
                                            long long limit) {
  for (long long i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort_flag) return false;
    __nanosleep(64);
  }
  *abort_flag = 1;
  report_status(status, MQC_DEVICE_STATUS_TIMEOUT);
  return false;
}

template <int N, int BK>
constexpr size_t smem_bytes() {
  using C = Cfg<N, BK>;
  return 1024 + size_t(C::kStages) * C::kStageBytes + size_t(C::kSlabBufs) * C::kSlabBytes +
         C::kSyBytes + sizeof(Ctl<C::kStages>);
}

struct Params {
  const void* delta;   // [B, T, D] (TY)
  const void* s;       // [B, T, D] (TY): the real signal, S = (s, 0, 0, 0)
  const float* lam;    // [D, N, 4]
  const float* dskip;  // skip weight of channel d at dskip[d * dsd]
  int64_t dsd;
  const float* h0;  // [B, D, N, 4] or null
  float* hT;        // [B, D, N, 4] or null
  void* y;          // [B, T, D, 4] (TY)
  int B, T, D, K;
  float eps;
  int* status;
  long long wait_limit;
};

template <int N, int BK, typename TY>
__global__ void __launch_bounds__(kThreads, 1)
    bc_proj_scan_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmWB,
                        const __grid_constant__ CUtensorMap tmWC, const Params p) {
  using C = Cfg<N, BK>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // slab buffer j: B rows at slabs + j * kSlabBytes, C rows kSlab rows later
  unsigned char* slabs = base + size_t(S) * C::kStageBytes;
  float4* sy = reinterpret_cast<float4*>(slabs + size_t(C::kSlabBufs) * C::kSlabBytes);
  Ctl<S>* ctl = reinterpret_cast<Ctl<S>*>(reinterpret_cast<unsigned char*>(sy) + C::kSyBytes);
  volatile int* abort_flag = &ctl->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x, d = blockIdx.y;
  const int T = p.T;
  const int ntiles = (T + BM - 1) / BM;
  const int nkb = p.K / BK;
  const long long lim = p.wait_limit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    mbar_init(&ctl->accum_full, 1);
    mbar_init(&ctl->accum_empty, 4);
    for (int j = 0; j < C::kSlabBufs; ++j) mbar_init(&ctl->slab_full[j], 1);
    mbar_init(&ctl->ydone, 1);
    mbar_init(&ctl->yread, 1);
    ctl->abort = 0;
    ctl->scan_done[0] = ctl->scan_done[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(&ctl->tmem_base, C::kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      const int total = ntiles * nkb;
      int issued = 0;
      for (int g = 0; g < total; ++g) {
        const int s = g % S;
        if (g >= S && !tc::wait_or_abort(&ctl->empty[s], uint32_t(((g / S) - 1) & 1), abort_flag,
                                         p.status, lim))
          break;
        if (*abort_flag) break;
        const int i = g / nkb, kb = g - i * nkb;
        unsigned char* st = base + size_t(s) * C::kStageBytes;
        mbar_arrive_expect_tx(&ctl->full[s], C::kStageBytes);
        // rows past the batch row's end (last tile) are the next row's or, at
        // the end of the tensor, zero-filled: computed, never read by the scan
        tc::tma_load_2d(st, &tmX, kb * BK, b * T + i * BM, &ctl->full[s]);
        tc::tma_load_2d(st + C::kXBytes, &tmWB, kb * BK, d * C::BN, &ctl->full[s]);
        tc::tma_load_2d(st + C::kXBytes + C::kWBytes, &tmWC, kb * BK, d * C::BN, &ctl->full[s]);
        issued = g + 1;
      }
      // the CTA must outlive its copies: wait (bounded) for the last ones issued
      for (int g = issued > S ? issued - S : 0; g < issued; ++g)
        mbar_wait_bounded(&ctl->full[g % S], uint32_t((g / S) & 1), kDrainPollLimit);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int i = 0; i < ntiles && ok; ++i) {
        if (i > 0)
          ok = tc::wait_or_abort(&ctl->accum_empty, uint32_t((i - 1) & 1), abort_flag, p.status,
                                 lim);
        if (!ok) break;
        tc::tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = g % S;
          ok = tc::wait_or_abort(&ctl->full[s], uint32_t((g / S) & 1), abort_flag, p.status, lim);
          if (!ok) break;
          tc::tc_fence_after();
          const uint32_t sx = smem_addr(base + size_t(s) * C::kStageBytes);
          const uint32_t sb = sx + C::kXBytes, sc = sb + C::kWBytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {  // 16 bf16 = 32 bytes along K per MMA
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            const uint64_t ad = tc::kmajor_desc<C::kRowBytes>(sx + 32 * k);
            tc::mma_bf16<C::kIdesc>(tmem, ad, tc::kmajor_desc<C::kRowBytes>(sb + 32 * k), acc);
            tc::mma_bf16<C::kIdesc>(tmem + uint32_t(C::BN), ad,
                                    tc::kmajor_desc<C::kRowBytes>(sc + 32 * k), acc);
          }
          tc::mma_commit(&ctl->empty[s]);  // frees the stage once these MMAs have read it
          ++g;
        }
        if (ok) tc::mma_commit(&ctl->accum_full);
      }
      // aborted: the MMAs already issued must finish before the memory is freed
      if (!ok && g > 0)
        mbar_wait_bounded(&ctl->empty[(g - 1) % S], uint32_t(((g - 1) / S) & 1), kDrainPollLimit);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- copy warps
    const int q = warp & 3;  // lanes 32 q .. 32 q + 31: time steps of slab q
    const uint32_t trow = tmem + (uint32_t(32 * q) << 16);
    volatile int* scan_done = ctl->scan_done;
    for (int i = 0; i < ntiles; ++i) {
      const int k = 4 * i + q;  // slab number
      const int buf = k % C::kSlabBufs;
      bool ok = wait_sleepy(&ctl->accum_full, uint32_t(i & 1), abort_flag, p.status, lim);
      // buffer `buf` is free once the scan has finished slab k - kSlabBufs
      if (ok && k >= C::kSlabBufs) {
        const int need = k - C::kSlabBufs + 1;
        long long it = 0;
        while (scan_done[0] < need || (C::kScanWarps == 2 && scan_done[1] < need)) {
          if (++it >= lim || ((it & 63) == 0 && *abort_flag)) {
            ok = false;
            break;
          }
          __nanosleep(64);
        }
        if (!ok && it >= lim) {
          *abort_flag = 1;
          report_status(p.status, MQC_DEVICE_STATUS_TIMEOUT);
        }
        __threadfence_block();
      }
      if (!__all_sync(kFull, ok)) break;
      tc::tc_fence_after();
      uint4* rowB = reinterpret_cast<uint4*>(slabs + size_t(buf) * C::kSlabBytes) +
                    lane * (C::kRowPad / 8);
      uint4* rowC = rowB + kSlab * (C::kRowPad / 8);
#pragma unroll 1
      for (int cb = 0; cb < 2 * C::BN / 32; cb += 2) {  // two 32-column loads in flight
        uint32_t r0[32], r1[32];
        tc::tmem_ld32_async(trow + uint32_t(cb * 32), r0);
        tc::tmem_ld32_async(trow + uint32_t(cb * 32 + 32), r1);
        tc::tmem_wait_ld(r0);
        tc::tmem_wait_ld(r1);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const uint32_t* r = h2 ? r1 : r0;
          const int col = (cb + h2) * 32;
          uint4* dst = col < C::BN ? rowB + col / 8 : rowC + (col - C::BN) / 8;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_uint4(
                tc::pack_bf16x2(__uint_as_float(r[8 * j]), __uint_as_float(r[8 * j + 1])),
                tc::pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3])),
                tc::pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5])),
                tc::pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7])));
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive_plain(&ctl->slab_full[buf]);
        tc::mbar_arrive_plain(&ctl->accum_empty);
      }
    }
  } else if (warp - 6 < C::kScanWarps) {
    // ---------------------------------------------------------- scan warps
    const int sw = warp - 6;
    const int n = 32 * sw + lane;
    const bool act = n < N;
    LamConst lc{0.f, 0.f, 0.f, 0.f, 0.f};
    float4 h = f4_zero();
    if (act) {
      lc = make_lam_const(QIO<float>::ld(p.lam + (int64_t(d) * N + n) * 4));
      if (p.h0 != nullptr) h = QIO<float>::ld(p.h0 + ((int64_t(b) * p.D + d) * N + n) * 4);
    }
    const float dsk = __ldg(p.dskip + int64_t(d) * p.dsd);
    const TY* gdelta = static_cast<const TY*>(p.delta);
    const TY* gs = static_cast<const TY*>(p.s);
    TY* gy = static_cast<TY*>(p.y);
    const float eps = p.eps;
    // lanes past d_state read state 0's rows (always inside the slab buffer) and
    // inject nothing: their state stays zero and their readout with it
    const int noff = 4 * (act ? n : 0);
    const float amask = act ? 1.f : 0.f;
    float* syf = reinterpret_cast<float*>(sy);
    // delta and s of a slab's steps (lane j holds step t0 + j), loaded a slab ahead
    auto load_ds = [&](int t0, float& dl_v, float& s_v) {
      dl_v = 0.f;
      s_v = 0.f;
      if (t0 + lane < T) {
        const int64_t row = (int64_t(b) * T + t0 + lane) * p.D + d;
        dl_v = to_f(gdelta[row]);
        s_v = to_f(gs[row]);
      }
    };
    float dl_n, s_n;
    load_ds(0, dl_n, s_n);
    bool ok = true;
    const int nslabs = 4 * ntiles;
    for (int k = 0; k < nslabs; ++k) {
      const int buf = k % C::kSlabBufs;
      ok = tc::wait_or_abort(&ctl->slab_full[buf], uint32_t((k / C::kSlabBufs) & 1), abort_flag,
                             p.status, lim);
      if (!__all_sync(kFull, ok)) {
        ok = false;
        break;
      }
      const int t0 = k * kSlab;
      const int nst = max(0, min(kSlab, T - t0));
      const float dl_l = dl_n, s_l = s_n;
      load_ds(t0 + kSlab, dl_n, s_n);
      // y partials of this slab: sy[k & 1][sw][step]. Warp 1 starts slab k only
      // once warp 0 has combined slab k - 1, so it is never more than one slab
      // ahead: its ydone arrivals and warp 0's yread arrivals then stay within
      // one phase of the other warp's wait (no parity aliasing).
      float* syk = syf + size_t(k & 1) * C::kScanWarps * kSlab * 4;
      if constexpr (C::kScanWarps == 2) {
        if (sw == 1 && k >= 1) {
          ok = tc::wait_or_abort(&ctl->yread, uint32_t((k - 1) & 1), abort_flag, p.status, lim);
          if (!__all_sync(kFull, ok)) {
            ok = false;
            break;
          }
        }
      }
      const __nv_bfloat16* pB =
          reinterpret_cast<const __nv_bfloat16*>(slabs + size_t(buf) * C::kSlabBytes) + noff;
      const __nv_bfloat16* pC = pB + kSlab * C::kRowPad;
      // four steps at a time: their readouts are reduced over the warp's states
      // together (16 sums, 16 shuffles), off the state's critical path
      for (int tt0 = 0; tt0 < nst; tt0 += 4) {
        float v[16];
        if (tt0 + 4 <= nst) {
          // a full group, in phases so that the four steps' shuffles, loads and
          // Cayley maps are all in flight before the state chain needs them
          float dlv[4], svv[4];
          float4 Bv[4], Cv[4], qv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            dlv[u] = __shfl_sync(kFull, dl_l, tt0 + u);
            svv[u] = __shfl_sync(kFull, s_l, tt0 + u) * amask;
            Bv[u] = QIO<__nv_bfloat16>::lds(pB + (tt0 + u) * C::kRowPad);
            Cv[u] = QIO<__nv_bfloat16>::lds(pC + (tt0 + u) * C::kRowPad);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) qv[u] = cayley_from_const(dlv[u], dlv[u] * dlv[u], lc, eps);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            h = qmul_acc(qv[u], h, make_float4(svv[u] * Bv[u].x, svv[u] * Bv[u].y,
                                               svv[u] * Bv[u].z, svv[u] * Bv[u].w));
            const float4 ya = qmul(Cv[u], h);
            v[4 * u] = ya.x;
            v[4 * u + 1] = ya.y;
            v[4 * u + 2] = ya.z;
            v[4 * u + 3] = ya.w;
          }
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) {  // the sequence's last, partial group
            const int tt = tt0 + u;
            const bool live = tt < nst;
            const float dl = __shfl_sync(kFull, dl_l, tt & 31);
            const float sv = __shfl_sync(kFull, s_l, tt & 31) * amask;
            const float4 Bv = QIO<__nv_bfloat16>::lds(pB + (tt & 31) * C::kRowPad);
            const float4 Cv = live ? QIO<__nv_bfloat16>::lds(pC + (tt & 31) * C::kRowPad)
                                   : f4_zero();
            const float4 qv = cayley_from_const(dl, dl * dl, lc, eps);
            const float4 hn =
                qmul_acc(qv, h, make_float4(sv * Bv.x, sv * Bv.y, sv * Bv.z, sv * Bv.w));
            if (live) h = hn;
            const float4 ya = qmul(Cv, h);  // zero for steps past the end
            v[4 * u] = ya.x;
            v[4 * u + 1] = ya.y;
            v[4 * u + 2] = ya.z;
            v[4 * u + 3] = ya.w;
          }
        }
        // reduce-scatter of the 16 values over the 32 lanes: afterwards lanes
        // 2m and 2m + 1 hold sum m = 4 (step) + (component)
        float w8[8], w4[4], w2[2];
        const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          w8[j] = (b4 ? v[8 + j] : v[j]) + __shfl_xor_sync(kFull, b4 ? v[j] : v[8 + j], 16);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w4[j] = (b3 ? w8[4 + j] : w8[j]) + __shfl_xor_sync(kFull, b3 ? w8[j] : w8[4 + j], 8);
#pragma unroll
        for (int j = 0; j < 2; ++j)
          w2[j] = (b2 ? w4[2 + j] : w4[j]) + __shfl_xor_sync(kFull, b2 ? w4[j] : w4[2 + j], 4);
        float r = (b1 ? w2[1] : w2[0]) + __shfl_xor_sync(kFull, b1 ? w2[0] : w2[1], 2);
        r += __shfl_xor_sync(kFull, r, 1);
        const int m = (lane >> 1) & 15;
        if (!(lane & 1) && tt0 + (m >> 2) < nst) syk[(sw * kSlab + tt0 + (m >> 2)) * 4 + (m & 3)] = r;
      }
      __syncwarp();
      if constexpr (C::kScanWarps == 2) {
        if (sw == 1) {
          if (lane == 0) tc::mbar_arrive_plain(&ctl->ydone);
        } else {
          ok = tc::wait_or_abort(&ctl->ydone, uint32_t(k & 1), abort_flag, p.status, lim);
          if (!__all_sync(kFull, ok)) {
            ok = false;
            break;
          }
        }
      }
      if (sw == 0 && lane < nst) {
        const float4* syk4 = reinterpret_cast<const float4*>(syk);
        float4 yv = syk4[lane];
        if constexpr (C::kScanWarps == 2) {
          const float4 y2 = syk4[kSlab + lane];
          yv.x += y2.x;
          yv.y += y2.y;
          yv.z += y2.z;
          yv.w += y2.w;
        }
        yv.x = fmaf(dsk, s_l, yv.x);
        QIO<TY>::st(gy + ((int64_t(b) * T + t0 + lane) * p.D + d) * 4, yv);
      }
      __syncwarp();
      // this warp is done with the slab buffer (and warp 0 with the y partials)
      if (lane == 0) {
        if (C::kScanWarps == 2 && sw == 0) tc::mbar_arrive_plain(&ctl->yread);
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&ctl->scan_done[sw]) = k + 1;
      }
    }
    if (ok && act && p.hT != nullptr)
      QIO<float>::st(p.hT + ((int64_t(b) * p.D + d) * N + n) * 4, h);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int N, int BK, typename TY>
int launch(const mqc_bc_proj_scan_args* a, cudaStream_t st, const char* name) {
  using C = Cfg<N, BK>;
  const uint64_t rows = uint64_t(a->batch) * uint64_t(a->seq_len);
  const uint64_t wrows = uint64_t(a->channels) * uint64_t(C::BN);
  CUtensorMap tmX, tmWB, tmWC;
  int rc = make_map_bf16_2d(&tmX, a->x, rows, uint64_t(a->in_features), BM, BK, C::kRowBytes,
                            name);
  if (rc == MQC_OK)
    rc = make_map_bf16_2d(&tmWB, a->w_b, wrows, uint64_t(a->in_features), C::BN, BK,
                          C::kRowBytes, name);
  if (rc == MQC_OK)
    rc = make_map_bf16_2d(&tmWC, a->w_c, wrows, uint64_t(a->in_features), C::BN, BK,
                          C::kRowBytes, name);
  if (rc != MQC_OK) return rc;
  constexpr size_t smem = smem_bytes<N, BK>();
  static_assert(smem <= 227 * 1024, "shared memory of one CTA");
  auto kern = bc_proj_scan_kernel<N, BK, TY>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "%s: smem attribute (%zu B): %s", name, smem, cudaGetErrorString(e));
  Params p{};
  p.delta = a->delta;
  p.s = a->s;
  p.lam = a->lambda_;
  p.dskip = a->dskip;
  p.dsd = a->dskip_sd;
  p.h0 = a->h0;
  p.hT = a->hT;
  p.y = a->y;
  p.B = int(a->batch);
  p.T = int(a->seq_len);
  p.D = int(a->channels);
  p.K = int(a->in_features);
  p.eps = a->eps;
  p.status = a->status;
  p.wait_limit = a->wait_poll_limit < 0 ? (1ll << 26) : a->wait_poll_limit;
  dim3 grid{unsigned(a->batch), unsigned(a->channels), 1u};
  kern<<<grid, kThreads, smem, st>>>(tmX, tmWB, tmWC, p);
  return check_launch(name);
}

template <int N>
int dispatch_n(const mqc_bc_proj_scan_args* a, cudaStream_t st, const char* name) {
  // K blocks of 32 (64-byte swizzle rows): the ring stages stay small enough for
  // three slab buffers beside them
  return a->dtype == MQC_DTYPE_F32 ? launch<N, 32, float>(a, st, name)
                                   : launch<N, 32, __nv_bfloat16>(a, st, name);
}

}  // namespace
}  // namespace bcscan
}  // namespace mqc

using namespace mqc;

extern "C" int mqc_bc_proj_scan_fwd(const mqc_bc_proj_scan_args* a, void* stream) {
  clear_error();
  const char* name = "mqc_bc_proj_scan_fwd";
  MQC_REQUIRE(a != nullptr, MQC_ERR_INVALID_VALUE, "%s: null args", name);
  MQC_REQUIRE(dtype_ok(a->dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name,
              int(a->dtype));
  MQC_REQUIRE(a->batch >= 0 && a->seq_len >= 0 && a->channels >= 0 && a->in_features >= 0,
              MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(a->d_state == 16 || a->d_state == 32 || a->d_state == 64, MQC_ERR_UNSUPPORTED,
              "%s: d_state must be 16, 32 or 64 (got %lld)", name, (long long)a->d_state);
  if (a->batch == 0 || a->seq_len == 0 || a->channels == 0) return MQC_OK;
  MQC_REQUIRE(a->in_features >= 64 && a->in_features % 64 == 0 && a->in_features <= (1 << 20),
              MQC_ERR_UNSUPPORTED, "%s: in_features must be a positive multiple of 64 (got %lld)",
              name, (long long)a->in_features);
  MQC_REQUIRE(a->x && a->w_b && a->w_c && a->delta && a->s && a->lambda_ && a->dskip && a->y,
              MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  MQC_REQUIRE(a->batch * a->seq_len <= 0x7fffffffll - 128 && a->channels <= 65535 &&
                  a->batch <= 0x7fffffffll && a->channels * a->d_state * 4 <= 0x7fffffffll,
              MQC_ERR_UNSUPPORTED, "%s: size out of range", name);
  MQC_REQUIRE(aligned(a->x, 16) && aligned(a->w_b, 16) && aligned(a->w_c, 16) &&
                  aligned(a->lambda_, 16) && aligned(a->y, a->dtype == MQC_DTYPE_F32 ? 16 : 8) &&
                  (a->h0 == nullptr || aligned(a->h0, 16)) &&
                  (a->hT == nullptr || aligned(a->hT, 16)),
              MQC_ERR_MISALIGNED, "%s: misaligned pointer", name);
  cudaStream_t st = as_stream(stream);
  switch (a->d_state) {
    case 16: return bcscan::dispatch_n<16>(a, st, name);
    case 32: return bcscan::dispatch_n<32>(a, st, name);
    default: return bcscan::dispatch_n<64>(a, st, name);
  }
}
