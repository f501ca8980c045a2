// Fused Cayley + quaternion selective scan, forward, for B/C shared by all
// channels ([B,T,N,4]; the layout of the hot-path configuration), with packed
// FP32 arithmetic.
//
// Same math as ssm_scan_fwd.cu (QuaternionMamba2Block._ssm_forward,
// mambaqc/models/quaternion_mamba2_block.py:214-228, without materialising z or
// q). The kernel is instruction-issue bound (about 47 FP32 operations per
// (b,t,d,n) element and little memory traffic), so it issues its FP32 work as
// sm_100 packed two-lane instructions (fma/mul/add .rn.f32x2): every lane keeps
// its G states as G/2 pairs (n, n + NG) and runs both halves of a pair through
// one packed instruction. A packed FMA takes a negated half or a broadcast
// scalar operand at no cost, so the Cayley map, the state update
// h = q (x) h + B (x) S and the readout C (x) h all map onto packed
// instructions without any register shuffling, provided the B/C rows present
// the two states of a pair side by side. Hence:
//
//  * a small pre-pass (`pack_bc_kernel`) rewrites B and C once per call into
//    fp32 rows of NP = NG*G states ordered [pair j][part][lane ng][4 floats]
//    (part 0: components x, y of both halves; part 1: z, w), so the 16-byte
//    loads of the NG lanes of a channel cover one contiguous 128-byte line (no
//    shared-memory bank conflicts),
//    state n = ng + NG*(2j + half), zero-padded above N (bf16 inputs are
//    widened here, so the scan never converts B/C);
//  * warp 0 is the producer: one lane streams tc packed rows of B and C per
//    chunk into a kRing-deep shared-memory ring with one bulk copy each (TMA
//    engine), signalling `full[stage]` by transaction bytes and waiting on
//    `empty[stage]` before it reuses a stage;
//  * every other warp is a consumer that owns 32/NG channels x NP states; it
//    stages its own channels' delta and x (or S) one chunk ahead into a
//    warp-private buffer, waits on `full`, runs the chunk and releases the stage
//    with one arrive on `empty`;
//  * the per-step readout sum over n runs in packed accumulators (even / odd
//    states in the two halves), then a shuffle reduce-scatter over the NG lanes
//    of a channel.
//
// Each half of a packed instruction rounds exactly like the scalar instruction,
// and the operation order per state and the readout summation order (even
// states, odd states, then their sum) are those of the scalar formulation, so
// the results are bitwise those of an unpacked kernel.
//
// All waits are bounded (poll limit); on timeout the kernel reports
// MQC_DEVICE_STATUS_TIMEOUT, raises a shared abort flag so the other warps stop
// at their next chunk, and the producer drains its copies in flight before it
// exits.
#include <cstdlib>
#include <type_traits>

#include "packed_math.cuh"
#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {
namespace {

using namespace ::mqc::pk;

constexpr int kRing = 3;
// CTA size cap: 8 states per lane run at ~160 registers per thread, which the
// register file holds for 3 warps per sub-partition (384 threads); capped at 512
// threads (128 registers) the kernel ran 3 % slower.
// (4 states per lane with twice the warps measured slower on config 3.)
__host__ __device__ constexpr int pk_max_threads(int g) { return g == 4 ? 768 : 384; }
constexpr size_t kPkSmemBudget = 220 * 1024;
constexpr int kPackThreads = 256;

// Predicated scalar store without a branch (no divergence / reconvergence code
// in the time loop).
__device__ __forceinline__ void st1_pred(float* p, float v, bool pred) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.global.f32 [%0], %1;\n\t}" ::"l"(p),
               "f"(v), "r"(unsigned(pred))
               : "memory");
}
__device__ __forceinline__ void st1_pred(__nv_bfloat16* p, float v, bool pred) {
  const unsigned short h = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.global.b16 [%0], %1;\n\t}" ::"l"(p),
               "h"(h), "r"(unsigned(pred))
               : "memory");
}

// One multimem store of a y quaternion to a multicast address: NVSwitch writes
// it into the buffer of every rank bound to the multicast object.
__device__ __forceinline__ void mc_store_q(float* p, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_store_q(__nv_bfloat16* p, float4 v) {
  const uint2 u = QIO<__nv_bfloat16>::pack(v);
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(p), "r"(u.x),
               "r"(u.y)
               : "memory");
}

// reduce_store_y (ssm_scan_common.cuh) with predicated stores: sums the partial
// readouts `a` over the NG lanes of a channel (reduce-scatter: afterwards lane ng
// holds component ng & 3), adds dsk * s and stores y[t, c, 0..3].
template <typename T, int NG>
__device__ __forceinline__ void reduce_store_y_pk(float4 a, float4 sv, float dsk, int ng,
                                                  bool active, T* yp) {
  constexpr unsigned kFull = 0xffffffffu;
  if constexpr (NG == 1) {
    st1_pred(yp + 0, fmaf(dsk, sv.x, a.x), active);
    st1_pred(yp + 1, fmaf(dsk, sv.y, a.y), active);
    st1_pred(yp + 2, fmaf(dsk, sv.z, a.z), active);
    st1_pred(yp + 3, fmaf(dsk, sv.w, a.w), active);
  } else {
    const bool odd = ng & 1;
    const float s0 = odd ? a.x : a.y;
    const float s1 = odd ? a.z : a.w;
    const float r0 = __shfl_xor_sync(kFull, s0, 1);
    const float r1 = __shfl_xor_sync(kFull, s1, 1);
    const float k0 = (odd ? a.y : a.x) + r0;  // component (odd)
    const float k1 = (odd ? a.w : a.z) + r1;  // component (odd + 2)
    if constexpr (NG == 2) {
      const int c0 = odd ? 1 : 0;
      st1_pred(yp + c0, fmaf(dsk, f4_get(sv, c0), k0), active);
      st1_pred(yp + c0 + 2, fmaf(dsk, f4_get(sv, c0 + 2), k1), active);
    } else {
      const bool hi = (ng >> 1) & 1;
      const float snd = hi ? k0 : k1;
      const float r = __shfl_xor_sync(kFull, snd, 2);
      float v = (hi ? k1 : k0) + r;
#pragma unroll
      for (int m = 4; m < NG; m <<= 1) v += __shfl_xor_sync(kFull, v, m);
      const int comp = ng & 3;
      st1_pred(yp + comp, fmaf(dsk, f4_get(sv, comp), v), active && ng < 4);
    }
  }
}

// The reduction of reduce_store_y_pk with the store left to `store(comp, value,
// pred)` (the peer-output form writes every value to several buffers).
template <int NG, typename Store>
__device__ __forceinline__ void reduce_y_pk(float4 a, float4 sv, float dsk, int ng, bool active,
                                            Store&& store) {
  constexpr unsigned kFull = 0xffffffffu;
  if constexpr (NG == 1) {
    store(0, fmaf(dsk, sv.x, a.x), active);
    store(1, fmaf(dsk, sv.y, a.y), active);
    store(2, fmaf(dsk, sv.z, a.z), active);
    store(3, fmaf(dsk, sv.w, a.w), active);
  } else {
    const bool odd = ng & 1;
    const float s0 = odd ? a.x : a.y;
    const float s1 = odd ? a.z : a.w;
    const float r0 = __shfl_xor_sync(kFull, s0, 1);
    const float r1 = __shfl_xor_sync(kFull, s1, 1);
    const float k0 = (odd ? a.y : a.x) + r0;
    const float k1 = (odd ? a.w : a.z) + r1;
    if constexpr (NG == 2) {
      const int c0 = odd ? 1 : 0;
      store(c0, fmaf(dsk, f4_get(sv, c0), k0), active);
      store(c0 + 2, fmaf(dsk, f4_get(sv, c0 + 2), k1), active);
    } else {
      const bool hi = (ng >> 1) & 1;
      const float snd = hi ? k0 : k1;
      const float r = __shfl_xor_sync(kFull, snd, 2);
      float v = (hi ? k1 : k0) + r;
#pragma unroll
      for (int m = 4; m < NG; m <<= 1) v += __shfl_xor_sync(kFull, v, m);
      const int comp = ng & 3;
      store(comp, fmaf(dsk, f4_get(sv, comp), v), active && ng < 4);
    }
  }
}

// Bounded wait for a thread off the critical path (the producer, which runs
// chunks ahead of the consumers): sleeps between polls so that its polling
// does not take issue slots from the consumer warps on its sub-partition.
__device__ __forceinline__ bool mbar_wait_bounded_backoff(uint64_t* bar, uint32_t parity,
                                                          long long limit) {
  for (long long i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(200);
  }
  return false;
}

// ------------------------------------------------------------ B/C pre-pass
// One thread per (row, pair j, lane ng): reads states n0 = ng + 2*NG*j and
// n1 = n0 + NG of B and C and writes their 8 interleaved floats as two 16-byte
// parts, [x0 x1 y0 y1] and [z0 z1 w0 w1], NG*16 bytes apart: a row is
// [pair j][part][lane ng][4]. Rows are the B*T (b, t) rows; output rows hold
// np = NG*G states (np*4 floats).
template <typename T>
__global__ void __launch_bounds__(kPackThreads)
    pack_bc_kernel(const T* __restrict__ Bm, const T* __restrict__ Cm, float* __restrict__ Bp,
                   float* __restrict__ Cp, int64_t rows, int N, int ng_log2, int pairs) {
  const int NG = 1 << ng_log2;
  const int64_t per_row = int64_t(pairs) << ng_log2;
  const int64_t total = rows * per_row;
  for (int64_t idx = int64_t(blockIdx.x) * kPackThreads + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * kPackThreads) {
    const int64_t row = idx / per_row;
    const int r = int(idx - row * per_row);
    const int j = r >> ng_log2, ng = r & (NG - 1);
    const int n0 = ng + 2 * NG * j, n1 = n0 + NG;
    const int64_t base = row * N;
    const float4 b0 = n0 < N ? QIO<T>::ld(Bm + (base + n0) * 4) : f4_zero();
    const float4 b1 = n1 < N ? QIO<T>::ld(Bm + (base + n1) * 4) : f4_zero();
    const int64_t o0 = (row * per_row * 2 + (int64_t(j) << ng_log2) * 2 + ng) * 4;
    float4* ob = reinterpret_cast<float4*>(Bp + o0);
    ob[0] = make_float4(b0.x, b1.x, b0.y, b1.y);
    ob[NG] = make_float4(b0.z, b1.z, b0.w, b1.w);
    if (Cm != nullptr) {  // C is not needed by the state-only pass
      const float4 c0 = n0 < N ? QIO<T>::ld(Cm + (base + n0) * 4) : f4_zero();
      const float4 c1 = n1 < N ? QIO<T>::ld(Cm + (base + n1) * 4) : f4_zero();
      float4* oc = reinterpret_cast<float4*>(Cp + o0);
      oc[0] = make_float4(c0.x, c1.x, c0.y, c1.y);
      oc[NG] = make_float4(c0.z, c1.z, c0.w, c1.w);
    }
  }
}

// bf16 -> fp32 for delta and S (the scan stages fp32 with cp.async). VEC: both
// pointers 16-byte aligned and n a multiple of 8 (8 elements per iteration).
template <bool VEC>
__global__ void __launch_bounds__(kPackThreads)
    widen_bf16_kernel(const __nv_bfloat16* __restrict__ in, float* __restrict__ out, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * kPackThreads;
  if constexpr (VEC) {
    for (int64_t i = int64_t(blockIdx.x) * kPackThreads + threadIdx.x; i < n / 8; i += stride) {
      const uint4 v = reinterpret_cast<const uint4*>(in)[i];
      float4* o = reinterpret_cast<float4*>(out) + 2 * i;
      o[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                         __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
      o[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u),
                         __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xffff0000u));
    }
  } else {
    for (int64_t i = int64_t(blockIdx.x) * kPackThreads + threadIdx.x; i < n; i += stride)
      out[i] = __bfloat162float(in[i]);
  }
}

int launch_widen(const void* in, float* out, int64_t n, cudaStream_t st) {
  const bool vec = aligned(in, 16) && aligned(out, 16) && n % 8 == 0;
  const int64_t work = vec ? n / 8 : n;
  const int64_t want = (work + kPackThreads - 1) / kPackThreads;
  const int grid = int(want < int64_t(num_sms()) * 16 ? (want > 0 ? want : 1) : int64_t(num_sms()) * 16);
  const auto* src = static_cast<const __nv_bfloat16*>(in);
  if (vec) widen_bf16_kernel<true><<<grid, kPackThreads, 0, st>>>(src, out, n);
  else widen_bf16_kernel<false><<<grid, kPackThreads, 0, st>>>(src, out, n);
  return check_launch("mqc_ssm_scan_fwd(widen)");
}

// ------------------------------------------------------------ scan kernel
struct PkLayout {
  size_t off_b, off_c, off_dx, off_sx, total;
};

// [full x kRing][empty x kRing][abort flag] | sB [kRing][tc][np*4] f32 | sC |
// per consumer warp: delta [2][tc][cpw] f32 | s [2][tc][cpw][sw] f32
__host__ __device__ inline PkLayout pk_layout(int tc, int np, int warps, int cpw, int sw) {
  PkLayout L;
  size_t off = 128;
  const size_t ring = size_t(kRing) * tc * np * 4 * sizeof(float);
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

// p.Bm / p.Cm point at the packed rows and p.delta / p.s at fp32 data here; T is
// the type of y. CKPT: p.ckpt is set (the forward of a training step stores
// states for the backward). DT: the skip weight varies over time (p.dst != 0).
// SO (state only, pass 1 of the time-chunked scan): no readout and no C; the
// kernel writes the final state to p.hT and the product of the step operators
// P = q_{T-1} (x) ... (x) q_0 to p.pout. All q_t of a lane lie in the plane
// span{1, u}, u = Im Lambda / |Im Lambda|, where quaternions commute and
// multiply like complex numbers, so P is kept as (Pa, Pb) with P = Pa + Pb u:
// 4 operations per step instead of a 16-term Hamilton product.
// PEER (channel-sharded scan, not with CKPT, DT or SO): y is written into the
// p.npeer output buffers p.ypeer[r] -- this GPU's and the other ranks' (peer
// memory over NVLink) -- at this shard's channel columns, so the exchange of y
// between the ranks happens in the scan's own stores, tile by tile.
template <typename T, int G, int NG, bool S_REAL, bool CKPT, bool DT, bool SO, bool PEER = false>
__global__ void __launch_bounds__(pk_max_threads(G), 1)
    scan_fwd_packed_kernel(const FwdParams p) {
  static_assert(G % 2 == 0, "states are processed in pairs");
  constexpr int G2 = G / 2;
  constexpr int NP = NG * G;
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

  const PkLayout L = pk_layout(tc, NP, nwarps_c, CPW, SW);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + kRing;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kRing);
  float* sB = reinterpret_cast<float*>(smem_raw + L.off_b);
  float* sC = reinterpret_cast<float*>(smem_raw + L.off_c);

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
      const float* gB = static_cast<const float*>(p.Bm);
      const float* gC = static_cast<const float*>(p.Cm);
      constexpr uint32_t row_bytes = uint32_t(NP) * 4 * sizeof(float);
      int issued = 0;
      bool ok = true;
      for (int k = 0; k < nchunks; ++k) {
        const int st = k % kRing;
        if (k >= kRing) {
          ok = mbar_wait_bounded_backoff(&empty[st], uint32_t(((k / kRing) - 1) & 1),
                                         p.wait_limit);
          if (!ok) break;
        }
        if (*abort_flag) break;
        const int t0 = k * tc;
        const int len = min(tc, T_ - t0);
        const uint32_t bytes = uint32_t(len) * row_bytes;
        mbar_arrive_expect_tx(&full[st], (SO ? 1u : 2u) * bytes);
        const int64_t g0 = (int64_t(b) * T_ + t0) * NP * 4;
        bulk_g2s(sB + int64_t(st) * tc * NP * 4, gB + g0, bytes, &full[st]);
        if (!SO) bulk_g2s(sC + int64_t(st) * tc * NP * 4, gC + g0, bytes, &full[st]);
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

  QPair h[G2];
  LamPair lc[G2];
#pragma unroll
  for (int j = 0; j < G2; ++j) {
    h[j] = qp_zero();
    LamConst k2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = ng + NG * (2 * j + e);
      k2[e] = LamConst{0.f, 0.f, 0.f, 0.f, 0.f};
      if (active && n < N) {
        if (p.h0 != nullptr)
          qp_set_half(h[j], e, QIO<float>::ld(p.h0 + ((int64_t(b) * D + c) * N + n) * 4));
        k2[e] = make_lam_const(QIO<float>::ld(p.lam + (int64_t(c) * N + n) * 4));
      }
    }
    lc[j] = LamPair{make_float2(k2[0].lr, k2[1].lr), make_float2(k2[0].li, k2[1].li),
                    make_float2(k2[0].lj, k2[1].lj), make_float2(k2[0].lk, k2[1].lk),
                    make_float2(k2[0].m, k2[1].m)};
  }
  // SO: |Im Lambda| per state and the operator product (Pa, Pb), P = Pa + Pb u
  float2 nim[SO ? G2 : 1], Pa[SO ? G2 : 1], Pb[SO ? G2 : 1];
  if constexpr (SO) {
#pragma unroll
    for (int j = 0; j < G2; ++j) {
      const LamPair& l = lc[j];
      nim[j] = make_float2(sqrtf(fmaf(l.li.x, l.li.x, fmaf(l.lj.x, l.lj.x, l.lk.x * l.lk.x))),
                           sqrtf(fmaf(l.li.y, l.li.y, fmaf(l.lj.y, l.lj.y, l.lk.y * l.lk.y))));
      Pa[j] = bc2(1.f);
      Pb[j] = bc2(0.f);
    }
  }
  const float dsk0 = active ? __ldg(p.dskip + int64_t(b) * p.dsb + int64_t(c) * p.dsd) : 0.f;

  // warp-private staging of delta and s: [2][tc][CPW] (+ [SW] for s)
  float* wdel = reinterpret_cast<float*>(smem_raw + L.off_dx) + int64_t(cw) * 2 * tc * CPW;
  float* wsig = reinterpret_cast<float*>(smem_raw + L.off_sx) + int64_t(cw) * 2 * tc * CPW * SW;
  // delta and s are fp32 here (bf16 inputs are widened by the pre-pass): they go
  // global -> shared with cp.async, one chunk ahead, holding no registers
  const float* gdelta = static_cast<const float*>(p.delta);
  const float* gs = static_cast<const float*>(p.s);
  const int per_chunk = tc * CPW;
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

  issue_dx_async(0, 0);
  cp_async_wait_all();
  __syncwarp();

  const float eps = p.eps;
  T* yb = (SO || PEER) ? nullptr : static_cast<T*>(p.y) + (int64_t(b) * T_ * D + c) * 4;
  // peer outputs: element offset of (b, t = 0, this channel) in every buffer
  const int64_t ypo = PEER ? int64_t(b) * T_ * p.y_ld + p.y_coff + int64_t(c) * 4 : 0;
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
    if (k + 1 < nchunks) issue_dx_async(k + 1, buf ^ 1);

    const int t0 = k * tc;
    const int len = min(tc, T_ - t0);
    const float* cdel = wdel + buf * per_chunk;
    const float* csig = wsig + buf * per_chunk * SW;
    // this lane's pair slots: [j][part][ng][4], parts [x0 x1 y0 y1], [z0 z1 w0 w1]
    const float* rowB = sB + int64_t(st) * tc * NP * 4 + ng * 4;
    const float* rowC = sC + int64_t(st) * tc * NP * 4 + ng * 4;
    // unrolled (by four: 1.58 ms against 1.61 ms by two on config 3) so the
    // loop-carried states rotate through register sets instead of being copied
    // back at every step
    T* yrow = PEER ? nullptr : yb + int64_t(t0) * D * 4;
    const int64_t ystep = PEER ? 0 : int64_t(D) * 4;
    int64_t yrow_peer = ypo + int64_t(t0) * p.y_ld;
#pragma unroll 4
    for (int tt = 0; tt < len; ++tt, yrow += ystep, yrow_peer += PEER ? p.y_ld : 0) {
      const float dl = cdel[tt * CPW + lc_ch];
      const float dl2 = dl * dl;
      float4 sv;
      if (S_REAL) sv = make_float4(csig[tt * CPW + lc_ch], 0.f, 0.f, 0.f);
      else sv = reinterpret_cast<const float4*>(csig)[tt * CPW + lc_ch];
      QPair ya = qp_zero();
#pragma unroll
      for (int j = 0; j < G2; ++j) {
        const float* pb = rowB + tt * NP * 4 + j * NG * 8;
        const float4 b01 = *reinterpret_cast<const float4*>(pb);
        const float4 b23 = *reinterpret_cast<const float4*>(pb + NG * 4);
        const QPair Bq{make_float2(b01.x, b01.y), make_float2(b01.z, b01.w),
                       make_float2(b23.x, b23.y), make_float2(b23.z, b23.w)};
        float2 sq;
        const QPair qv = cayley_pair(dl, dl2, lc[j], eps, &sq);
        QPair inj;
        if (S_REAL) {
          const float2 s2 = bc2(sv.x);
          inj = QPair{mul2(s2, Bq.x), mul2(s2, Bq.y), mul2(s2, Bq.z), mul2(s2, Bq.w)};
        } else {
          inj = qp_mul_bcast(Bq, sv);
        }
        h[j] = qp_mul_acc(qv, h[j], inj);
        if constexpr (SO) {
          // q = qa + qb u with qa = q.x, qb = (delta / den) |Im Lambda|; P <- q P
          const float2 qb = mul2(sq, nim[j]);
          const float2 pa = fma2(qv.x, Pa[j], neg2(mul2(qb, Pb[j])));
          Pb[j] = fma2(qv.x, Pb[j], mul2(qb, Pa[j]));
          Pa[j] = pa;
        } else {
          const float* pc = rowC + tt * NP * 4 + j * NG * 8;
          const float4 c01 = *reinterpret_cast<const float4*>(pc);
          const float4 c23 = *reinterpret_cast<const float4*>(pc + NG * 4);
          const QPair Cq{make_float2(c01.x, c01.y), make_float2(c01.z, c01.w),
                         make_float2(c23.x, c23.y), make_float2(c23.z, c23.w)};
          ya = qp_mul_acc(Cq, h[j], ya);
        }
      }
      if constexpr (!SO) {
        // even states + odd states, as the scalar kernel's two accumulators
        const float4 yv =
            make_float4(ya.x.x + ya.x.y, ya.y.x + ya.y.y, ya.z.x + ya.z.y, ya.w.x + ya.w.y);
        float dsk = dsk0;
        if constexpr (DT)
          dsk = (active && ng < 4) ? __ldg(p.dskip + int64_t(b) * p.dsb +
                                           int64_t(t0 + tt) * p.dst + int64_t(c) * p.dsd)
                                   : 0.f;
        if constexpr (PEER) {
          bool mc_done = false;
          if constexpr (NG >= 4) {
            if (p.peer_mc) {
              // lanes ng = 0..3 of the channel hold components 0..3 after the
              // reduction: gather them on lane 0 for one multicast store
              float mv = 0.f;
              reduce_y_pk<NG>(yv, sv, dsk, ng, active,
                              [&](int, float v, bool) { mv = v; });
              const int base = lane - ng;
              const float4 q = make_float4(__shfl_sync(kFull, mv, base),
                                           __shfl_sync(kFull, mv, base + 1),
                                           __shfl_sync(kFull, mv, base + 2),
                                           __shfl_sync(kFull, mv, base + 3));
              if (ng == 0 && active) mc_store_q(static_cast<T*>(p.ypeer[0]) + yrow_peer, q);
              mc_done = true;
            }
          }
          if (!mc_done)
            reduce_y_pk<NG>(yv, sv, dsk, ng, active, [&](int comp, float v, bool pred) {
#pragma unroll
              for (int r = 0; r < kMaxPeerOutputs; ++r)
                if (r < p.npeer) st1_pred(static_cast<T*>(p.ypeer[r]) + yrow_peer + comp, v, pred);
            });
        } else {
          reduce_store_y_pk<T, NG>(yv, sv, dsk, ng, active, yrow);
        }
      }
      if constexpr (CKPT) {
        const int t = t0 + tt;
        if (active && (t + 1) % p.ckpt_every == 0 && t + 1 < T_) {
          float* base = p.ckpt +
                        ((int64_t(b) * p.nck + (t + 1) / p.ckpt_every - 1) * D + c) * int64_t(N) * 4;
#pragma unroll
          for (int j = 0; j < G2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int n = ng + NG * (2 * j + e);
              if (n < N) QIO<float>::st(base + int64_t(n) * 4, qp_half(h[j], e));
            }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (k + 1 < nchunks) {
      cp_async_wait_all();
      __syncwarp();
    }
  }
  if (p.hT != nullptr && active) {
#pragma unroll
    for (int j = 0; j < G2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = ng + NG * (2 * j + e);
        if (n < N) QIO<float>::st(p.hT + ((int64_t(b) * D + c) * N + n) * 4, qp_half(h[j], e));
      }
  }
  // stores to peer memory: visible system-wide before the kernel is seen as
  // complete by the ranks that synchronise with it
  if constexpr (PEER) __threadfence_system();
  if constexpr (SO) {
    if (active) {
#pragma unroll
      for (int j = 0; j < G2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int n = ng + NG * (2 * j + e);
          if (n < N) {
            const float nm = e ? nim[j].y : nim[j].x;
            const float pa = e ? Pa[j].y : Pa[j].x;
            const float pbu = (nm > 0.f ? (e ? Pb[j].y : Pb[j].x) / nm : 0.f);
            const LamPair& l = lc[j];
            const float4 P4 = make_float4(pa, pbu * (e ? l.li.y : l.li.x),
                                          pbu * (e ? l.lj.y : l.lj.x), pbu * (e ? l.lk.y : l.lk.x));
            QIO<float>::st(p.pout + ((int64_t(b) * D + c) * N + n) * 4, P4);
          }
        }
    }
  }
}

template <typename T, int G, int NG, bool S_REAL>
int launch_packed(FwdParams p, bool state_only, cudaStream_t st) {
  constexpr int CPW = 32 / NG;
  constexpr int NP = NG * G;
  const int sw = S_REAL ? 1 : 4;
  // one CTA per SM: nb CTAs per batch row with B * nb <= #SMs (never a partial
  // second wave); rows beyond #SMs simply queue
  const int sms = num_sms();
  int nb = sms / p.B;
  if (nb > p.D) nb = p.D;
  if (nb < 1) nb = 1;
  int cpb = (p.D + nb - 1) / nb;
  const int cap = (pk_max_threads(G) / 32 - 1) * CPW;
  if (cpb > cap) {
    nb = (p.D + cap - 1) / cap;
    cpb = (p.D + nb - 1) / nb;
  }
  const int warps = (cpb + CPW - 1) / CPW;
  int tc = kMaxTc;
  if (tc > p.T) tc = p.T;
  size_t smem = pk_layout(tc, NP, warps, CPW, sw).total;
  while (smem > kPkSmemBudget && tc > 1) {
    tc >>= 1;
    smem = pk_layout(tc, NP, warps, CPW, sw).total;
  }
  if (smem > kPkSmemBudget)
    return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_fwd: shared staging does not fit (N=%d)", p.N);

  // stream-ordered scratch: packed, fp32, zero-padded B/C rows, and for bf16
  // inputs fp32 copies of delta and S
  constexpr bool kWiden = !std::is_same<T, float>::value;
  const int64_t rows = int64_t(p.B) * p.T;
  const size_t plane = size_t(rows) * NP * 4 * sizeof(float);
  const int64_t n_delta = rows * p.D;
  const int64_t n_s = n_delta * (S_REAL ? 1 : 4);
  const size_t bytes = 2 * plane + (kWiden ? size_t(n_delta + n_s) * sizeof(float) : 0);
  float* ws = nullptr;
  cudaError_t e = scratch_alloc(reinterpret_cast<void**>(&ws), bytes, st);
  if (e != cudaSuccess)
    return fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd: scratch allocation of %zu bytes: %s", bytes,
                cudaGetErrorString(e));
  float* Bp = ws;
  float* Cp = ws + plane / sizeof(float);
  int ng_log2 = 0;
  while ((1 << ng_log2) < NG) ++ng_log2;
  const int64_t items = rows * (G / 2) * NG;
  const int64_t want = (items + kPackThreads - 1) / kPackThreads;
  const int pgrid = int(want < int64_t(sms) * 16 ? want : int64_t(sms) * 16);
  pack_bc_kernel<T><<<pgrid, kPackThreads, 0, st>>>(
      static_cast<const T*>(p.Bm), state_only ? nullptr : static_cast<const T*>(p.Cm), Bp, Cp,
      rows, p.N, ng_log2, G / 2);
  int rc = check_launch("mqc_ssm_scan_fwd(pack)");
  if (kWiden && rc == MQC_OK) {
    float* dw = Cp + plane / sizeof(float);
    float* sw32 = dw + n_delta;
    rc = launch_widen(p.delta, dw, n_delta, st);
    if (rc == MQC_OK) rc = launch_widen(p.s, sw32, n_s, st);
    p.delta = dw;
    p.s = sw32;
  }
  if (rc == MQC_OK) {
    p.Bm = Bp;
    p.Cm = Cp;
    p.nb = nb;
    p.cpb = cpb;
    p.tc = tc;
    const bool ck = p.ckpt != nullptr, dt = p.dst != 0;
    auto kern = state_only ? scan_fwd_packed_kernel<T, G, NG, S_REAL, false, false, true>
                : p.npeer > 0 ? scan_fwd_packed_kernel<T, G, NG, S_REAL, false, false, false, true>
                : ck ? (dt ? scan_fwd_packed_kernel<T, G, NG, S_REAL, true, true, false>
                           : scan_fwd_packed_kernel<T, G, NG, S_REAL, true, false, false>)
                     : (dt ? scan_fwd_packed_kernel<T, G, NG, S_REAL, false, true, false>
                           : scan_fwd_packed_kernel<T, G, NG, S_REAL, false, false, false>);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) {
      rc = fail(MQC_ERR_CUDA, "mqc_ssm_scan_fwd: smem attribute (%zu B): %s", smem,
                cudaGetErrorString(e));
    } else {
      dim3 grid{unsigned(nb), unsigned(p.B), 1u};
      kern<<<grid, 32 * (warps + 1), smem, st>>>(p);
      rc = check_launch("mqc_ssm_scan_fwd(packed)");
    }
  }
  scratch_free(ws, st);
  return rc;
}

template <typename T, int G, bool S_REAL>
int dispatch_packed_g(const FwdParams& p, bool so, cudaStream_t st) {
  // NG = lanes per channel, the power of two covering ceil(N / G), at most 32
  const int need = (p.N + G - 1) / G;
  int ng = 1;
  while (ng < need) ng <<= 1;
  switch (ng) {
    case 1: return launch_packed<T, G, 1, S_REAL>(p, so, st);
    case 2: return launch_packed<T, G, 2, S_REAL>(p, so, st);
    case 4: return launch_packed<T, G, 4, S_REAL>(p, so, st);
    case 8: return launch_packed<T, G, 8, S_REAL>(p, so, st);
    case 16: return launch_packed<T, G, 16, S_REAL>(p, so, st);
    case 32: return launch_packed<T, G, 32, S_REAL>(p, so, st);
    default:
      return fail(MQC_ERR_UNSUPPORTED, "mqc_ssm_scan_fwd: d_state=%d (supported 1..%d)", p.N,
                  32 * G);
  }
}

template <typename T, bool S_REAL>
int dispatch_packed_t(const FwdParams& p, bool so, cudaStream_t st) {
  return dispatch_packed_g<T, 8, S_REAL>(p, so, st);
}

int dispatch_packed(const FwdParams& p, int dtype, bool s_real, bool so, cudaStream_t st) {
  if (dtype == MQC_DTYPE_F32)
    return s_real ? dispatch_packed_t<float, true>(p, so, st)
                  : dispatch_packed_t<float, false>(p, so, st);
  return s_real ? dispatch_packed_t<__nv_bfloat16, true>(p, so, st)
                : dispatch_packed_t<__nv_bfloat16, false>(p, so, st);
}

}  // namespace

int pack_bc_pairs(const void* Bm, const void* Cm, float* Bp, float* Cp, int64_t rows, int N,
                  int NG, int G, int dtype, cudaStream_t st) {
  int ng_log2 = 0;
  while ((1 << ng_log2) < NG) ++ng_log2;
  const int64_t items = rows * (G / 2) * NG;
  const int64_t want = (items + kPackThreads - 1) / kPackThreads;
  const int64_t cap = int64_t(num_sms()) * 16;
  const int grid = int(want < cap ? (want > 0 ? want : 1) : cap);
  if (dtype == MQC_DTYPE_F32)
    pack_bc_kernel<float><<<grid, kPackThreads, 0, st>>>(
        static_cast<const float*>(Bm), static_cast<const float*>(Cm), Bp, Cp, rows, N, ng_log2,
        G / 2);
  else
    pack_bc_kernel<__nv_bfloat16><<<grid, kPackThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(Bm), static_cast<const __nv_bfloat16*>(Cm), Bp, Cp,
        rows, N, ng_log2, G / 2);
  return check_launch("pack_bc_pairs");
}

int widen_bf16_to_f32(const void* in, float* out, int64_t n, cudaStream_t st) {
  return launch_widen(in, out, n, st);
}

int dispatch_shared_packed(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  return dispatch_packed(p, dtype, s_real, false, st);
}

int dispatch_state_only_packed(const FwdParams& p, int dtype, bool s_real, cudaStream_t st) {
  return dispatch_packed(p, dtype, s_real, true, st);
}

}  // namespace scan
}  // namespace mqc
