// Pieces shared by the scan backward kernels (ssm_scan_bwd.cu for channel-shared
// B/C and the generic layouts, ssm_scan_bwd_pc.cu for per-channel B/C): the
// parameter block, the sub-block length and the lane reductions.
#pragma once

#include "ssm_scan_common.cuh"

namespace mqc {
namespace scan {

constexpr int kSub = MQC_SSM_CKPT_EVERY;
// Warps per CTA: the recomputed-state buffer is kSub * G * 32 lanes * 16 B per
// warp, so the CTA shrinks as G grows (G=2: 8 warps, 64 KiB; G=8: 2 warps).
// Per-channel B/C with G=2 keeps its states in registers and uses no shared
// memory; there 4-warp CTAs let 3 CTAs (12 warps) share an SM at ~170
// registers per thread, against one 8-warp CTA, and shorten the last wave.
__host__ __device__ constexpr int bwd_warps(int g, bool bc_shared = true) {
  return (g == 2 && !bc_shared) ? 4 : 16 / g;
}
constexpr int kMaxBwdSmem = 227 * 1024;

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

// In-register reduce-scatter of V values over the NG lanes of a channel by
// recursive halving: afterwards the lane holds W = max(V / NG, 1) sums
// v[0..W) whose original indices are base .. base + W - 1. Lanes that differ
// only in ng bits >= log2(V) hold the same sums.
template <int V, int NG>
__device__ __forceinline__ int reduce_scatter(float (&v)[V], int ng) {
  int base = 0;
#pragma unroll
  for (int lvl = 0; (1 << lvl) < NG; ++lvl) {
    const int m = 1 << lvl;
    constexpr int kUnused = 0;
    (void)kUnused;
    const int W = V >> lvl;
    if (W > 1) {
      const int half = W >> 1;
      const bool upper = (ng & m) != 0;
#pragma unroll
      for (int j = 0; j < (V >> (lvl + 1)); ++j) {
        const float send = upper ? v[j] : v[j + half];
        const float keep = upper ? v[j + half] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
      if (upper) base += half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
    }
  }
  return base;
}

// Packed backward for per-channel B/C [B,T,D,N,4] with 16 < N <= 64 (N even for
// bf16), ssm_scan_bwd_pc.cu. Returns MQC_ERR_UNSUPPORTED (without launching) for
// shapes it does not serve; the caller then takes the unpacked kernel.
int launch_bwd_perchannel(const BwdParams& p, int dtype, bool s_real, cudaStream_t st);
bool perchannel_bwd_serves(int N, int dtype);

}  // namespace scan
}  // namespace mqc
