// The real-valued glue of QuaternionMamba2Block around the scan, as streaming
// kernels: each reads its inputs once and writes its outputs once, in place of
// the chain of torch ops (and transposes) the reference block runs.
//
//   before the scan   conv_silu      a = bias + causal depthwise conv(x); out = silu(a)
//                                    (models/quaternion_mamba2_block.py:140-144,
//                                     layers/causal_conv1d.py:68-91)
//                     scan_inputs    delta = softplus(u); s = sigmoid(gate) * x
//                                    (block lines 183, 197-198)
//   after the scan    gate_residual  out = x + sigmoid(z) * y   (block lines 154-164)
//
// Each forward has a backward kernel. All arithmetic is fp32; activations are
// fp32 or bf16. A thread owns one 16-byte vector of adjacent channels (4 fp32 or
// 8 bf16) when the widths, strides and alignment allow it, else one channel;
// warps cover consecutive channel groups of one row, so every row access is
// coalesced. The conv kernels walk runs of time steps with the K-1 preceding
// inputs in registers, so x is read once from HBM (the (K-1)-row halo of each
// run is an L2 hit).
#include <initializer_list>

#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

constexpr int kMaxK = 8;
constexpr int kFwdRun = 4;       // time steps per thread, forward conv
constexpr int kBwdRun = 16;      // time steps per thread, backward conv
constexpr int kBwdRunsPerCta = 4;
constexpr int kPre = 3;         // rows of x and dout loaded ahead of use, backward conv
constexpr int kBwdParts = 128;   // max CTAs along the run axis (rows of partial sums)
constexpr int kConvThreads = 128;
constexpr int kEwThreads = 256;

// channels per thread on the 16-byte vector path
template <typename T>
constexpr int kVec = 16 / int(sizeof(T));

template <typename T, int V>
struct VIO;

template <>
struct VIO<float, 4> {
  static __device__ __forceinline__ void ld(const float* p, float (&v)[4]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  static __device__ __forceinline__ void st(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};

template <>
struct VIO<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <>
struct VIO<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void ld(const __nv_bfloat16* p, float (&v)[4]) {
    const float4 a = QIO<__nv_bfloat16>::ld(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, const float (&v)[4]) {
    QIO<__nv_bfloat16>::st(p, make_float4(v[0], v[1], v[2], v[3]));
  }
};

template <typename T>
struct VIO<T, 1> {
  static __device__ __forceinline__ void ld(const T* p, float (&v)[1]) { v[0] = QIO<T>::ld1(p); }
  static __device__ __forceinline__ void st(T* p, const float (&v)[1]) { QIO<T>::st1(p, v[0]); }
};

// 1 / (1 + e^-a): the fast exponential (__expf, relative error ~1e-6 over the
// range where sigmoid is not saturated) and the Newton-refined reciprocal
// (rcp_nr); 0 as a -> -inf. The accurate expf cost ~8 instructions per element
// and left these streaming kernels issue-bound.
__device__ __forceinline__ float sigmoid_f(float a) { return rcp_nr(1.f + __expf(-a)); }

// torch.nn.functional.softplus with beta = 1, threshold = 20
__device__ __forceinline__ float softplus_f(float u) { return u > 20.f ? u : log1pf(expf(u)); }

// ---------------------------------------------------------------- conv + SiLU

// grid (ceil(groups / kConvThreads), ny); one thread per channel group walks
// runs blockIdx.y, blockIdx.y + ny, ... of kFwdRun steps. The rows of the next
// run are loaded before the current run is computed and stored, so every warp
// keeps a run's loads in flight while it works (the kernel is latency-bound
// without this: one run per thread left DRAM at ~20 % of peak).
template <typename T, int V, int K>
__device__ __forceinline__ void conv_fwd_load(const T* __restrict__ x, int64_t x_row, int seq_len,
                                              int runs_per_seq, int c0, int r,
                                              float (&xr)[kFwdRun + K - 1][V]) {
  const int b = r / runs_per_seq;
  const int t0 = (r - b * runs_per_seq) * kFwdRun;
  const T* xb = x + int64_t(b) * seq_len * x_row + c0;
#pragma unroll
  for (int j = 0; j < kFwdRun + K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    if (t >= 0 && t < seq_len) {
      VIO<T, V>::ld(xb + int64_t(t) * x_row, xr[j]);
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) xr[j][v] = 0.f;
    }
  }
}

template <typename T, int V, int K>
__global__ void __launch_bounds__(kConvThreads)
    conv_silu_fwd_kernel(const T* __restrict__ x, int64_t x_row, const float* __restrict__ w,
                         const float* __restrict__ bias, T* __restrict__ out, int seq_len,
                         int channels, int runs_per_seq, int runs_total) {
  const int gi = blockIdx.x * kConvThreads + threadIdx.x;
  const int c0 = gi * V;
  if (c0 >= channels) return;
  float wk[K][V], bb[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    bb[v] = bias != nullptr ? __ldg(bias + c0 + v) : 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k][v] = __ldg(w + (c0 + v) * K + k);
  }
  // rows t0-(K-1) .. t0+kFwdRun-1 of a run; rows before 0 or past the end are 0
  float cur[kFwdRun + K - 1][V], nxt[kFwdRun + K - 1][V];
  int r = blockIdx.y;
  if (r < runs_total) conv_fwd_load<T, V, K>(x, x_row, seq_len, runs_per_seq, c0, r, cur);
  for (; r < runs_total; r += gridDim.y) {
    const int rn = r + int(gridDim.y);
    if (rn < runs_total) conv_fwd_load<T, V, K>(x, x_row, seq_len, runs_per_seq, c0, rn, nxt);
    const int b = r / runs_per_seq;
    const int t0 = (r - b * runs_per_seq) * kFwdRun;
    T* ob = out + (int64_t(b) * seq_len) * int64_t(channels) + c0;
#pragma unroll
    for (int i = 0; i < kFwdRun; ++i) {
      const int t = t0 + i;
      if (t < seq_len) {
        float o[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float a = bb[v];
#pragma unroll
          for (int k = 0; k < K; ++k) a = fmaf(wk[k][v], cur[i + k][v], a);
          o[v] = a * sigmoid_f(a);
        }
        VIO<T, V>::st(ob + int64_t(t) * channels, o);
      }
    }
#pragma unroll
    for (int j = 0; j < kFwdRun + K - 1; ++j)
#pragma unroll
      for (int v = 0; v < V; ++v) cur[j][v] = nxt[j][v];
  }
}

// block (32, kBwdRunsPerCta); grid (ceil(groups / 32), parts). Thread (x, y) owns
// channel group blockIdx.x*32+x and runs y, y+parts*kBwdRunsPerCta, ... of
// kBwdRun steps. A run walks t' = t0 .. t0+kBwdRun+K-2 with two rolling windows
// of K rows: x rows t'-(K-1)..t' (the pre-activation at t') and pre-activation
// gradients ga at t'-(K-1)..t'. Once ga(t') is known, dx at t = t'-(K-1) is
// complete: x_t feeds outputs t..t+K-1, output t+(K-1)-k through weight k.
// The x and dout rows are loaded kPre steps ahead of their use into a register
// ring (64.5 -> 57.2 us at the config-4 block shape, fp32), so each thread keeps
// loads in flight while it computes.
// Weight/bias gradient sums over the run's own outputs are reduced over y in
// shared memory and written as one row of `part` [parts, channels, K+1] per CTA.
template <typename T, int V, int K>
__global__ void __launch_bounds__(32 * kBwdRunsPerCta)
    conv_silu_bwd_kernel(const T* __restrict__ x, int64_t x_row, const float* __restrict__ w,
                         const float* __restrict__ bias, const T* __restrict__ dout,
                         T* __restrict__ dx, float* __restrict__ part, int seq_len, int channels,
                         int runs_per_seq, int64_t runs_total) {
  __shared__ float red[kBwdRunsPerCta][32][(K + 1) * V + 1];
  const int gi = blockIdx.x * 32 + threadIdx.x;
  const int c0 = gi * V;
  const bool live = c0 < channels;
  float acc[K + 1][V];
#pragma unroll
  for (int k = 0; k <= K; ++k)
#pragma unroll
    for (int v = 0; v < V; ++v) acc[k][v] = 0.f;
  if (live) {
    float wk[K][V], bb[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      bb[v] = bias != nullptr ? __ldg(bias + c0 + v) : 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) wk[k][v] = __ldg(w + (c0 + v) * K + k);
    }
    for (int64_t r = int64_t(blockIdx.y) * kBwdRunsPerCta + threadIdx.y; r < runs_total;
         r += int64_t(gridDim.y) * kBwdRunsPerCta) {
      const int64_t b = r / runs_per_seq;
      const int t0 = int(r % runs_per_seq) * kBwdRun;
      const T* xb = x + b * seq_len * x_row + c0;
      const T* gb = dout + (b * seq_len) * int64_t(channels) + c0;
      T* dxb = dx + (b * seq_len) * int64_t(channels) + c0;
      // before the first slide the x window holds rows t0-K .. t0-1
      float xw[K][V], gw[K][V];
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const int t = t0 - K + j;
        if (t >= 0) {
          VIO<T, V>::ld(xb + int64_t(t) * x_row, xw[j]);
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) xw[j][v] = 0.f;
        }
#pragma unroll
        for (int v = 0; v < V; ++v) gw[j][v] = 0.f;
      }
      // rows t0 .. t0+kPre-1 of x and dout, kPre steps ahead of their use
      float px[kPre][V], pg[kPre][V];
#pragma unroll
      for (int j = 0; j < kPre; ++j) {
        const int tp = t0 + j;
#pragma unroll
        for (int v = 0; v < V; ++v) px[j][v] = pg[j][v] = 0.f;
        if (tp < seq_len) {
          VIO<T, V>::ld(xb + int64_t(tp) * x_row, px[j]);
          VIO<T, V>::ld(gb + int64_t(tp) * channels, pg[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kBwdRun + K - 1; ++j) {
        const int tp = t0 + j;
        // slide both windows by one row
#pragma unroll
        for (int m = 0; m < K - 1; ++m)
#pragma unroll
          for (int v = 0; v < V; ++v) {
            xw[m][v] = xw[m + 1][v];
            gw[m][v] = gw[m + 1][v];
          }
        float g[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
          xw[K - 1][v] = px[j % kPre][v];
          g[v] = pg[j % kPre][v];
        }
        {
          const int tq = tp + kPre;
          if (j + kPre < kBwdRun + K - 1 && tq < seq_len) {
            VIO<T, V>::ld(xb + int64_t(tq) * x_row, px[j % kPre]);
            VIO<T, V>::ld(gb + int64_t(tq) * channels, pg[j % kPre]);
          }
        }
        if (tp < seq_len) {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            float a = bb[v];
#pragma unroll
            for (int k = 0; k < K; ++k) a = fmaf(wk[k][v], xw[k][v], a);
            const float s = sigmoid_f(a);
            gw[K - 1][v] = g[v] * s * fmaf(a, 1.f - s, 1.f);
          }
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            xw[K - 1][v] = 0.f;
            gw[K - 1][v] = 0.f;
          }
        }
        if (j < kBwdRun) {
          // output t' is this run's: weight k met input t'-(K-1)+k
#pragma unroll
          for (int v = 0; v < V; ++v) {
#pragma unroll
            for (int k = 0; k < K; ++k) acc[k][v] = fmaf(gw[K - 1][v], xw[k][v], acc[k][v]);
            acc[K][v] += gw[K - 1][v];
          }
        }
        const int t = tp - (K - 1);
        if (j >= K - 1 && t < seq_len) {
          float o[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) s = fmaf(wk[k][v], gw[K - 1 - k][v], s);
            o[v] = s;
          }
          VIO<T, V>::st(dxb + int64_t(t) * channels, o);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k <= K; ++k)
#pragma unroll
    for (int v = 0; v < V; ++v) red[threadIdx.y][threadIdx.x][k * V + v] = acc[k][v];
  __syncthreads();
  if (threadIdx.y == 0 && live) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
#pragma unroll
      for (int k = 0; k <= K; ++k) {
        float s = 0.f;
#pragma unroll
        for (int y = 0; y < kBwdRunsPerCta; ++y) s += red[y][threadIdx.x][k * V + v];
        part[(int64_t(blockIdx.y) * channels + c0 + v) * (K + 1) + k] = s;
      }
    }
  }
}

// dweight[c,k] = sum_p part[p,c,k]; dbias[c] = sum_p part[p,c,K] (fixed order)
__global__ void __launch_bounds__(kEwThreads)
    conv_param_grad_kernel(const float* __restrict__ part, float* __restrict__ dw,
                           float* __restrict__ db, int parts, int channels, int K) {
  const int i = blockIdx.x * kEwThreads + threadIdx.x;
  if (i >= channels * (K + 1)) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += part[int64_t(p) * channels * (K + 1) + i];
  const int c = i / (K + 1), k = i % (K + 1);
  if (k < K) {
    dw[c * K + k] = s;
  } else if (db != nullptr) {
    db[c] = s;
  }
}

// ---------------------------------------------------------------- scan inputs

template <typename T, int V>
__global__ void __launch_bounds__(kEwThreads)
    scan_inputs_fwd_kernel(const T* __restrict__ u, int64_t u_row, const T* __restrict__ g,
                           int64_t g_row, const T* __restrict__ x, T* __restrict__ delta,
                           T* __restrict__ s, int64_t rows, int groups) {
  const int64_t n = rows * groups;
  for (int64_t i = int64_t(blockIdx.x) * kEwThreads + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * kEwThreads) {
    const int64_t r = i / groups;
    const int64_t c = (i - r * groups) * V;
    const int64_t o = r * groups * V + c;
    float uv[V], gv[V], xv[V], dv[V], sv[V];
    VIO<T, V>::ld(u + r * u_row + c, uv);
    VIO<T, V>::ld(g + r * g_row + c, gv);
    VIO<T, V>::ld(x + o, xv);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      dv[v] = softplus_f(uv[v]);
      sv[v] = sigmoid_f(gv[v]) * xv[v];
    }
    VIO<T, V>::st(delta + o, dv);
    VIO<T, V>::st(s + o, sv);
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(kEwThreads)
    scan_inputs_bwd_kernel(const T* __restrict__ u, int64_t u_row, const T* __restrict__ g,
                           int64_t g_row, const T* __restrict__ x, const T* __restrict__ dd,
                           const T* __restrict__ ds, T* __restrict__ du, T* __restrict__ dg,
                           T* __restrict__ dx, int64_t rows, int groups) {
  const int64_t n = rows * groups;
  for (int64_t i = int64_t(blockIdx.x) * kEwThreads + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * kEwThreads) {
    const int64_t r = i / groups;
    const int64_t c = (i - r * groups) * V;
    const int64_t o = r * groups * V + c;
    float uv[V], gv[V], xv[V], ddv[V], dsv[V], o_u[V], o_g[V], o_x[V];
    VIO<T, V>::ld(u + r * u_row + c, uv);
    VIO<T, V>::ld(g + r * g_row + c, gv);
    VIO<T, V>::ld(x + o, xv);
    if (dd != nullptr) {
      VIO<T, V>::ld(dd + o, ddv);
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) ddv[v] = 0.f;
    }
    if (ds != nullptr) {
      VIO<T, V>::ld(ds + o, dsv);
    } else {
#pragma unroll
      for (int v = 0; v < V; ++v) dsv[v] = 0.f;
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      // torch's softplus backward: dout * e/(e+1), e = exp(u), pass-through above 20
      const float e = expf(uv[v]);
      o_u[v] = uv[v] > 20.f ? ddv[v] : ddv[v] * (e / (e + 1.f));
      const float sg = sigmoid_f(gv[v]);
      o_g[v] = dsv[v] * xv[v] * (1.f - sg) * sg;
      o_x[v] = dsv[v] * sg;
    }
    VIO<T, V>::st(du + o, o_u);
    VIO<T, V>::st(dg + o, o_g);
    VIO<T, V>::st(dx + o, o_x);
  }
}

// ---------------------------------------------------------------- gate + residual

template <typename T, int V>
__global__ void __launch_bounds__(kEwThreads)
    gate_residual_fwd_kernel(const T* __restrict__ x, const T* __restrict__ z, int64_t z_row,
                             const T* __restrict__ y, T* __restrict__ out, int64_t rows,
                             int groups) {
  const int64_t n = rows * groups;
  for (int64_t i = int64_t(blockIdx.x) * kEwThreads + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * kEwThreads) {
    const int64_t r = i / groups;
    const int64_t c = (i - r * groups) * V;
    const int64_t o = r * groups * V + c;
    float xv[V], zv[V], yv[V], ov[V];
    VIO<T, V>::ld(x + o, xv);
    VIO<T, V>::ld(z + r * z_row + c, zv);
    VIO<T, V>::ld(y + o, yv);
#pragma unroll
    for (int v = 0; v < V; ++v) ov[v] = fmaf(sigmoid_f(zv[v]), yv[v], xv[v]);
    VIO<T, V>::st(out + o, ov);
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(kEwThreads)
    gate_residual_bwd_kernel(const T* __restrict__ z, int64_t z_row, const T* __restrict__ y,
                             const T* __restrict__ dout, T* __restrict__ dz, T* __restrict__ dy,
                             int64_t rows, int groups) {
  const int64_t n = rows * groups;
  for (int64_t i = int64_t(blockIdx.x) * kEwThreads + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * kEwThreads) {
    const int64_t r = i / groups;
    const int64_t c = (i - r * groups) * V;
    const int64_t o = r * groups * V + c;
    float zv[V], yv[V], gv[V], o_z[V], o_y[V];
    VIO<T, V>::ld(z + r * z_row + c, zv);
    VIO<T, V>::ld(y + o, yv);
    VIO<T, V>::ld(dout + o, gv);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const float sg = sigmoid_f(zv[v]);
      o_z[v] = gv[v] * yv[v] * (1.f - sg) * sg;
      o_y[v] = gv[v] * sg;
    }
    VIO<T, V>::st(dz + o, o_z);
    VIO<T, V>::st(dy + o, o_y);
  }
}

// ---------------------------------------------------------------- host side

// V channels per thread when the channel count, the strides (elements) and the
// pointers allow V-element vectors: the elementwise kernels use 16-byte vectors
// (4 fp32 / 8 bf16), the conv kernels 4 channels in both dtypes (their rolling
// windows hold K rows of V values per thread).
bool vec_ok(int64_t channels, int64_t V, int dtype, std::initializer_list<const void*> ptrs,
            std::initializer_list<int64_t> strides) {
  if (channels % V != 0) return false;
  const uintptr_t al = uintptr_t(V) * uintptr_t(dtype_size(dtype));
  for (const void* p : ptrs)
    if (p != nullptr && !aligned(p, al)) return false;
  for (int64_t s : strides)
    if (s % V != 0) return false;
  return true;
}

int ew_vec(int dtype) { return 16 / dtype_size(dtype); }

int ck_zero(float* p, size_t bytes, cudaStream_t st) {
  const cudaError_t e = cudaMemsetAsync(p, 0, bytes, st);
  return e == cudaSuccess ? MQC_OK
                          : fail(MQC_ERR_CUDA, "mqc_conv_silu_bwd: memset: %s", cudaGetErrorString(e));
}

int ew_grid(int64_t n) {
  int64_t g = (n + kEwThreads - 1) / kEwThreads;
  const int64_t cap = int64_t(num_sms()) * 8;
  return int(g < 1 ? 1 : (g > cap ? cap : g));
}

template <typename T, int V, int K>
void launch_conv_fwd(const void* x, int64_t x_row, const float* w, const float* bias, void* out,
                     int64_t B, int64_t T_, int64_t D, cudaStream_t st) {
  const int groups = int(D / V);
  const int runs_per_seq = int((T_ + kFwdRun - 1) / kFwdRun);
  const int64_t runs_total = B * runs_per_seq;  // <= INT32_MAX, checked by the entry point
  // one wave of resident CTAs, each thread walking several runs
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv_silu_fwd_kernel<T, V, K>,
                                                    kConvThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int gx = (groups + kConvThreads - 1) / kConvThreads;
  int64_t gy = int64_t(num_sms()) * per_sm / gx;
  if (gy < 1) gy = 1;
  if (gy > runs_total) gy = runs_total;
  if (gy > 65535) gy = 65535;
  dim3 grid{unsigned(gx), unsigned(gy), 1u};
  conv_silu_fwd_kernel<T, V, K><<<grid, kConvThreads, 0, st>>>(
      static_cast<const T*>(x), x_row, w, bias, static_cast<T*>(out), int(T_), int(D),
      runs_per_seq, int(runs_total));
}

template <typename T, int V, int K>
void launch_conv_bwd(const void* x, int64_t x_row, const float* w, const float* bias,
                     const void* dout, void* dx, float* part, int parts, int64_t B, int64_t T_,
                     int64_t D, cudaStream_t st) {
  const int groups = int(D / V);
  const int runs_per_seq = int((T_ + kBwdRun - 1) / kBwdRun);
  const int64_t runs_total = B * runs_per_seq;
  dim3 grid{unsigned((groups + 31) / 32), unsigned(parts), 1u};
  dim3 block{32u, unsigned(kBwdRunsPerCta), 1u};
  conv_silu_bwd_kernel<T, V, K><<<grid, block, 0, st>>>(
      static_cast<const T*>(x), x_row, w, bias, static_cast<const T*>(dout),
      static_cast<T*>(dx), part, int(T_), int(D), runs_per_seq, runs_total);
}

// dispatch over dtype, vector width and K (1..8)
template <template <typename, int, int> class L, typename... A>
int dispatch_conv(int dtype, bool v4, int64_t K, A... args) {
#define MQC_CONV_K(KK)                                                     \
  case KK:                                                                 \
    if (dtype == MQC_DTYPE_F32) {                                          \
      if (v4) L<float, 4, KK>::run(args...);                               \
      else L<float, 1, KK>::run(args...);                                  \
    } else {                                                               \
      if (v4) L<__nv_bfloat16, 4, KK>::run(args...);                       \
      else L<__nv_bfloat16, 1, KK>::run(args...);                          \
    }                                                                      \
    return MQC_OK;
  switch (K) {
    MQC_CONV_K(1) MQC_CONV_K(2) MQC_CONV_K(3) MQC_CONV_K(4)
    MQC_CONV_K(5) MQC_CONV_K(6) MQC_CONV_K(7) MQC_CONV_K(8)
    default: return fail(MQC_ERR_UNSUPPORTED, "conv kernel size %lld not in 1..8", (long long)K);
  }
#undef MQC_CONV_K
}

template <typename T, int V, int K>
struct ConvFwd {
  template <typename... A>
  static void run(A... a) { launch_conv_fwd<T, V, K>(a...); }
};
template <typename T, int V, int K>
struct ConvBwd {
  template <typename... A>
  static void run(A... a) { launch_conv_bwd<T, V, K>(a...); }
};

int conv_parts(int64_t B, int64_t T_) {
  const int64_t runs_total = B * ((T_ + kBwdRun - 1) / kBwdRun);
  const int64_t p = (runs_total + kBwdRunsPerCta - 1) / kBwdRunsPerCta;
  return int(p < 1 ? 1 : (p > kBwdParts ? kBwdParts : p));
}

int check_conv(const void* x, int64_t x_row, const float* w, int64_t B, int64_t T_, int64_t D,
               int64_t K, int dtype, const char* name) {
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, dtype);
  MQC_REQUIRE(B >= 0 && T_ >= 0 && D >= 0, MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(K >= 1 && K <= kMaxK, MQC_ERR_UNSUPPORTED, "%s: kernel size %lld not in 1..8", name,
              (long long)K);
  MQC_REQUIRE(x_row >= D, MQC_ERR_INVALID_VALUE, "%s: row stride %lld < channels %lld", name,
              (long long)x_row, (long long)D);
  MQC_REQUIRE(B * T_ * D == 0 || (x != nullptr && w != nullptr), MQC_ERR_INVALID_VALUE,
              "%s: null pointer", name);
  MQC_REQUIRE(T_ <= INT32_MAX && D <= INT32_MAX && B * ((T_ + kFwdRun - 1) / kFwdRun) <= INT32_MAX,
              MQC_ERR_UNSUPPORTED, "%s: sizes too large", name);
  return MQC_OK;
}

int check_ew(int64_t rows, int64_t cols, int dtype, const char* name,
             std::initializer_list<const void*> ptrs) {
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, dtype);
  MQC_REQUIRE(rows >= 0 && cols >= 0, MQC_ERR_INVALID_VALUE, "%s: negative size", name);
  MQC_REQUIRE(cols <= INT32_MAX, MQC_ERR_UNSUPPORTED, "%s: too many columns", name);
  if (rows * cols == 0) return MQC_OK;
  for (const void* p : ptrs)
    MQC_REQUIRE(p != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  return MQC_OK;
}

}  // namespace
}  // namespace mqc

using namespace mqc;

extern "C" int mqc_conv_silu_fwd(const void* x, int64_t x_row_stride, const float* weight,
                                 const float* bias, void* out, int64_t batch, int64_t seq_len,
                                 int64_t channels, int64_t kernel_size, int dtype, void* stream) {
  clear_error();
  const char* name = "mqc_conv_silu_fwd";
  int rc = check_conv(x, x_row_stride, weight, batch, seq_len, channels, kernel_size, dtype, name);
  if (rc != MQC_OK || batch * seq_len * channels == 0) return rc;
  MQC_REQUIRE(out != nullptr, MQC_ERR_INVALID_VALUE, "%s: null out", name);
  const bool v4 = vec_ok(channels, 4, dtype, {x, out}, {x_row_stride});
  rc = dispatch_conv<ConvFwd>(dtype, v4, kernel_size, x, x_row_stride, weight, bias, out, batch,
                              seq_len, channels, as_stream(stream));
  if (rc != MQC_OK) return rc;
  return check_launch(name);
}

extern "C" size_t mqc_conv_silu_bwd_workspace_size(int64_t batch, int64_t seq_len,
                                                   int64_t channels, int64_t kernel_size) {
  if (batch <= 0 || seq_len <= 0 || channels <= 0 || kernel_size < 1 || kernel_size > kMaxK)
    return 0;
  return size_t(conv_parts(batch, seq_len)) * size_t(channels) * size_t(kernel_size + 1) * 4;
}

extern "C" int mqc_conv_silu_bwd(const void* x, int64_t x_row_stride, const float* weight,
                                 const float* bias, const void* dout, void* dx, float* dweight,
                                 float* dbias, int64_t batch, int64_t seq_len, int64_t channels,
                                 int64_t kernel_size, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  clear_error();
  const char* name = "mqc_conv_silu_bwd";
  int rc = check_conv(x, x_row_stride, weight, batch, seq_len, channels, kernel_size, dtype, name);
  if (rc != MQC_OK || channels == 0) return rc;
  MQC_REQUIRE(dweight != nullptr, MQC_ERR_INVALID_VALUE, "%s: null dweight", name);
  cudaStream_t st = as_stream(stream);
  if (batch * seq_len == 0) {
    // no (b, t): the parameter gradients are zero
    rc = ck_zero(dweight, size_t(channels * kernel_size) * 4, st);
    if (rc == MQC_OK && dbias != nullptr) rc = ck_zero(dbias, size_t(channels) * 4, st);
    return rc;
  }
  MQC_REQUIRE(dout != nullptr && dx != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  const size_t need = mqc_conv_silu_bwd_workspace_size(batch, seq_len, channels, kernel_size);
  MQC_REQUIRE(workspace != nullptr && workspace_bytes >= need && aligned(workspace, 16),
              MQC_ERR_INVALID_VALUE, "%s: 16-byte aligned workspace of %zu bytes required", name,
              need);
  const int parts = conv_parts(batch, seq_len);
  float* part = static_cast<float*>(workspace);
  const bool v4 = vec_ok(channels, 4, dtype, {x, dout, dx}, {x_row_stride});
  rc = dispatch_conv<ConvBwd>(dtype, v4, kernel_size, x, x_row_stride, weight, bias, dout, dx,
                              part, parts, batch, seq_len, channels, st);
  if (rc != MQC_OK) return rc;
  rc = check_launch(name);
  if (rc != MQC_OK) return rc;
  const int64_t n = channels * (kernel_size + 1);
  conv_param_grad_kernel<<<unsigned((n + kEwThreads - 1) / kEwThreads), kEwThreads, 0, st>>>(
      part, dweight, dbias, parts, int(channels), int(kernel_size));
  return check_launch(name);
}

extern "C" int mqc_scan_inputs_fwd(const void* u, int64_t u_row_stride, const void* gate,
                                   int64_t gate_row_stride, const void* x, void* delta, void* s,
                                   int64_t rows, int64_t channels, int dtype, void* stream) {
  clear_error();
  const char* name = "mqc_scan_inputs_fwd";
  int rc = check_ew(rows, channels, dtype, name, {u, gate, x, delta, s});
  if (rc != MQC_OK || rows * channels == 0) return rc;
  MQC_REQUIRE(u_row_stride >= channels && gate_row_stride >= channels, MQC_ERR_INVALID_VALUE,
              "%s: row stride below channels", name);
  const bool v4 = vec_ok(channels, ew_vec(dtype), dtype, {u, gate, x, delta, s}, {u_row_stride, gate_row_stride});
  const int V = v4 ? ew_vec(dtype) : 1;
  const int g = ew_grid(rows * (channels / V));
  cudaStream_t st = as_stream(stream);
#define MQC_SI_FWD(TT, VV)                                                                 \
  scan_inputs_fwd_kernel<TT, VV><<<g, kEwThreads, 0, st>>>(                                \
      static_cast<const TT*>(u), u_row_stride, static_cast<const TT*>(gate), gate_row_stride, \
      static_cast<const TT*>(x), static_cast<TT*>(delta), static_cast<TT*>(s), rows,      \
      int(channels / VV))
  if (dtype == MQC_DTYPE_F32) {
    if (v4) MQC_SI_FWD(float, 4); else MQC_SI_FWD(float, 1);
  } else {
    if (v4) MQC_SI_FWD(__nv_bfloat16, 8); else MQC_SI_FWD(__nv_bfloat16, 1);
  }
#undef MQC_SI_FWD
  return check_launch(name);
}

extern "C" int mqc_scan_inputs_bwd(const void* u, int64_t u_row_stride, const void* gate,
                                   int64_t gate_row_stride, const void* x, const void* ddelta,
                                   const void* ds, void* du, void* dgate, void* dx, int64_t rows,
                                   int64_t channels, int dtype, void* stream) {
  clear_error();
  const char* name = "mqc_scan_inputs_bwd";
  int rc = check_ew(rows, channels, dtype, name, {u, gate, x, du, dgate, dx});
  if (rc != MQC_OK || rows * channels == 0) return rc;
  MQC_REQUIRE(u_row_stride >= channels && gate_row_stride >= channels, MQC_ERR_INVALID_VALUE,
              "%s: row stride below channels", name);
  const bool v4 = vec_ok(channels, ew_vec(dtype), dtype, {u, gate, x, ddelta, ds, du, dgate, dx},
                          {u_row_stride, gate_row_stride});
  const int V = v4 ? ew_vec(dtype) : 1;
  const int g = ew_grid(rows * (channels / V));
  cudaStream_t st = as_stream(stream);
#define MQC_SI_BWD(TT, VV)                                                                    \
  scan_inputs_bwd_kernel<TT, VV><<<g, kEwThreads, 0, st>>>(                                   \
      static_cast<const TT*>(u), u_row_stride, static_cast<const TT*>(gate), gate_row_stride,    \
      static_cast<const TT*>(x), static_cast<const TT*>(ddelta), static_cast<const TT*>(ds),   \
      static_cast<TT*>(du), static_cast<TT*>(dgate), static_cast<TT*>(dx), rows,              \
      int(channels / VV))
  if (dtype == MQC_DTYPE_F32) {
    if (v4) MQC_SI_BWD(float, 4); else MQC_SI_BWD(float, 1);
  } else {
    if (v4) MQC_SI_BWD(__nv_bfloat16, 8); else MQC_SI_BWD(__nv_bfloat16, 1);
  }
#undef MQC_SI_BWD
  return check_launch(name);
}

extern "C" int mqc_gate_residual_fwd(const void* x, const void* z, int64_t z_row_stride,
                                     const void* y, void* out, int64_t rows, int64_t cols,
                                     int dtype, void* stream) {
  clear_error();
  const char* name = "mqc_gate_residual_fwd";
  int rc = check_ew(rows, cols, dtype, name, {x, z, y, out});
  if (rc != MQC_OK || rows * cols == 0) return rc;
  MQC_REQUIRE(z_row_stride >= cols, MQC_ERR_INVALID_VALUE, "%s: row stride below cols", name);
  const bool v4 = vec_ok(cols, ew_vec(dtype), dtype, {x, z, y, out}, {z_row_stride});
  const int V = v4 ? ew_vec(dtype) : 1;
  const int g = ew_grid(rows * (cols / V));
  cudaStream_t st = as_stream(stream);
#define MQC_GR_FWD(TT, VV)                                                                \
  gate_residual_fwd_kernel<TT, VV><<<g, kEwThreads, 0, st>>>(                             \
      static_cast<const TT*>(x), static_cast<const TT*>(z), z_row_stride,                 \
      static_cast<const TT*>(y), static_cast<TT*>(out), rows, int(cols / VV))
  if (dtype == MQC_DTYPE_F32) {
    if (v4) MQC_GR_FWD(float, 4); else MQC_GR_FWD(float, 1);
  } else {
    if (v4) MQC_GR_FWD(__nv_bfloat16, 8); else MQC_GR_FWD(__nv_bfloat16, 1);
  }
#undef MQC_GR_FWD
  return check_launch(name);
}

extern "C" int mqc_gate_residual_bwd(const void* z, int64_t z_row_stride, const void* y,
                                     const void* dout, void* dz, void* dy, int64_t rows,
                                     int64_t cols, int dtype, void* stream) {
  clear_error();
  const char* name = "mqc_gate_residual_bwd";
  int rc = check_ew(rows, cols, dtype, name, {z, y, dout, dz, dy});
  if (rc != MQC_OK || rows * cols == 0) return rc;
  MQC_REQUIRE(z_row_stride >= cols, MQC_ERR_INVALID_VALUE, "%s: row stride below cols", name);
  const bool v4 = vec_ok(cols, ew_vec(dtype), dtype, {z, y, dout, dz, dy}, {z_row_stride});
  const int V = v4 ? ew_vec(dtype) : 1;
  const int g = ew_grid(rows * (cols / V));
  cudaStream_t st = as_stream(stream);
#define MQC_GR_BWD(TT, VV)                                                                 \
  gate_residual_bwd_kernel<TT, VV><<<g, kEwThreads, 0, st>>>(                              \
      static_cast<const TT*>(z), z_row_stride, static_cast<const TT*>(y),                  \
      static_cast<const TT*>(dout), static_cast<TT*>(dz), static_cast<TT*>(dy), rows,      \
      int(cols / VV))
  if (dtype == MQC_DTYPE_F32) {
    if (v4) MQC_GR_BWD(float, 4); else MQC_GR_BWD(float, 1);
  } else {
    if (v4) MQC_GR_BWD(__nv_bfloat16, 8); else MQC_GR_BWD(__nv_bfloat16, 1);
  }
#undef MQC_GR_BWD
  return check_launch(name);
}
