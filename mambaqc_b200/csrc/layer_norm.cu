// Quaternion LayerNorm (norm-only rescale that preserves each quaternion's
// direction), forward and backward.
//
// Reference: quaternion_layer_norm_fused / quaternion_layer_norm_reference,
// mambaqc/kernels/quaternion_norm.py:119-174 and :219-245. One CTA owns one row
// of d_model quaternions, staged in shared memory by cp.async (16-byte coalesced
// copies), so the row is read from HBM once and written once. Mean and variance of the norms are two-pass over registers
// (mean first, then centred squares), with warp-shuffle + shared-memory sums.
#include <type_traits>

#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

constexpr int kVpt = 8;           // quaternions per thread
constexpr int kMaxRowThreads = 512;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red[] reuse across calls
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];  // same order on every thread
  return s;
}

// Two block sums in one pass (one pair of barriers): red must hold 64 floats.
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red[] reuse across calls
  if (l == 0) {
    red[w] = a;
    red[32 + w] = b;
  }
  __syncthreads();
  float sa = 0.f, sb = 0.f;
  for (int i = 0; i < nw; ++i) {  // same order on every thread
    sa += red[i];
    sb += red[32 + i];
  }
  return make_float2(sa, sb);
}

// 8-byte asynchronous global -> shared copy (one bf16 quaternion).
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

// The row is staged in shared memory with cp.async (no registers held while it
// is in flight), so many rows per SM are in flight at once; each thread then
// works on quaternions d = threadIdx.x + j * blockDim.x of the staged row.
template <typename T>
__global__ void __launch_bounds__(kMaxRowThreads) qln_fwd_kernel(
    const T* __restrict__ q, const float* __restrict__ gamma, const float* __restrict__ beta,
    T* __restrict__ out, float* __restrict__ mean_out, float* __restrict__ rstd_out, int D,
    float eps, int pad_lanes) {
  __shared__ float red[32];
  extern __shared__ __align__(16) unsigned char srow_raw[];
  T* srow = reinterpret_cast<T*>(srow_raw);
  const int64_t row = blockIdx.x;
  const T* qr = q + row * D * 4;
  T* orow = out + row * D * 4;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    if constexpr (sizeof(T) == 4) cp_async16(srow + d * 4, qr + d * 4, true);
    else cp_async8(srow + d * 4, qr + d * 4);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  float nrm[kVpt];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    const int d = threadIdx.x + j * blockDim.x;
    nrm[j] = 0.f;
    if (d < D) {
      const float4 a = QIO<T>::lds(srow + d * 4);
      nrm[j] = sqrtf(fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, a.w * a.w))) + eps);
      s += nrm[j];
    }
  }
  const float pad_norm = sqrtf(eps);
  float tot = block_sum(s, red);
  if (pad_lanes) tot += float(pad_lanes) * pad_norm;
  const float mu = tot / float(D);
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    const int d = threadIdx.x + j * blockDim.x;
    if (d < D) {
      const float c = nrm[j] - mu;
      s2 = fmaf(c, c, s2);
    }
  }
  float tot2 = block_sum(s2, red);
  if (pad_lanes) tot2 += float(pad_lanes) * (pad_norm - mu) * (pad_norm - mu);
  const float var = tot2 / float(D);
  const float sd = sqrtf(var + eps);
  const float rsd = 1.f / sd;
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rsd;
  }
  if (out == nullptr) return;  // row statistics only (qln_row_stats)
  // one reciprocal per quaternion (and one per row) instead of a division per
  // component: out = gamma * nh * q / (n + eps) + beta
#pragma unroll
  for (int j = 0; j < kVpt; ++j) {
    const int d = threadIdx.x + j * blockDim.x;
    if (d < D) {
      const float nh = (nrm[j] - mu) * rsd;
      const float g = __ldg(gamma + d) * nh * (1.f / (nrm[j] + eps));
      const float4 bt = QIO<float>::ld(beta + d * 4);
      const float4 v = QIO<T>::lds(srow + d * 4);
      float4 o;
      o.x = fmaf(g, v.x, bt.x);
      o.y = fmaf(g, v.y, bt.y);
      o.z = fmaf(g, v.z, bt.z);
      o.w = fmaf(g, v.w, bt.w);
      QIO<T>::st_stream(orow + d * 4, o);
    }
  }
}

// Backward. Per row, with n = sqrt(|q|^2 + eps), nh = (n - mu) * rstd,
// u = q / (n + eps), g = dL/dout and a = gamma * <g, u>:
//   dL/dn = rstd * (a - mean(a) - nh * mean(a * nh)) - nh * a / (n + eps)
//   dq    = gamma * nh * g / (n + eps) + dL/dn * q / n
//   dgamma += nh * <g, u>,  dbeta += g        (summed over rows)
// A CTA walks rows blockIdx.x, blockIdx.x + gridDim.x, ...; each thread keeps the
// dgamma/dbeta partials of its own columns in registers and writes one partial
// row per CTA; qln_bwd_reduce_kernel sums the partials in a fixed order, so the
// parameter gradients are deterministic.
constexpr int kVptB = 4;

// Offset (in floats) of the dbeta partials: after parts*D dgamma partials,
// rounded up to a multiple of 4 floats so every float4 store is 16-byte aligned.
__host__ __device__ inline int64_t beta_partial_offset(int64_t parts, int64_t D) {
  return (parts * D + 3) / 4 * 4;
}

// The rows are staged in shared memory with cp.async, double-buffered where two
// rows of q and dout fit (nstage = 2): the copies of the next row are in flight
// while the current one is reduced and written, so no registers wait on loads.
// Every thread copies, and later reads, only its own quaternions
// d = threadIdx.x + j * blockDim.x, so the staging needs no barrier.
// MAXT: the CTA size the register budget is sized for (512 for d_model <= 2048,
// 1024 for the widest rows).
template <typename T, int MAXT>
__global__ void __launch_bounds__(MAXT) qln_bwd_kernel(
    const T* __restrict__ q, const float* __restrict__ gamma, const T* __restrict__ dout,
    const float* __restrict__ mean, const float* __restrict__ rstd, T* __restrict__ dq,
    float* __restrict__ partial, int64_t rows, int D, float eps, int nstage) {
  __shared__ float red[64];
  extern __shared__ __align__(16) unsigned char sbuf_raw[];
  T* sbuf = reinterpret_cast<T*>(sbuf_raw);
  const int64_t rlen = int64_t(D) * 4;  // elements of one row
  // stage s: the q row at sbuf + 2 s rlen, the dout row right after it
  auto stage_row = [&](int64_t row, int s) {
    const T* qr = q + row * rlen;
    const T* gr = dout + row * rlen;
    T* sq = sbuf + 2 * s * rlen;
    T* sg = sq + rlen;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      if constexpr (sizeof(T) == 4) {
        cp_async16(sq + d * 4, qr + d * 4, true);
        cp_async16(sg + d * 4, gr + d * 4, true);
      } else {
        cp_async8(sq + d * 4, qr + d * 4);
        cp_async8(sg + d * 4, gr + d * 4);
      }
    }
    cp_async_commit();
  };
  float dg[kVptB];
  float4 db[kVptB];
  float gm[kVptB];
#pragma unroll
  for (int j = 0; j < kVptB; ++j) {
    dg[j] = 0.f;
    db[j] = f4_zero();
    const int d = threadIdx.x + j * blockDim.x;
    gm[j] = d < D ? __ldg(gamma + d) : 0.f;
  }
  int s = 0;
  if (blockIdx.x < rows) stage_row(blockIdx.x, 0);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t nxt = row + gridDim.x;
    if (nstage == 2 && nxt < rows) {
      stage_row(nxt, s ^ 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    const T* sq = sbuf + 2 * s * rlen;
    const T* sg = sq + rlen;
    const float mu = __ldg(mean + row), rs = __ldg(rstd + row);
    // rdn = 1 / (n + eps) and rn = 1 / n, Newton-refined reciprocals: each
    // quaternion takes two instead of four divisions
    float nrm[kVptB], nh[kVptB], av[kVptB], rdn[kVptB];
    float sa = 0.f, san = 0.f;
#pragma unroll
    for (int j = 0; j < kVptB; ++j) {
      const int d = threadIdx.x + j * blockDim.x;
      nrm[j] = 1.f;
      nh[j] = 0.f;
      av[j] = 0.f;
      rdn[j] = 0.f;
      if (d < D) {
        const float4 a = QIO<T>::lds(sq + d * 4);
        const float4 gv = QIO<T>::lds(sg + d * 4);
        nrm[j] = sqrtf(fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, a.w * a.w))) + eps);
        nh[j] = (nrm[j] - mu) * rs;
        rdn[j] = rcp_nr(nrm[j] + eps);
        const float gu = fmaf(gv.x, a.x, fmaf(gv.y, a.y, fmaf(gv.z, a.z, gv.w * a.w))) * rdn[j];
        av[j] = gm[j] * gu;
        sa += av[j];
        san = fmaf(av[j], nh[j], san);
        dg[j] = fmaf(nh[j], gu, dg[j]);
        db[j].x += gv.x;
        db[j].y += gv.y;
        db[j].z += gv.z;
        db[j].w += gv.w;
      }
    }
    const float2 sums = block_sum2(sa, san, red);
    const float ma = sums.x / float(D);
    const float man = sums.y / float(D);
#pragma unroll
    for (int j = 0; j < kVptB; ++j) {
      const int d = threadIdx.x + j * blockDim.x;
      if (d < D) {
        const float4 qv = QIO<T>::lds(sq + d * 4);
        const float4 gv = QIO<T>::lds(sg + d * 4);
        const float dldn = rs * (av[j] - ma - nh[j] * man) - nh[j] * av[j] * rdn[j];
        const float cg = gm[j] * nh[j] * rdn[j];
        const float cq = dldn * rcp_nr(nrm[j]);
        float4 o;
        o.x = fmaf(cg, gv.x, cq * qv.x);
        o.y = fmaf(cg, gv.y, cq * qv.y);
        o.z = fmaf(cg, gv.z, cq * qv.z);
        o.w = fmaf(cg, gv.w, cq * qv.w);
        QIO<T>::st_stream(dq + row * rlen + d * 4, o);
      }
    }
    if (nstage == 2) {
      s ^= 1;
    } else if (nxt < rows) {
      stage_row(nxt, 0);  // this thread has read all of its staged quaternions
    }
  }
  // partial layout: [parts][D] dgamma, then (16-byte aligned) [parts][D] float4 dbeta
  float* pg = partial + int64_t(blockIdx.x) * D;
  float4* pb = reinterpret_cast<float4*>(partial + beta_partial_offset(gridDim.x, D)) +
               int64_t(blockIdx.x) * D;
#pragma unroll
  for (int j = 0; j < kVptB; ++j) {
    const int d = threadIdx.x + j * blockDim.x;
    if (d < D) {
      pg[d] = dg[j];
      pb[d] = db[j];
    }
  }
}

// dgamma[d] = sum_c gamma_part[c][d]; dbeta[d][k] = sum_c beta_part[c][d][k]
__global__ void qln_bwd_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dgamma,
                                      float* __restrict__ dbeta, int nparts, int D) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // 0 .. 5D-1
  if (i >= 5 * D) return;
  float s = 0.f;
  if (i < D) {
    for (int c = 0; c < nparts; ++c) s += partial[int64_t(c) * D + i];
    dgamma[i] = s;
  } else {
    const float* pb = partial + beta_partial_offset(nparts, D);
    const int j = i - D;  // element of the [D][4] block
    for (int c = 0; c < nparts; ++c) s += pb[int64_t(c) * D * 4 + j];
    dbeta[j] = s;
  }
}

int qln_bwd_parts(int64_t rows) {
  int64_t p = int64_t(num_sms()) * 3;
  if (p > rows) p = rows;
  return p < 1 ? 1 : int(p);
}

}  // namespace
}  // namespace mqc

using namespace mqc;

extern "C" int mqc_qln_fwd(const void* q, const float* gamma, const float* beta, void* out,
                           float* mean, float* rstd, int64_t rows, int64_t d_model, float eps,
                           int flags, int dtype, void* stream) {
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_qln_fwd: unknown dtype %d", dtype);
  MQC_REQUIRE(rows >= 0 && d_model >= 0, MQC_ERR_INVALID_VALUE, "mqc_qln_fwd: negative size");
  MQC_REQUIRE((flags & ~MQC_QLN_PADDED_COMPAT) == 0, MQC_ERR_INVALID_VALUE,
              "mqc_qln_fwd: unknown flags 0x%x", flags);
  if (rows == 0) return MQC_OK;
  MQC_REQUIRE(d_model >= 1, MQC_ERR_INVALID_VALUE, "mqc_qln_fwd: d_model must be >= 1");
  MQC_REQUIRE(d_model <= int64_t(kMaxRowThreads) * kVpt, MQC_ERR_UNSUPPORTED,
              "mqc_qln_fwd: d_model=%lld > %d", (long long)d_model, kMaxRowThreads * kVpt);
  MQC_REQUIRE(rows <= 0x7fffffff, MQC_ERR_UNSUPPORTED, "mqc_qln_fwd: too many rows");
  MQC_REQUIRE(q && gamma && beta && out, MQC_ERR_INVALID_VALUE, "mqc_qln_fwd: null pointer");
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(q, al) && aligned(out, al) && aligned(beta, 16), MQC_ERR_MISALIGNED,
              "mqc_qln_fwd: q/out must be %d-byte and beta 16-byte aligned", int(al));
  const int D = int(d_model);
  int threads = (D + kVpt - 1) / kVpt;
  threads = (threads + 31) / 32 * 32;
  if (threads < 32) threads = 32;
  int pad = 0;
  if (flags & MQC_QLN_PADDED_COMPAT) {
    int block = 1;
    while (block < D) block <<= 1;
    pad = block - D;
  }
  cudaStream_t st = as_stream(stream);
  const size_t srow_bytes = size_t(D) * 4 * (dtype == MQC_DTYPE_F32 ? 4 : 2);
  if (srow_bytes + 1024 > 48 * 1024) {  // (the static reduction buffer counts too)
    cudaError_t e = dtype == MQC_DTYPE_F32
                        ? cudaFuncSetAttribute(qln_fwd_kernel<float>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(srow_bytes))
                        : cudaFuncSetAttribute(qln_fwd_kernel<__nv_bfloat16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(srow_bytes));
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "mqc_qln_fwd: smem attribute (%zu B): %s", srow_bytes,
                  cudaGetErrorString(e));
  }
  if (dtype == MQC_DTYPE_F32) {
    qln_fwd_kernel<float><<<unsigned(rows), threads, srow_bytes, st>>>(
        static_cast<const float*>(q), gamma, beta, static_cast<float*>(out), mean, rstd, D, eps,
        pad);
  } else {
    qln_fwd_kernel<__nv_bfloat16><<<unsigned(rows), threads, srow_bytes, st>>>(
        static_cast<const __nv_bfloat16*>(q), gamma, beta, static_cast<__nv_bfloat16*>(out), mean,
        rstd, D, eps, pad);
  }
  return check_launch("mqc_qln_fwd");
}

namespace mqc {

// Mean and 1/std of the quaternion norms of every row: the first half of
// mqc_qln_fwd (same kernel, same arithmetic, so the statistics are bit for bit
// those the LayerNorm itself uses), without writing the normalised row.
int qln_row_stats(const void* q, float* mean, float* rstd, int64_t rows, int64_t d_model,
                  float eps, int dtype, cudaStream_t st) {
  MQC_REQUIRE(d_model >= 1 && d_model <= int64_t(kMaxRowThreads) * kVpt && rows <= 0x7fffffff,
              MQC_ERR_UNSUPPORTED, "qln_row_stats: d_model=%lld", (long long)d_model);
  const int D = int(d_model);
  int threads = (D + kVpt - 1) / kVpt;
  threads = (threads + 31) / 32 * 32;
  if (threads < 32) threads = 32;
  const size_t srow_bytes = size_t(D) * 4 * (dtype == MQC_DTYPE_F32 ? 4 : 2);
  if (srow_bytes + 1024 > 48 * 1024) {  // (the static reduction buffer counts too)
    cudaError_t e = dtype == MQC_DTYPE_F32
                        ? cudaFuncSetAttribute(qln_fwd_kernel<float>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(srow_bytes))
                        : cudaFuncSetAttribute(qln_fwd_kernel<__nv_bfloat16>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(srow_bytes));
    if (e != cudaSuccess)
      return fail(MQC_ERR_CUDA, "qln_row_stats: smem attribute: %s", cudaGetErrorString(e));
  }
  if (rows == 0) return MQC_OK;
  if (dtype == MQC_DTYPE_F32)
    qln_fwd_kernel<float><<<unsigned(rows), threads, srow_bytes, st>>>(
        static_cast<const float*>(q), nullptr, nullptr, nullptr, mean, rstd, D, eps, 0);
  else
    qln_fwd_kernel<__nv_bfloat16><<<unsigned(rows), threads, srow_bytes, st>>>(
        static_cast<const __nv_bfloat16*>(q), nullptr, nullptr, nullptr, mean, rstd, D, eps, 0);
  return check_launch("qln_row_stats");
}

}  // namespace mqc

extern "C" size_t mqc_qln_bwd_workspace_size(int64_t rows, int64_t d_model) {
  if (rows <= 0 || d_model <= 0) return 0;
  const int64_t parts = qln_bwd_parts(rows);
  return size_t(beta_partial_offset(parts, d_model) + parts * d_model * 4) * sizeof(float);
}

extern "C" int mqc_qln_bwd(const void* q, const float* gamma, const void* dout, const float* mean,
                           const float* rstd, void* dq, float* dgamma, float* dbeta,
                           void* workspace, size_t workspace_bytes, int64_t rows, int64_t d_model,
                           float eps, int dtype, void* stream) {
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_qln_bwd: unknown dtype %d", dtype);
  MQC_REQUIRE(rows >= 0 && d_model >= 1, MQC_ERR_INVALID_VALUE, "mqc_qln_bwd: bad size");
  MQC_REQUIRE(d_model <= 1024 * kVptB, MQC_ERR_UNSUPPORTED, "mqc_qln_bwd: d_model=%lld > %d",
              (long long)d_model, 1024 * kVptB);
  MQC_REQUIRE(q && gamma && dout && mean && rstd && dq && dgamma && dbeta, MQC_ERR_INVALID_VALUE,
              "mqc_qln_bwd: null pointer");
  const size_t need = mqc_qln_bwd_workspace_size(rows, d_model);
  MQC_REQUIRE(rows == 0 || (workspace != nullptr && workspace_bytes >= need), MQC_ERR_INVALID_VALUE,
              "mqc_qln_bwd: workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(q, al) && aligned(dout, al) && aligned(dq, al) && aligned(workspace, 16),
              MQC_ERR_MISALIGNED, "mqc_qln_bwd: misaligned pointer");
  const int D = int(d_model);
  cudaStream_t st = as_stream(stream);
  if (rows == 0) {
    cudaMemsetAsync(dgamma, 0, size_t(D) * 4, st);
    cudaMemsetAsync(dbeta, 0, size_t(D) * 16, st);
    return check_launch("mqc_qln_bwd");
  }
  int threads = (D + kVptB - 1) / kVptB;
  threads = (threads + 31) / 32 * 32;
  const int parts = qln_bwd_parts(rows);
  float* partial = static_cast<float*>(workspace);
  const bool wide = threads > 512;
  // two staged rows of q and dout where they fit in 100 KB (two CTAs per SM at
  // least), else one
  const size_t row_bytes = size_t(D) * 4 * (dtype == MQC_DTYPE_F32 ? 4 : 2);
  const int nstage = 4 * row_bytes <= 100 * 1024 ? 2 : 1;
  const size_t smem = size_t(nstage) * 2 * row_bytes;
  auto launch = [&](auto kern, auto tq) -> int {
    using TT = std::remove_const_t<std::remove_pointer_t<decltype(tq)>>;
    if (smem + 1024 > 48 * 1024) {  // (the static reduction buffer counts too)
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(smem));
      if (e != cudaSuccess)
        return fail(MQC_ERR_CUDA, "mqc_qln_bwd: smem attribute (%zu B): %s", smem,
                    cudaGetErrorString(e));
    }
    kern<<<parts, threads, smem, st>>>(static_cast<const TT*>(q), gamma,
                                       static_cast<const TT*>(dout), mean, rstd,
                                       static_cast<TT*>(dq), partial, rows, D, eps, nstage);
    return MQC_OK;
  };
  int rc;
  if (dtype == MQC_DTYPE_F32)
    rc = launch(wide ? qln_bwd_kernel<float, 1024> : qln_bwd_kernel<float, 512>,
                static_cast<const float*>(nullptr));
  else
    rc = launch(wide ? qln_bwd_kernel<__nv_bfloat16, 1024> : qln_bwd_kernel<__nv_bfloat16, 512>,
                static_cast<const __nv_bfloat16*>(nullptr));
  if (rc != MQC_OK) return rc;
  qln_bwd_reduce_kernel<<<(5 * D + 255) / 256, 256, 0, st>>>(partial, dgamma, dbeta, parts, D);
  return check_launch("mqc_qln_bwd");
}
