// Elementwise quaternion kernels: Hamilton product, conjugate, inverse, norm and
// the Cayley map. All are HBM-streaming: each thread moves UNROLL quaternions
// per operand per iteration with 16-byte (fp32) / 8-byte (bf16) vector loads,
// all loads issued before any store, over a grid of a few CTAs per SM.
//
// Reference counterparts: mambaqc/kernels/quaternion_ops.py:259-461 and
// mambaqc/kernels/cayley_transform.py:132-195.
#include "mqc_common.cuh"
#include "mqc_host.h"

namespace mqc {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct OpMul {
  __device__ float4 operator()(float4 p, float4 q) const { return qmul(p, q); }
};
struct OpConj {
  __device__ float4 operator()(float4 q) const { return qconj(q); }
};
struct OpInv {
  float eps;
  __device__ float4 operator()(float4 q) const {
    const float n2 = fmaxf(fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, q.w * q.w))), eps);
    return make_float4(q.x / n2, -q.y / n2, -q.z / n2, -q.w / n2);
  }
};
struct OpCayley {
  float eps;
  __device__ float4 operator()(float4 z) const { return cayley_closed(z, eps); }
};
struct OpCayleyVjp {
  float eps;
  __device__ float4 operator()(float4 z, float4 g) const { return cayley_vjp(z, g, eps); }
};

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) binary_kernel(const T* __restrict__ a,
                                                          const T* __restrict__ b,
                                                          T* __restrict__ out, int64_t n, Op op) {
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t base = int64_t(blockIdx.x) * kThreads + threadIdx.x; base < n;
       base += stride * kUnroll) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) {
        va[u] = QIO<T>::ld_stream(a + 4 * i);
        vb[u] = QIO<T>::ld_stream(b + 4 * i);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) QIO<T>::st_stream(out + 4 * i, op(va[u], vb[u]));
    }
  }
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) unary_kernel(const T* __restrict__ a,
                                                         T* __restrict__ out, int64_t n, Op op) {
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t base = int64_t(blockIdx.x) * kThreads + threadIdx.x; base < n;
       base += stride * kUnroll) {
    float4 va[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) va[u] = QIO<T>::ld_stream(a + 4 * i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) QIO<T>::st_stream(out + 4 * i, op(va[u]));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) norm_kernel(const T* __restrict__ a,
                                                        T* __restrict__ out, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t base = int64_t(blockIdx.x) * kThreads + threadIdx.x; base < n;
       base += stride * kUnroll) {
    float4 va[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) va[u] = QIO<T>::ld_stream(a + 4 * i);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      if (i < n) {
        const float4 q = va[u];
        QIO<T>::st1(out + i,
                    sqrtf(fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, q.w * q.w)))));
      }
    }
  }
}

int grid_for(int64_t n) {
  const int64_t per_cta = int64_t(kThreads) * kUnroll;
  int64_t g = (n + per_cta - 1) / per_cta;
  const int64_t cap = int64_t(num_sms()) * 8;  // 8 CTAs x 256 threads = full SM
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return int(g);
}

template <typename Op>
int launch_binary(const void* a, const void* b, void* out, int64_t n, int dtype, void* stream,
                  Op op, const char* name) {
  if (n == 0) return MQC_OK;
  const int g = grid_for(n);
  if (dtype == MQC_DTYPE_F32) {
    binary_kernel<float, Op><<<g, kThreads, 0, as_stream(stream)>>>(
        static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out), n,
        op);
  } else {
    binary_kernel<__nv_bfloat16, Op><<<g, kThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
        static_cast<__nv_bfloat16*>(out), n, op);
  }
  return check_launch(name);
}

template <typename Op>
int launch_unary(const void* a, void* out, int64_t n, int dtype, void* stream, Op op,
                 const char* name) {
  if (n == 0) return MQC_OK;
  const int g = grid_for(n);
  if (dtype == MQC_DTYPE_F32) {
    unary_kernel<float, Op><<<g, kThreads, 0, as_stream(stream)>>>(
        static_cast<const float*>(a), static_cast<float*>(out), n, op);
  } else {
    unary_kernel<__nv_bfloat16, Op><<<g, kThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(a), static_cast<__nv_bfloat16*>(out), n, op);
  }
  return check_launch(name);
}

int check_common(const void* a, const void* out, int64_t n, int dtype, const char* name) {
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "%s: unknown dtype %d", name, dtype);
  MQC_REQUIRE(n >= 0, MQC_ERR_INVALID_VALUE, "%s: negative n", name);
  if (n == 0) return MQC_OK;
  MQC_REQUIRE(a != nullptr && out != nullptr, MQC_ERR_INVALID_VALUE, "%s: null pointer", name);
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(a, al) && aligned(out, al), MQC_ERR_MISALIGNED,
              "%s: quaternion pointers must be %d-byte aligned", name, int(al));
  return MQC_OK;
}

}  // namespace
}  // namespace mqc

using namespace mqc;

extern "C" int mqc_qmul(const void* p, const void* q, void* out, int64_t n, int dtype,
                        void* stream) {
  clear_error();
  int rc = check_common(p, out, n, dtype, "mqc_qmul");
  if (rc != MQC_OK) return rc;
  if (n > 0) {
    MQC_REQUIRE(q != nullptr, MQC_ERR_INVALID_VALUE, "mqc_qmul: null q");
    MQC_REQUIRE(aligned(q, dtype == MQC_DTYPE_F32 ? 16 : 8), MQC_ERR_MISALIGNED,
                "mqc_qmul: q misaligned");
  }
  return launch_binary(p, q, out, n, dtype, stream, OpMul{}, "mqc_qmul");
}

extern "C" int mqc_qconj(const void* q, void* out, int64_t n, int dtype, void* stream) {
  clear_error();
  int rc = check_common(q, out, n, dtype, "mqc_qconj");
  if (rc != MQC_OK) return rc;
  return launch_unary(q, out, n, dtype, stream, OpConj{}, "mqc_qconj");
}

extern "C" int mqc_qinv(const void* q, void* out, int64_t n, float eps, int dtype,
                        void* stream) {
  clear_error();
  int rc = check_common(q, out, n, dtype, "mqc_qinv");
  if (rc != MQC_OK) return rc;
  return launch_unary(q, out, n, dtype, stream, OpInv{eps}, "mqc_qinv");
}

extern "C" int mqc_cayley(const void* z, void* q, int64_t n, float eps, int dtype,
                          void* stream) {
  clear_error();
  int rc = check_common(z, q, n, dtype, "mqc_cayley");
  if (rc != MQC_OK) return rc;
  return launch_unary(z, q, n, dtype, stream, OpCayley{eps}, "mqc_cayley");
}

extern "C" int mqc_cayley_bwd(const void* z, const void* dq, void* dz, int64_t n, float eps,
                              int dtype, void* stream) {
  clear_error();
  int rc = check_common(z, dz, n, dtype, "mqc_cayley_bwd");
  if (rc != MQC_OK) return rc;
  if (n > 0) {
    MQC_REQUIRE(dq != nullptr, MQC_ERR_INVALID_VALUE, "mqc_cayley_bwd: null dq");
    MQC_REQUIRE(aligned(dq, dtype == MQC_DTYPE_F32 ? 16 : 8), MQC_ERR_MISALIGNED,
                "mqc_cayley_bwd: dq misaligned");
  }
  return launch_binary(z, dq, dz, n, dtype, stream, OpCayleyVjp{eps}, "mqc_cayley_bwd");
}

extern "C" int mqc_qnorm(const void* q, void* out, int64_t n, int dtype, void* stream) {
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_qnorm: unknown dtype %d", dtype);
  MQC_REQUIRE(n >= 0, MQC_ERR_INVALID_VALUE, "mqc_qnorm: negative n");
  if (n == 0) return MQC_OK;
  MQC_REQUIRE(q != nullptr && out != nullptr, MQC_ERR_INVALID_VALUE, "mqc_qnorm: null pointer");
  MQC_REQUIRE(aligned(q, dtype == MQC_DTYPE_F32 ? 16 : 8), MQC_ERR_MISALIGNED,
              "mqc_qnorm: q misaligned");
  const int g = grid_for(n);
  if (dtype == MQC_DTYPE_F32) {
    norm_kernel<float><<<g, kThreads, 0, as_stream(stream)>>>(static_cast<const float*>(q),
                                                             static_cast<float*>(out), n);
  } else {
    norm_kernel<__nv_bfloat16><<<g, kThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), n);
  }
  return check_launch("mqc_qnorm");
}
