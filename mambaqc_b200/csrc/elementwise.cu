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

// Division by a fixed divisor d >= 1 of numerators below 2^31 with one
// multiply-high and a shift (Granlund & Montgomery, "Division by invariant
// integers using multiplication", 1994): s = ceil(log2 d),
// m = floor(2^32 (2^s - d) / d) + 1, x / d = (umulhi(x, m) + x) >> s.
struct FastDiv {
  uint32_t d, m, s;
  explicit FastDiv(uint32_t div = 1) : d(div), m(0), s(0) {
    while ((uint64_t(1) << s) < d) ++s;
    m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << s) - d)) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t x) const { return (__umulhi(x, m) + x) >> s; }
};

// Strided Hamilton product over a 4-axis index space (i0, i1, i2, i3), the
// [batch, seq_len, d_model, d_state] of the reference's batched multiply. p and
// q are addressed by per-axis element strides (quaternion axis contiguous); out
// is dense, so stores are coalesced. Rows (i0, i1) are walked by blockIdx.y,
// the inner (i2, i3) plane by x, kUnroll quaternions per thread in flight.
struct StridedArgs {
  int64_t ps[4], qs[4];
  uint32_t rows, inner;  // s0 * s1 and s2 * s3
  FastDiv div1, div3;    // by s1 and s3
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    qmul_strided_kernel(const T* __restrict__ p, const T* __restrict__ q, T* __restrict__ out,
                        const StridedArgs a) {
  const uint32_t stride = gridDim.x * kThreads;
  for (uint32_t r = blockIdx.y; r < a.rows; r += gridDim.y) {
    const uint32_t i0 = a.div1.div(r), i1 = r - i0 * a.div1.d;
    const int64_t prow = int64_t(i0) * a.ps[0] + int64_t(i1) * a.ps[1];
    const int64_t qrow = int64_t(i0) * a.qs[0] + int64_t(i1) * a.qs[1];
    T* orow = out + int64_t(r) * a.inner * 4;
    for (uint32_t base = blockIdx.x * kThreads + threadIdx.x; base < a.inner;
         base += stride * kUnroll) {
      float4 va[kUnroll], vb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const uint32_t j = base + u * stride;
        if (j < a.inner) {
          const uint32_t i2 = a.div3.div(j), i3 = j - i2 * a.div3.d;
          va[u] = QIO<T>::ld_stream(p + prow + int64_t(i2) * a.ps[2] + int64_t(i3) * a.ps[3]);
          vb[u] = QIO<T>::ld_stream(q + qrow + int64_t(i2) * a.qs[2] + int64_t(i3) * a.qs[3]);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const uint32_t j = base + u * stride;
        if (j < a.inner) QIO<T>::st_stream(orow + int64_t(j) * 4, qmul(va[u], vb[u]));
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

extern "C" int mqc_qmul_strided(const void* p, const void* q, void* out, const int64_t* shape,
                                const int64_t* p_strides, const int64_t* q_strides, int dtype,
                                void* stream) {
  clear_error();
  MQC_REQUIRE(dtype_ok(dtype), MQC_ERR_INVALID_VALUE, "mqc_qmul_strided: unknown dtype %d", dtype);
  MQC_REQUIRE(shape != nullptr && p_strides != nullptr && q_strides != nullptr,
              MQC_ERR_INVALID_VALUE, "mqc_qmul_strided: null shape or strides");
  int64_t n = 1;
  for (int k = 0; k < 4; ++k) {
    MQC_REQUIRE(shape[k] >= 0, MQC_ERR_INVALID_VALUE, "mqc_qmul_strided: negative extent");
    MQC_REQUIRE(p_strides[k] >= 0 && q_strides[k] >= 0 && p_strides[k] % 4 == 0 &&
                    q_strides[k] % 4 == 0,
                MQC_ERR_INVALID_VALUE,
                "mqc_qmul_strided: strides must be non-negative multiples of 4 elements");
    n *= shape[k];
  }
  if (n == 0) return MQC_OK;
  MQC_REQUIRE(p != nullptr && q != nullptr && out != nullptr, MQC_ERR_INVALID_VALUE,
              "mqc_qmul_strided: null pointer");
  const uintptr_t al = dtype == MQC_DTYPE_F32 ? 16 : 8;
  MQC_REQUIRE(aligned(p, al) && aligned(q, al) && aligned(out, al), MQC_ERR_MISALIGNED,
              "mqc_qmul_strided: quaternion pointers must be %d-byte aligned", int(al));
  const int64_t rows = shape[0] * shape[1], inner = shape[2] * shape[3];
  MQC_REQUIRE(rows < (int64_t(1) << 31) && inner < (int64_t(1) << 31), MQC_ERR_UNSUPPORTED,
              "mqc_qmul_strided: more than 2^31 rows or inner quaternions");
  StridedArgs a;
  for (int k = 0; k < 4; ++k) {
    a.ps[k] = p_strides[k];
    a.qs[k] = q_strides[k];
  }
  a.rows = uint32_t(rows);
  a.inner = uint32_t(inner);
  a.div1 = FastDiv(uint32_t(shape[1]));
  a.div3 = FastDiv(uint32_t(shape[3]));
  // x covers the inner plane, y the rows: about 8 CTAs per SM in all
  const int64_t per_cta = int64_t(kThreads) * kUnroll;
  int64_t gx = (inner + per_cta - 1) / per_cta;
  const int64_t want = int64_t(num_sms()) * 8;
  if (gx > want) gx = want;
  int64_t gy = (want + gx - 1) / gx;
  if (gy > rows) gy = rows;
  if (gy > 65535) gy = 65535;
  const dim3 grid{unsigned(gx), unsigned(gy), 1u};
  if (dtype == MQC_DTYPE_F32)
    qmul_strided_kernel<float><<<grid, kThreads, 0, as_stream(stream)>>>(
        static_cast<const float*>(p), static_cast<const float*>(q), static_cast<float*>(out), a);
  else
    qmul_strided_kernel<__nv_bfloat16><<<grid, kThreads, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(p), static_cast<const __nv_bfloat16*>(q),
        static_cast<__nv_bfloat16*>(out), a);
  return check_launch("mqc_qmul_strided");
}
