// Shared device helpers for the mambaqc_b200 sm_100a kernels.
//
// Quaternions are 4 contiguous scalars (r, i, j, k) -- the reference's
// [..., 4] last axis. fp32 quaternions move as one 16-byte vector, bf16
// quaternions as one 8-byte vector; arithmetic is always fp32.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "mambaqc_b200.h"

namespace mqc {

// ---------------------------------------------------------------------------
// Loads / stores of one quaternion in the storage type
// ---------------------------------------------------------------------------

template <typename T> struct QIO;

template <> struct QIO<float> {
  static __device__ __forceinline__ float4 ld(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
  }
  static __device__ __forceinline__ float4 ld_stream(const float* p) {
    return __ldcs(reinterpret_cast<const float4*>(p));
  }
  static __device__ __forceinline__ float4 lds(const float* p) {
    return *reinterpret_cast<const float4*>(p);
  }
  static __device__ __forceinline__ void st(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
  }
  static __device__ __forceinline__ void st_stream(float* p, float4 v) {
    __stcs(reinterpret_cast<float4*>(p), v);
  }
  static __device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ void st1(float* p, float v) { *p = v; }
};

template <> struct QIO<__nv_bfloat16> {
  static __device__ __forceinline__ float4 unpack(uint2 u) {
    float4 v;
    v.x = __uint_as_float(u.x << 16);
    v.y = __uint_as_float(u.x & 0xffff0000u);
    v.z = __uint_as_float(u.y << 16);
    v.w = __uint_as_float(u.y & 0xffff0000u);
    return v;
  }
  static __device__ __forceinline__ uint2 pack(float4 v) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    return u;
  }
  static __device__ __forceinline__ float4 ld(const __nv_bfloat16* p) {
    return unpack(__ldg(reinterpret_cast<const uint2*>(p)));
  }
  static __device__ __forceinline__ float4 ld_stream(const __nv_bfloat16* p) {
    return unpack(__ldcs(reinterpret_cast<const uint2*>(p)));
  }
  static __device__ __forceinline__ float4 lds(const __nv_bfloat16* p) {
    return unpack(*reinterpret_cast<const uint2*>(p));
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = pack(v);
  }
  static __device__ __forceinline__ void st_stream(__nv_bfloat16* p, float4 v) {
    __stcs(reinterpret_cast<uint2*>(p), pack(v));
  }
  static __device__ __forceinline__ float ld1(const __nv_bfloat16* p) {
    return __bfloat162float(__ldg(p));
  }
  static __device__ __forceinline__ void st1(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
  }
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// ---------------------------------------------------------------------------
// Quaternion arithmetic (Hamilton product convention of the reference,
// mambaqc/kernels/quaternion_ops.py:66-69)
// ---------------------------------------------------------------------------

// p (x) q
__device__ __forceinline__ float4 qmul(float4 p, float4 q) {
  float4 r;
  r.x = fmaf(p.x, q.x, fmaf(-p.y, q.y, fmaf(-p.z, q.z, -p.w * q.w)));
  r.y = fmaf(p.x, q.y, fmaf(p.y, q.x, fmaf(p.z, q.w, -p.w * q.z)));
  r.z = fmaf(p.x, q.z, fmaf(-p.y, q.w, fmaf(p.z, q.x, p.w * q.y)));
  r.w = fmaf(p.x, q.w, fmaf(p.y, q.z, fmaf(-p.z, q.y, p.w * q.x)));
  return r;
}

// acc + p (x) q
__device__ __forceinline__ float4 qmul_acc(float4 p, float4 q, float4 acc) {
  float4 r;
  r.x = fmaf(p.x, q.x, fmaf(-p.y, q.y, fmaf(-p.z, q.z, fmaf(-p.w, q.w, acc.x))));
  r.y = fmaf(p.x, q.y, fmaf(p.y, q.x, fmaf(p.z, q.w, fmaf(-p.w, q.z, acc.y))));
  r.z = fmaf(p.x, q.z, fmaf(-p.y, q.w, fmaf(p.z, q.x, fmaf(p.w, q.y, acc.z))));
  r.w = fmaf(p.x, q.w, fmaf(p.y, q.z, fmaf(-p.z, q.y, fmaf(p.w, q.x, acc.w))));
  return r;
}

__device__ __forceinline__ float4 qconj(float4 q) { return make_float4(q.x, -q.y, -q.z, -q.w); }

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }

// 1/d for normal, finite d: the hardware reciprocal approximation
// (rcp.approx.ftz.f32) refined by one Newton-Raphson step for f(r) = 1/r - d,
// r' = r + r (1 - d r). Branch-free; for d in the normal range the refined
// value is within about one ulp of 1/d (the Cayley kernels built on it are
// checked against the fp64 oracle over denominators spanning 1e-6 .. 1e6 in
// tests/test_gpu_ops.py::test_cayley_denominator_sweep).
__device__ __forceinline__ float rcp_nr(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float e = fmaf(-d, r, 1.f);
  return fmaf(r, e, r);
}

// Cayley map q = (1 - z/2)^-1 (x) (1 + z/2) in closed form.
//
// With w = z/2 = a + v (v pure), conj(1 - w) (x) (1 + w) = (1 - a^2 - |v|^2) + 2v,
// and |1 - w|^2 = (1 - a)^2 + |v|^2, clamped below by eps exactly as the
// reference clamps |den|^2 (cayley_transform.py:106-108). 2v = Im z.
__device__ __forceinline__ float4 cayley_closed(float4 z, float eps) {
  const float a = 0.5f * z.x;
  const float om = 1.f - a;
  const float op = 1.f + a;
  const float vv = 0.25f * fmaf(z.y, z.y, fmaf(z.z, z.z, z.w * z.w));
  const float den = fmaxf(fmaf(om, om, vv), eps);
  const float inv = rcp_nr(den);
  return make_float4(fmaf(om, op, -vv) * inv, z.y * inv, z.z * inv, z.w * inv);
}

// Vector-Jacobian product of cayley_closed: given z and g = dL/dq, returns dL/dz.
// With w = z/2 = (a, v), den = (1-a)^2 + |v|^2, D = max(den, eps),
// num_r = (1-a)(1+a) - |v|^2, q = (num_r, 2v) / D, and u = 1 where the clamp is
// inactive (den >= eps), u = 0 where it is (D is then the constant eps):
//   dq_r/da = -2a/D + u 2(1-a) num_r/D^2     dq_r/dv = -2v/D - u 2 num_r v/D^2
//   dq_v/da = u 4(1-a) v/D^2                 dq_v/dv = 2I/D - u 4 v v^T/D^2
// Branch-free; dz = (dL/da, dL/dv) / 2.
__device__ __forceinline__ float4 cayley_vjp(float4 z, float4 g, float eps) {
  const float a = 0.5f * z.x;
  const float v1 = 0.5f * z.y, v2 = 0.5f * z.z, v3 = 0.5f * z.w;
  const float om = 1.f - a;
  const float vv = fmaf(v1, v1, fmaf(v2, v2, v3 * v3));
  const float den = fmaf(om, om, vv);
  const float D = fmaxf(den, eps);
  const float inv = rcp_nr(D);
  const float w = den >= eps ? inv * inv : 0.f;
  const float num_r = fmaf(om, 1.f + a, -vv);
  const float gv = fmaf(g.y, v1, fmaf(g.z, v2, g.w * v3));
  // halves folded in: dz = 0.5 * (dL/da, dL/dv)
  const float hw = w * om;
  const float da = fmaf(g.x, fmaf(hw, num_r, -a * inv), 2.f * hw * gv);
  const float cv = -(g.x * fmaf(w, num_r, inv) + 2.f * w * gv);  // coefficient of v
  return make_float4(da, fmaf(cv, v1, g.y * inv), fmaf(cv, v2, g.z * inv), fmaf(cv, v3, g.w * inv));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA engine) wrappers, hand-written PTX.
// Local, non-multicast copies only.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// One contiguous global -> shared copy on the bulk-copy (TMA) engine; completion
// is signalled on `bar` as transaction bytes. dst, src and bytes: multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Plain arrive (count 1), release semantics at CTA scope.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: gives up after `limit` polls and returns false. Never spins forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit) {
  for (long long i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// Poll limit used to drain copies still in flight on an error path.
constexpr long long kDrainPollLimit = 1ll << 22;

// 4-byte asynchronous global -> shared copy (LDGSTS) that bypasses registers;
// with `valid` false nothing is read and the 4 destination bytes are zero-filled.
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
// 16-byte variant (both addresses 16-byte aligned), zero-filled when !valid.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
// Waits until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) atomicOr(status, code);
}

}  // namespace mqc
