// Packed two-lane FP32 quaternion arithmetic for sm_100 (fma/mul/add .rn.f32x2).
//
// A QPair holds two quaternions component-interleaved, x = (q0.x, q1.x), ...;
// every operation runs both through one packed instruction per scalar
// instruction of the unpacked formula, in the same order, so each half rounds
// exactly like the scalar code. Negated halves and broadcast scalar operands are
// free operand forms of the packed instructions (swapped halves are not), so the
// helpers below only ever negate or broadcast.
#pragma once

#include "mqc_common.cuh"

namespace mqc {
namespace pk {

__device__ __forceinline__ float2 bc2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// Two quaternions, component-interleaved: x = (q0.x, q1.x), ...
struct QPair {
  float2 x, y, z, w;
};

__device__ __forceinline__ QPair qp_zero() {
  const float2 z = make_float2(0.f, 0.f);
  return QPair{z, z, z, z};
}

// p (x) h + acc for both halves (the scalar qmul_acc, one packed op per FMA).
__device__ __forceinline__ QPair qp_mul_acc(const QPair& p, const QPair& h, const QPair& a) {
  QPair r;
  r.x = fma2(p.x, h.x, fma2(neg2(p.y), h.y, fma2(neg2(p.z), h.z, fma2(neg2(p.w), h.w, a.x))));
  r.y = fma2(p.x, h.y, fma2(p.y, h.x, fma2(p.z, h.w, fma2(neg2(p.w), h.z, a.y))));
  r.z = fma2(p.x, h.z, fma2(neg2(p.y), h.w, fma2(p.z, h.x, fma2(p.w, h.y, a.z))));
  r.w = fma2(p.x, h.w, fma2(p.y, h.z, fma2(neg2(p.z), h.y, fma2(p.w, h.x, a.w))));
  return r;
}

// p (x) s with s the same quaternion for both halves (the scalar qmul). The
// broadcast scalar is the first multiplicand of every packed op (the operand
// slot where a broadcast is free); a*b == b*a exactly, so the rounding is that
// of the scalar formula.
__device__ __forceinline__ QPair qp_mul_bcast(const QPair& p, float4 s) {
  QPair r;
  r.x = fma2(bc2(s.x), p.x, fma2(bc2(-s.y), p.y, fma2(bc2(-s.z), p.z, mul2(bc2(-s.w), p.w))));
  r.y = fma2(bc2(s.y), p.x, fma2(bc2(s.x), p.y, fma2(bc2(s.w), p.z, mul2(bc2(-s.z), p.w))));
  r.z = fma2(bc2(s.z), p.x, fma2(bc2(-s.w), p.y, fma2(bc2(s.x), p.z, mul2(bc2(s.y), p.w))));
  r.w = fma2(bc2(s.w), p.x, fma2(bc2(s.z), p.y, fma2(bc2(-s.y), p.z, mul2(bc2(s.x), p.w))));
  return r;
}

__device__ __forceinline__ float2 rcp_nr2(float2 d) {
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  const float2 e = fma2(neg2(d), r, bc2(1.f));
  return fma2(r, e, r);
}

// Per-(d, n) Cayley constants of a state pair (lr, Im Lambda, m = |Lambda|^2 / 4).
struct LamPair {
  float2 lr, li, lj, lk, m;
};

// cayley_from_const (ssm_scan_common.cuh) for both halves; *s_out (if given)
// receives delta / den, the factor of Im Lambda in q.
__device__ __forceinline__ QPair cayley_pair(float dl, float dl2, const LamPair& c, float eps,
                                             float2* s_out = nullptr) {
  const float2 P = mul2(bc2(dl2), c.m);
  float2 den = fma2(bc2(-dl), c.lr, add2(bc2(1.f), P));
  den.x = fmaxf(den.x, eps);
  den.y = fmaxf(den.y, eps);
  const float2 inv = rcp_nr2(den);
  const float2 s = mul2(bc2(dl), inv);
  if (s_out != nullptr) *s_out = s;
  return QPair{fma2(neg2(P), inv, inv), mul2(s, c.li), mul2(s, c.lj), mul2(s, c.lk)};
}

// cayley_pair that also hands out 1 / max(den, eps) and the unclamped
// den = 1 + P - delta*lr, for cayley_vjp_pair_shared at the same step.
__device__ __forceinline__ QPair cayley_pair_keep(float dl, float dl2, const LamPair& c, float eps,
                                                  float2* inv_out, float2* den_out) {
  const float2 P = mul2(bc2(dl2), c.m);
  const float2 den = fma2(bc2(-dl), c.lr, add2(bc2(1.f), P));
  const float2 inv = rcp_nr2(make_float2(fmaxf(den.x, eps), fmaxf(den.y, eps)));
  const float2 s = mul2(bc2(dl), inv);
  *inv_out = inv;
  *den_out = den;
  return QPair{fma2(neg2(P), inv, inv), mul2(s, c.li), mul2(s, c.lj), mul2(s, c.lk)};
}

__device__ __forceinline__ float4 qp_half(const QPair& q, int e) {
  return e == 0 ? make_float4(q.x.x, q.y.x, q.z.x, q.w.x) : make_float4(q.x.y, q.y.y, q.z.y, q.w.y);
}

__device__ __forceinline__ void qp_set_half(QPair& q, int e, float4 v) {
  if (e == 0) {
    q.x.x = v.x; q.y.x = v.y; q.z.x = v.z; q.w.x = v.w;
  } else {
    q.x.y = v.x; q.y.y = v.y; q.z.y = v.z; q.w.y = v.w;
  }
}

// s (x) p with s the same quaternion for both halves.
__device__ __forceinline__ QPair qp_bmul(float4 s, const QPair& p) {
  QPair r;
  r.x = fma2(bc2(s.x), p.x, fma2(bc2(-s.y), p.y, fma2(bc2(-s.z), p.z, mul2(bc2(-s.w), p.w))));
  r.y = fma2(bc2(s.x), p.y, fma2(bc2(s.y), p.x, fma2(bc2(s.z), p.w, mul2(bc2(-s.w), p.z))));
  r.z = fma2(bc2(s.x), p.z, fma2(bc2(-s.y), p.w, fma2(bc2(s.z), p.x, mul2(bc2(s.w), p.y))));
  r.w = fma2(bc2(s.x), p.w, fma2(bc2(s.y), p.z, fma2(bc2(-s.z), p.y, mul2(bc2(s.w), p.x))));
  return r;
}

__device__ __forceinline__ QPair qp_conj(const QPair& q) {
  return QPair{q.x, neg2(q.y), neg2(q.z), neg2(q.w)};
}

__device__ __forceinline__ float2 qp_dot(const QPair& a, const QPair& b) {
  return fma2(a.x, b.x, fma2(a.y, b.y, fma2(a.z, b.z, mul2(a.w, b.w))));
}

// QPair from two quaternions (state-wise float4 each).
__device__ __forceinline__ QPair qp_from(float4 a, float4 b) {
  return QPair{make_float2(a.x, b.x), make_float2(a.y, b.y), make_float2(a.z, b.z),
               make_float2(a.w, b.w)};
}

// cayley_vjp (mqc_common.cuh) for both halves, same operations in the same order.
__device__ __forceinline__ QPair cayley_vjp_pair(const QPair& z, const QPair& g, float eps) {
  const float2 h = bc2(0.5f);
  const float2 a = mul2(h, z.x);
  const float2 v1 = mul2(h, z.y), v2 = mul2(h, z.z), v3 = mul2(h, z.w);
  const float2 om = add2(bc2(1.f), neg2(a));
  const float2 vv = fma2(v1, v1, fma2(v2, v2, mul2(v3, v3)));
  const float2 den = fma2(om, om, vv);
  const float2 Dd = make_float2(fmaxf(den.x, eps), fmaxf(den.y, eps));
  const float2 inv = rcp_nr2(Dd);
  float2 w = mul2(inv, inv);
  w.x = den.x >= eps ? w.x : 0.f;
  w.y = den.y >= eps ? w.y : 0.f;
  const float2 num_r = fma2(om, add2(bc2(1.f), a), neg2(vv));
  const float2 gv = fma2(g.y, v1, fma2(g.z, v2, mul2(g.w, v3)));
  const float2 hw = mul2(w, om);
  const float2 da = fma2(g.x, fma2(hw, num_r, neg2(mul2(a, inv))), mul2(mul2(bc2(2.f), hw), gv));
  const float2 cv = neg2(add2(mul2(g.x, fma2(w, num_r, inv)), mul2(mul2(bc2(2.f), w), gv)));
  return QPair{da, fma2(cv, v1, mul2(g.y, inv)), fma2(cv, v2, mul2(g.z, inv)),
               fma2(cv, v3, mul2(g.w, inv))};
}

// cayley_vjp_pair for z = delta * Lambda, given the reciprocal and unclamped
// denominator of the forward map at the same step (cayley_pair_keep):
// |1 - z/2|^2 = (1 - a)^2 + |v|^2 = 1 + P - delta*lr is that denominator, so no
// second reciprocal is taken, and a, v come from delta/2 directly. Same
// formulas as cayley_vjp_pair otherwise.
__device__ __forceinline__ QPair cayley_vjp_pair_shared(float dl, const LamPair& c, float2 inv,
                                                        float2 den, const QPair& g, float eps) {
  const float2 hd = bc2(0.5f * dl);
  const float2 a = mul2(hd, c.lr);
  const float2 v1 = mul2(hd, c.li), v2 = mul2(hd, c.lj), v3 = mul2(hd, c.lk);
  const float2 om = add2(bc2(1.f), neg2(a));
  const float2 vv = fma2(v1, v1, fma2(v2, v2, mul2(v3, v3)));
  float2 w = mul2(inv, inv);
  w.x = den.x >= eps ? w.x : 0.f;
  w.y = den.y >= eps ? w.y : 0.f;
  const float2 num_r = fma2(om, add2(bc2(1.f), a), neg2(vv));
  const float2 gv = fma2(g.y, v1, fma2(g.z, v2, mul2(g.w, v3)));
  const float2 hw = mul2(w, om);
  const float2 da = fma2(g.x, fma2(hw, num_r, neg2(mul2(a, inv))), mul2(mul2(bc2(2.f), hw), gv));
  const float2 cv = neg2(add2(mul2(g.x, fma2(w, num_r, inv)), mul2(mul2(bc2(2.f), w), gv)));
  return QPair{da, fma2(cv, v1, mul2(g.y, inv)), fma2(cv, v2, mul2(g.z, inv)),
               fma2(cv, v3, mul2(g.w, inv))};
}

}  // namespace pk
}  // namespace mqc
