// The pair test and kernel of the anchored sum (csrc/atl_cpu.cpp:181-196), rounding-exact.
#pragma once
#include "common.cuh"

namespace atlb {

struct PairConsts {
  float tau;     // (float)tau
  float r2max;   // cut*cut*h*h in fp32, left to right (atl_cpu.cpp:184)
  float inv2h2;  // 1 / (2 h h) in fp32 (atl_cpu.cpp:184)
  float invh2;   // 1 / (float)(h*h)   (atl_cpu.cpp:236)
  float k2;      // log2(e) / (2 h h): exp(-d2 / 2h^2) = 2^(-d2 * k2)
};

inline PairConsts make_pair_consts(double h, double tau, double cut) {
  const float hf = (float)h, cf = (float)cut;
  PairConsts C;
  C.tau = (float)tau;
  volatile float r = cf * cf;  // volatile: keep the reference's left-to-right rounding order
  r = r * hf;
  r = r * hf;
  C.r2max = r;
  volatile float d = 2.f * hf;
  d = d * hf;
  C.inv2h2 = 1.f / d;
  C.invh2 = 1.f / (float)(h * h);
  C.k2 = (float)(1.4426950408889634 / (2.0 * h * h));
  return C;
}

// dt = t_i - t_j; r = x_i - (y_j + v_j (t_i - c_s)); accepted iff |dt| <= tau and |r|^2 <= r2max.
// NaN inputs are accepted, as the reference's "skip if greater" tests accept them.
__device__ __forceinline__ bool pair_test(const PairConsts& C, float xi, float yi, float ti, float dti, float2 sy,
                                          float2 sv, float st, float* rx, float* ry, float* d2, float* dt) {
  *dt = sub_rn(ti, st);
  if (fabsf(*dt) > C.tau) return false;
  *rx = sub_rn(xi, add_rn(sy.x, mul_rn(sv.x, dti)));
  *ry = sub_rn(yi, add_rn(sy.y, mul_rn(sv.y, dti)));
  *d2 = add_rn(mul_rn(*rx, *rx), mul_rn(*ry, *ry));
  return !(*d2 > C.r2max);
}

__device__ __forceinline__ float pair_kernel(const PairConsts& C, float d2) { return expf(mul_rn(-d2, C.inv2h2)); }

// 2^x with the SFU (PTX ex2.approx: relative error below 2^-22).  exp(-d2 / 2h^2) as 2^(-d2 k2) differs
// from expf by < 1e-6 relative for the kernel's range d2 <= (cut h)^2.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// f = gS_i * k * dt / h^2, in the reference's order (atl_cpu.cpp:244).
__device__ __forceinline__ float pair_grad_factor(const PairConsts& C, float gi, float kern, float dt) {
  return mul_rn(mul_rn(mul_rn(gi, kern), dt), C.invh2);
}

// ---- packed fp32x2 arithmetic (sm_100: add/sub/mul .rn.f32x2, each lane rounded like the scalar op) ----
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 upk2(f32x2 r) {
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(r));
  return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// r = x_i - (y_j + v_j * dti) for both components, each op rounded as the reference's scalar code
// (atl_cpu.cpp:192-193); returns d^2 = rx*rx + ry*ry (atl_cpu.cpp:194) and r in *r.
// The products v_j * dti are scalar __fmul_rn: the code generator contracts a packed mul.rn.f32x2 followed
// by add.rn.f32x2 into one fused multiply-add (measured: y + v dt rounded once; an explicit packed fma with a
// -0 addend is folded the same way), which would change the acceptance of pairs at the cut; __fmul_rn is
// never contracted.  The squares may stay packed: their sum is __fadd_rn, which is never merged into an FMA.
__device__ __forceinline__ float residual2(f32x2 xi, f32x2 dti2, f32x2 y, f32x2 v, float2* r) {
  const float2 vv = upk2(v), dd = upk2(dti2);
  const f32x2 vd = pk2(__fmul_rn(vv.x, dd.x), __fmul_rn(vv.y, dd.y));
  const f32x2 rr = sub2(xi, add2(y, vd));
  *r = upk2(rr);
  const float2 sq = upk2(mul2(rr, rr));
  return add_rn(sq.x, sq.y);
}
// The same with the time difference dti as one scalar.
__device__ __forceinline__ float residual2s(f32x2 xi, float dti, f32x2 y, f32x2 v, float2* r) {
  const float2 vv = upk2(v);
  const f32x2 vd = pk2(__fmul_rn(vv.x, dti), __fmul_rn(vv.y, dti));
  const f32x2 rr = sub2(xi, add2(y, vd));
  *r = upk2(rr);
  const float2 sq = upk2(mul2(rr, rr));
  return add_rn(sq.x, sq.y);
}

}  // namespace atlb
