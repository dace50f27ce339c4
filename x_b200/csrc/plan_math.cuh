// Bit-exact index arithmetic of the pair plan (atl/ops/functional.py:139-175), shared by the plan
// builder, the pair kernels and the fused objective path.  Every expression rounds exactly as the
// torch eager op it restates (fp32 ops with Python scalars rounded to fp32 first).
#pragma once
#include "common.cuh"

namespace atlb {

struct PlanConsts {
  float tau_f, hd_f, delta_f;  // tau, delta/2, delta = 1/S (rounded to fp32)
  float ox_f, oy_f, cell_f;    // grid origin and cell size (rounded to fp32)
  float rcell_f;               // RN(1 / cell_f), the fp32 division
  long long GW, GH;
  int S;
  long long B;
  long long src0, src1;  // events that are sources of the pair sums (fused path), [src0, src1)
  float rfine_f;         // fused path: kFine / cell, the reciprocal of the sub-cell size
  long long GWf, GHf;    // fused path: sub-cells per row / sub-cell rows of a plane (GW, GH times kFine)
};

// The fused path splits every plan cell into kFine x kFine sub-cells (pair_fine.cuh).
constexpr int kFine = 3;

// Sub-cell index along one axis of a point at coordinate p (grid origin o, rf = kFine / cell) whose plan cell
// index is q (exact): floor((p - o) rf) clamped into [q kFine, q kFine + kFine - 1].  Only the pair windows
// depend on it, and they carry a margin for its rounding; the clamp keeps the plan cells exact.
__device__ __forceinline__ int fine_index(float p, float o, float rf, int q) {
  const float u = (p - o) * rf;
  const int lo = q * kFine;
  return u == u ? (int)fmaxf(fminf(floorf(u), (float)(lo + kFine - 1)), (float)lo) : lo;
}

// torch's row norm of an (N,2) float32 tensor (vectorised last-dim reduction): sqrt(fma(y, y, x*x)).
__device__ __forceinline__ float row_norm(float x, float y) {
  return __fsqrt_rn(__fmaf_rn(y, y, __fmul_rn(x, x)));
}

// functional.py:151-152: s_lo = clamp(ceil((t - tau - delta/2)/delta - 0.5), 0, S-1), s_hi likewise.
__device__ __forceinline__ void slice_range(const PlanConsts& P, float t, int* lo, int* hi) {
  const float a = ceilf(sub_rn(div_rn(sub_rn(sub_rn(t, P.tau_f), P.hd_f), P.delta_f), 0.5f));
  const float b = floorf(sub_rn(div_rn(add_rn(add_rn(t, P.tau_f), P.hd_f), P.delta_f), 0.5f));
  const float smax = (float)(P.S - 1);
  *lo = (int)clampf(a, 0.f, smax);
  *hi = (int)clampf(b, 0.f, smax);
}

// functional.py:157: slice centre (s + 0.5) * delta in fp32.
__device__ __forceinline__ float slice_centre(const PlanConsts& P, int s) {
  return mul_rn(add_rn((float)s, 0.5f), P.delta_f);
}

// functional.py:158: transported position y = x + v (c_s - t) at the centre of slice s.
__device__ __forceinline__ void transported(const PlanConsts& P, float xj, float yj, float vx, float vy, float tj,
                                            int s, float* yx, float* yy) {
  const float dtc = sub_rn(slice_centre(P, s), tj);
  *yx = add_rn(xj, mul_rn(vx, dtc));
  *yy = add_rn(yj, mul_rn(vy, dtc));
}

// floorf(div_rn(a, c)) for c > 0, given rc = RN(1 / c), without the division in all but rare cases.
// q = RN(a * rc) differs from a / c by at most (2^-23 + 2^-48) |a / c| (the rounding of rc, then of the
// product), and RN(a / c) differs from a / c by at most 2^-24 |a / c|; so |q - RN(a / c)| < 1.6 * 2^-23 |q|.
// When q's distance to the nearest integer exceeds 2^-21 |q| (more than twice that), no integer lies between
// the two and floor(q) = floor(RN(a / c)); otherwise (and for NaN / infinite q) the quotient is computed.
__device__ __forceinline__ float floor_div(float a, float c, float rc) {
  const float q = __fmul_rn(a, rc);
  const float f = floorf(q);
  const float fr = __fsub_rn(q, f);              // exact: q - floor(q) for |q| < 2^23
  const float d = __fmul_rn(fabsf(q), 0x1p-21f);
  if (fr > d && fr < __fsub_rn(1.f, d)) return f;  // false for NaN and infinities
  return floorf(div_rn(a, c));
}

// functional.py:158-163: transported position and its cell key (-1 = dropped).
__device__ __forceinline__ long long source_key(const PlanConsts& P, float xj, float yj, float vx, float vy, float tj,
                                                long long bj, int s, float* yx_out, float* yy_out) {
  float yx, yy;
  transported(P, xj, yj, vx, vy, tj, s, &yx, &yy);
  *yx_out = yx;
  *yy_out = yy;
  const float qx = floor_div(sub_rn(yx, P.ox_f), P.cell_f, P.rcell_f);
  const float qy = floor_div(sub_rn(yy, P.oy_f), P.cell_f, P.rcell_f);
  // in-range tests on the integral float (NaN fails them, as the reference's int64 cast then does)
  if (!(qx >= 0.f && qx < (float)P.GW && qy >= 0.f && qy < (float)P.GH)) return -1;
  if (bj < 0 || bj >= P.B) return -1;  // batch index outside [0, B): no cell (the reference's key would overflow)
  const long long cx = (long long)qx, cy = (long long)qy;
  return ((bj * P.S + s) * P.GH + cy) * P.GW + cx;
}

// The sub-cell key of the fused path, ((b S + s) GHf + fy) GWf + fx, of a source at slice s (-1 = dropped,
// exactly when source_key drops it): the plan cell as source_key computes it, then the sub-cell inside it.
__device__ __forceinline__ int source_fine_key(const PlanConsts& P, float xj, float yj, float vx, float vy, float tj,
                                               long long bj, int s) {
  float yx, yy;
  transported(P, xj, yj, vx, vy, tj, s, &yx, &yy);
  const float qx = floor_div(sub_rn(yx, P.ox_f), P.cell_f, P.rcell_f);
  const float qy = floor_div(sub_rn(yy, P.oy_f), P.cell_f, P.rcell_f);
  if (!(qx >= 0.f && qx < (float)P.GW && qy >= 0.f && qy < (float)P.GH)) return -1;
  if (bj < 0 || bj >= P.B) return -1;
  const int fx = fine_index(yx, P.ox_f, P.rfine_f, (int)qx), fy = fine_index(yy, P.oy_f, P.rfine_f, (int)qy);
  return (int)((((long long)bj * P.S + s) * P.GHf + fy) * P.GWf + fx);
}

// functional.py:170-175: anchor grid g = b*S + clamp(floor(t/delta), 0, S-1) and clamped cell.
__device__ __forceinline__ void anchor_cell(const PlanConsts& P, float xa, float ya, float ta, long long ba,
                                            long long* g, long long* cx, long long* cy) {
  const int sa = (int)clampf(floorf(div_rn(ta, P.delta_f)), 0.f, (float)(P.S - 1));
  const float qx = floorf(div_rn(sub_rn(xa, P.ox_f), P.cell_f));
  const float qy = floorf(div_rn(sub_rn(ya, P.oy_f), P.cell_f));
  long long ix = qx != qx ? LLONG_MIN : (long long)qx;  // x86 cvttss2si gives INT64_MIN for NaN
  long long iy = qy != qy ? LLONG_MIN : (long long)qy;
  ix = ix < 0 ? 0 : (ix > P.GW - 1 ? P.GW - 1 : ix);
  iy = iy < 0 ? 0 : (iy > P.GH - 1 ? P.GH - 1 : iy);
  *g = ba * P.S + sa;
  *cx = ix;
  *cy = iy;
}

inline size_t align_up(size_t n, size_t a = 256) { return (n + a - 1) / a * a; }
inline void* align_ptr(void* p, size_t a = 256) { return (void*)(((uintptr_t)p + a - 1) / a * a); }

}  // namespace atlb
