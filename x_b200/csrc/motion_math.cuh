// Motion fields linear at the event, evaluated with torch's eager CPU rounding sequence.
#pragma once
#include "common.cuh"

namespace atlb {

struct MotionView {
  int kind;             // ATLB_MOTION_*
  const float* theta;   // (B,2) | (B,6) | (B,2,Hg,Wg)
  long long B, Hg, Wg;  // grid shape (dense)
  long long H, W;       // image shape
  float cx, cy;         // (W-1)/2, (H-1)/2 rounded to fp32 (parametric.py:98)
  float sx, sy;         // (float)max(W-1, 1), (float)max(H-1, 1)   (parametric.py:275-276)
  float gxm, gym;       // (float)(Wg-1), (float)(Hg-1)
};

inline MotionView make_motion_view(int kind, const float* theta, long long B, long long Hg, long long Wg, long long H,
                                   long long W) {
  MotionView m;
  m.kind = kind; m.theta = theta; m.B = B; m.Hg = Hg; m.Wg = Wg; m.H = H; m.W = W;
  m.cx = (float)((double)(W - 1) / 2.0);
  m.cy = (float)((double)(H - 1) / 2.0);
  m.sx = (float)(W - 1 > 1 ? W - 1 : 1);
  m.sy = (float)(H - 1 > 1 ? H - 1 : 1);
  m.gxm = (float)(Wg - 1);
  m.gym = (float)(Hg - 1);
  return m;
}

struct DenseTaps {
  long long x0, x1, y0, y1;
  float w[4];  // w00, w01, w10, w11
};

// sample_grid geometry (parametric.py:296-312) for DenseLinearFlow.field (parametric.py:273-277).
__device__ __forceinline__ void dense_taps(const MotionView& m, float x, float y, DenseTaps* T) {
  float gx = mul_rn(div_rn(x, m.sx), m.gxm);
  float gy = mul_rn(div_rn(y, m.sy), m.gym);
  gx = clampf(gx, 0.f, m.gxm);
  gy = clampf(gy, 0.f, m.gym);
  const float xm = (float)(m.Wg - 2 > 0 ? m.Wg - 2 : 0), ym = (float)(m.Hg - 2 > 0 ? m.Hg - 2 : 0);
  float x0 = floorf(gx), y0 = floorf(gy);
  x0 = x0 > xm ? xm : x0;
  y0 = y0 > ym ? ym : y0;
  const float ax = sub_rn(gx, x0), ay = sub_rn(gy, y0);
  T->x0 = (long long)x0;
  T->y0 = (long long)y0;
  T->x1 = T->x0 + 1 < m.Wg - 1 ? T->x0 + 1 : m.Wg - 1;
  T->y1 = T->y0 + 1 < m.Hg - 1 ? T->y0 + 1 : m.Hg - 1;
  const float bx = sub_rn(1.f, ax), by = sub_rn(1.f, ay);
  T->w[0] = mul_rn(bx, by);
  T->w[1] = mul_rn(ax, by);
  T->w[2] = mul_rn(bx, ay);
  T->w[3] = mul_rn(ax, ay);
}

__device__ __forceinline__ float2 motion_field(const MotionView& m, float x, float y, long long b) {
  if (m.kind == ATLB_MOTION_TRANSLATION) {
    return make_float2(m.theta[2 * b], m.theta[2 * b + 1]);
  }
  if (m.kind == ATLB_MOTION_AFFINE) {
    const float* th = m.theta + 6 * b;
    const float d0 = sub_rn(x, m.cx), d1 = sub_rn(y, m.cy);
    const float p0 = add_rn(mul_rn(th[2], d0), mul_rn(th[3], d1));
    const float p1 = add_rn(mul_rn(th[4], d0), mul_rn(th[5], d1));
    return make_float2(add_rn(th[0], p0), add_rn(th[1], p1));
  }
  DenseTaps T;
  dense_taps(m, x, y, &T);
  const long long plane = m.Hg * m.Wg;
  const float* F = m.theta + b * 2 * plane;
  const long long i00 = T.y0 * m.Wg + T.x0, i01 = T.y0 * m.Wg + T.x1, i10 = T.y1 * m.Wg + T.x0,
                  i11 = T.y1 * m.Wg + T.x1;
  float out[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float* Fc = F + c * plane;
    float s = mul_rn(__ldg(Fc + i00), T.w[0]);
    s = add_rn(s, mul_rn(__ldg(Fc + i01), T.w[1]));
    s = add_rn(s, mul_rn(__ldg(Fc + i10), T.w[2]));
    s = add_rn(s, mul_rn(__ldg(Fc + i11), T.w[3]));
    out[c] = s;
  }
  return make_float2(out[0], out[1]);
}

// Slice centre k of torch.linspace(0, 1, n+1) midpoints (ats.py:37-38; linspace's two-sided formula).
__device__ __forceinline__ float check_centre(int k, int n) {
  const float step = div_rn(1.f, (float)n);
  const int half = (n + 1) / 2;
  auto edge = [&](int i) { return i < half ? add_rn(0.f, mul_rn(step, (float)i)) : sub_rn(1.f, mul_rn(step, (float)(n - i))); };
  return mul_rn(0.5f, add_rn(edge(k), edge(k + 1)));
}

// visible_fraction for one anchor (ats.py:42-50) with the linear transport x + v(x) (c - t).
// counts_b: the anchor's batch row of per-slice event counts (exact integers).
__device__ __forceinline__ float visible_fraction_one(const MotionView& m, float xa, float ya, float ta, long long ba,
                                                      const int* __restrict__ counts_b, int n_check, float tau,
                                                      float wmax, float hmax) {
  const float2 v = motion_field(m, xa, ya, ba);
  float vis = 0.f, tot = 0.f;
  for (int k = 0; k < n_check; ++k) {
    const float c = check_centre(k, n_check);
    const float near = fabsf(sub_rn(ta, c)) <= tau ? 1.f : 0.f;
    const float dt = sub_rn(c, ta);
    const float yx = add_rn(xa, mul_rn(v.x, dt)), yy = add_rn(ya, mul_rn(v.y, dt));
    const float inside = (yx >= 0.f && yx <= wmax && yy >= 0.f && yy <= hmax) ? 1.f : 0.f;
    const float w = mul_rn((float)counts_b[k], near);
    vis = add_rn(vis, mul_rn(w, inside));
    tot = add_rn(tot, w);
  }
  const float r = div_rn(vis, tot < 1.f ? 1.f : tot);
  return r < 1e-3f ? 1e-3f : r;
}

}  // namespace atlb
