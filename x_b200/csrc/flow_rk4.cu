// Exact transport of the dense velocity grid (DenseLinearFlow, mode="exact"; atl/motion/parametric.py:72-80):
// `steps` classic fourth-order Runge-Kutta steps of dx/ds = v(x) over dt = t' - t, h = dt / steps,
//     k1 = v(x), k2 = v(x + (h/2) k1), k3 = v(x + (h/2) k2), k4 = v(x + h k3),
//     x <- x + h (k1 + 2 k2 + 2 k3 + k4) / 6,
// with v the grid's bilinear sample (border clamp) evaluated by motion_field, and every product, sum and
// quotient rounded in the reference's order.  One thread per event.
//
// Backward (dL/dgrid for dL/dy): the step-start states are kept, each step's stages are evaluated again, and
// reverse mode runs through them: with u = dL/dx_{s+1}, the stage adjoints are u h/6, u h/3, u h/3, u h/6;
// stage j at z_j adds J_v(z_j)^T (its adjoint) to dL/dx_s and, through z_j = x_s + c_j h k_{j-1}, to the
// adjoint of the previous stage; and its grid taps receive w_q(z_j) (its adjoint) by red.global.add.
#include "common.cuh"
#include "motion_math.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxSteps = 64;

// v(z) and the bilinear taps of the sample (for the backward).
struct DenseSample {
  DenseTaps T;
  bool inx, iny;  // inside the clamp range (the clamp passes gradient there)
};

__device__ __forceinline__ float2 dense_value(const MotionView& m, float x, float y, long long b) {
  return motion_field(m, x, y, b);
}

// J_v(z)^T u and the grid gradient of v(z) for the adjoint u (red.add into G).
__device__ __forceinline__ float2 dense_adjoint(const MotionView& m, float x, float y, long long b, float2 u,
                                                float* __restrict__ G) {
  DenseTaps T;
  dense_taps(m, x, y, &T);
  const float gxr = mul_rn(div_rn(x, m.sx), m.gxm), gyr = mul_rn(div_rn(y, m.sy), m.gym);
  const bool inx = gxr >= 0.f && gxr <= m.gxm, iny = gyr >= 0.f && gyr <= m.gym;
  const long long plane = m.Hg * m.Wg;
  const float* F = m.theta + b * 2 * plane;
  float* Gb = G + b * 2 * plane;
  const long long idx[4] = {T.y0 * m.Wg + T.x0, T.y0 * m.Wg + T.x1, T.y1 * m.Wg + T.x0, T.y1 * m.Wg + T.x1};
  // weights as functions of (ax, ay): w00 = (1-ax)(1-ay), w01 = ax(1-ay), w10 = (1-ax)ay, w11 = ax ay
  const float ax = T.w[1] + T.w[3], ay = T.w[2] + T.w[3];  // ax(1-ay) + ax ay, (1-ax)ay + ax ay
  const float dwx[4] = {-(1.f - ay), 1.f - ay, -ay, ay}, dwy[4] = {-(1.f - ax), -ax, 1.f - ax, ax};
  float jx = 0.f, jy = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float fx = __ldg(F + idx[q]), fy = __ldg(F + plane + idx[q]);
    const float s = u.x * fx + u.y * fy;
    jx += dwx[q] * s;
    jy += dwy[q] * s;
    if (T.w[q] != 0.f) {
      red_add_f1(Gb + idx[q], T.w[q] * u.x);
      red_add_f1(Gb + plane + idx[q], T.w[q] * u.y);
    }
  }
  const float sx = inx ? m.gxm / m.sx : 0.f, sy = iny ? m.gym / m.sy : 0.f;
  return make_float2(jx * sx, jy * sy);
}

struct Rk4Stages {
  float2 z[4], k[4];
};

// One RK4 step from x with step h: the stage points, slopes and the new state (the reference's rounding).
__device__ __forceinline__ float2 rk4_step(const MotionView& m, float2 x, float h, long long b, Rk4Stages* S) {
  const float hh = mul_rn(0.5f, h);
  S->z[0] = x;
  S->k[0] = dense_value(m, x.x, x.y, b);
  S->z[1] = make_float2(add_rn(x.x, mul_rn(hh, S->k[0].x)), add_rn(x.y, mul_rn(hh, S->k[0].y)));
  S->k[1] = dense_value(m, S->z[1].x, S->z[1].y, b);
  S->z[2] = make_float2(add_rn(x.x, mul_rn(hh, S->k[1].x)), add_rn(x.y, mul_rn(hh, S->k[1].y)));
  S->k[2] = dense_value(m, S->z[2].x, S->z[2].y, b);
  S->z[3] = make_float2(add_rn(x.x, mul_rn(h, S->k[2].x)), add_rn(x.y, mul_rn(h, S->k[2].y)));
  S->k[3] = dense_value(m, S->z[3].x, S->z[3].y, b);
  float sx = add_rn(add_rn(add_rn(S->k[0].x, mul_rn(2.f, S->k[1].x)), mul_rn(2.f, S->k[2].x)), S->k[3].x);
  float sy = add_rn(add_rn(add_rn(S->k[0].y, mul_rn(2.f, S->k[1].y)), mul_rn(2.f, S->k[2].y)), S->k[3].y);
  return make_float2(add_rn(x.x, div_rn(mul_rn(h, sx), 6.f)), add_rn(x.y, div_rn(mul_rn(h, sy), 6.f)));
}

__device__ __forceinline__ float step_size(const float* t, const float* tdst, float tdst_s, long long n, int steps) {
  return div_rn(sub_rn(tdst ? tdst[n] : tdst_s, t[n]), (float)steps);
}

__global__ void __launch_bounds__(kThreads) k_flow_rk4(MotionView m, const float2* __restrict__ xy,
                                                       const float* __restrict__ t, const float* __restrict__ tdst,
                                                       float tdst_s, const long long* __restrict__ b, long long N,
                                                       int steps, float2* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    if (b[n] < 0 || b[n] >= m.B) {
      out[n] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      continue;
    }
    const float h = step_size(t, tdst, tdst_s, n, steps);
    float2 x = xy[n];
    Rk4Stages S;
    for (int s = 0; s < steps; ++s) x = rk4_step(m, x, h, b[n], &S);
    out[n] = x;
  }
}

__global__ void __launch_bounds__(kThreads) k_flow_rk4_bwd(MotionView m, const float2* __restrict__ gy,
                                                           const float2* __restrict__ xy,
                                                           const float* __restrict__ t,
                                                           const float* __restrict__ tdst, float tdst_s,
                                                           const long long* __restrict__ b, long long N, int steps,
                                                           float* __restrict__ G) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 u0 = gy[n];
    if ((u0.x == 0.f && u0.y == 0.f) || b[n] < 0 || b[n] >= m.B) continue;
    const long long bb = b[n];
    const float h = step_size(t, tdst, tdst_s, n, steps);
    float2 X[kMaxSteps];  // step-start states
    float2 x = xy[n];
    Rk4Stages S;
    for (int s = 0; s < steps; ++s) {
      X[s] = x;
      x = rk4_step(m, x, h, bb, &S);
    }
    float2 u = u0;  // dL/dx of the state after step s
    for (int s = steps - 1; s >= 0; --s) {
      rk4_step(m, X[s], h, bb, &S);
      const float c6 = h / 6.f, c3 = h / 3.f;
      float2 a[4] = {make_float2(u.x * c6, u.y * c6), make_float2(u.x * c3, u.y * c3),
                     make_float2(u.x * c3, u.y * c3), make_float2(u.x * c6, u.y * c6)};
      float2 gx = u;  // direct term of x_{s+1} = x_s + ...
      const float cz[4] = {0.f, 0.5f * h, 0.5f * h, h};  // z_j = x_s + cz[j] k_{j-1}
#pragma unroll
      for (int j = 3; j >= 0; --j) {
        const float2 gz = dense_adjoint(m, S.z[j].x, S.z[j].y, bb, a[j], G);
        gx.x += gz.x;
        gx.y += gz.y;
        if (j > 0) {
          a[j - 1].x += cz[j] * gz.x;
          a[j - 1].y += cz[j] * gz.y;
        }
      }
      u = gx;
    }
  }
}

}  // namespace

int flow_rk4_steps_max() { return kMaxSteps; }

int flow_rk4(const MotionView& m, const float* xy, const float* t, const float* tdst, float tdst_s,
             const long long* b, long long N, int steps, float* out, cudaStream_t s) {
  if (N > 0)
    launch(k_flow_rk4, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, m, (const float2*)xy, t, tdst, tdst_s, b,
           N, steps, (float2*)out);
  return launch_status("flow_rk4");
}

int flow_rk4_bwd(const MotionView& m, const float* gy, const float* xy, const float* t, const float* tdst,
                 float tdst_s, const long long* b, long long N, int steps, float* gtheta, cudaStream_t s) {
  cudaMemsetAsync(gtheta, 0, (size_t)(m.B * 2 * m.Hg * m.Wg) * sizeof(float), s);
  if (N > 0)
    launch(k_flow_rk4_bwd, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, m, (const float2*)gy,
           (const float2*)xy, t, tdst, tdst_s, b, N, steps, gtheta);
  return launch_status("flow_rk4_bwd");
}

}  // namespace atlb
