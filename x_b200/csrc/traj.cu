// Continuous-time pixel trajectories (atl/motion/trajectories.py:40-90): transport of events and its
// backward to the tile coefficients, one thread per event.
//
//   q(p, t) = p + sum_k c_k(p) g_k(t),   c(p) = bilinear sample (border clamp) of the tile coefficient grid
//                                              at ((p - offset) / tile)            (parametric.py:296-312)
//   transport(x, t -> t'):  p_0 = x,  p_{i+1} = x - d(p_i, t)  (n_fp times),  y = p_n + d(p_n, t')
//
// The coefficients are read channels-last (B, Hq, Wq, 2K) with channels [y_1..y_K, x_1..x_K], so one tap of
// a sample is 2K consecutive floats.  The backward recomputes the iterates and runs reverse mode through
// them: dL/dp_i = -J_d(p_i)^T dL/dp_{i+1}, and every sample scatters w_tap * g_k(t) * dL/dp into the four
// taps of its coefficient cell (red.global).  The rounding sequence follows the reference's torch ops
// (p - offset, / tile, clamp, floor, weights, products summed in tap order, then over k).
#include "common.cuh"
#include "traj.cuh"

namespace atlb {
namespace {

constexpr int kTThreads = 256;

// g_k(t) - g_k(0), k = 1..K (trajectories.py:26-37): t^k, or (c_k t^k) (1 - t)^(K - k).
__device__ __forceinline__ void traj_basis(const TrajView& V, float t, float* g) {
  for (int k = 0; k < V.K; ++k) {
    const float tk = powf(t, (float)(k + 1));
    g[k] = V.basis == 0 ? tk : mul_rn(mul_rn(V.bc[k], tk), powf(sub_rn(1.f, t), (float)(V.K - k - 1)));
  }
}

struct Taps {
  long long base[4];  // offsets of the four taps (channels-last)
  float w[4];         // bilinear weights (1-ax)(1-ay), ax(1-ay), (1-ax)ay, ax ay
  float ax, ay;
  bool gx_in, gy_in;  // inside the clamp range (the clamp passes gradient)
};

__device__ __forceinline__ Taps traj_taps(const TrajView& V, int b, float px, float py) {
  Taps T;
  const float gxr = div_rn(sub_rn(px, V.offset), V.tile), gyr = div_rn(sub_rn(py, V.offset), V.tile);
  const float wq = (float)(V.Wq - 1), hq = (float)(V.Hq - 1);
  T.gx_in = gxr >= 0.f && gxr <= wq;
  T.gy_in = gyr >= 0.f && gyr <= hq;
  const float gx = fminf(fmaxf(gxr, 0.f), wq), gy = fminf(fmaxf(gyr, 0.f), hq);
  const float x0 = fminf(floorf(gx), (float)max(V.Wq - 2, 0)), y0 = fminf(floorf(gy), (float)max(V.Hq - 2, 0));
  T.ax = sub_rn(gx, x0);
  T.ay = sub_rn(gy, y0);
  const int ix0 = (int)x0, iy0 = (int)y0, ix1 = min(ix0 + 1, V.Wq - 1), iy1 = min(iy0 + 1, V.Hq - 1);
  const long long C2 = 2LL * V.K, plane = (long long)b * V.Hq * V.Wq;
  T.base[0] = (plane + (long long)iy0 * V.Wq + ix0) * C2;
  T.base[1] = (plane + (long long)iy0 * V.Wq + ix1) * C2;
  T.base[2] = (plane + (long long)iy1 * V.Wq + ix0) * C2;
  T.base[3] = (plane + (long long)iy1 * V.Wq + ix1) * C2;
  const float oax = sub_rn(1.f, T.ax), oay = sub_rn(1.f, T.ay);
  T.w[0] = mul_rn(oax, oay);
  T.w[1] = mul_rn(T.ax, oay);
  T.w[2] = mul_rn(oax, T.ay);
  T.w[3] = mul_rn(T.ax, T.ay);
  return T;
}

// displacement d(p, t) = sum_k (cx_k, cy_k) g_k with c the bilinear sample at p
__device__ __forceinline__ float2 traj_disp(const TrajView& V, const Taps& T, const float* g) {
  float dx = 0.f, dy = 0.f;
  for (int k = 0; k < V.K; ++k) {
    float cy = 0.f, cx = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      cy = add_rn(cy, mul_rn(__ldg(V.C + T.base[q] + k), T.w[q]));
      cx = add_rn(cx, mul_rn(__ldg(V.C + T.base[q] + V.K + k), T.w[q]));
    }
    dx = add_rn(dx, mul_rn(cx, g[k]));
    dy = add_rn(dy, mul_rn(cy, g[k]));
  }
  return make_float2(dx, dy);
}

__global__ void __launch_bounds__(kTThreads) k_traj_fwd(TrajView V, const float2* __restrict__ xy,
                                                        const float* __restrict__ t, const float* __restrict__ tdst,
                                                        float tdst_s, const long long* __restrict__ b, long long N,
                                                        float2* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 x = xy[n];
    if (b[n] < 0 || b[n] >= V.B) {  // no coefficient grid for this batch index
      out[n] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      continue;
    }
    const int bb = (int)b[n];
    float g[kTrajKMax];
    traj_basis(V, t[n], g);
    float px = x.x, py = x.y;
    for (int i = 0; i < V.n_fp; ++i) {
      const float2 d = traj_disp(V, traj_taps(V, bb, px, py), g);
      px = sub_rn(x.x, d.x);
      py = sub_rn(x.y, d.y);
    }
    traj_basis(V, tdst ? tdst[n] : tdst_s, g);
    const float2 d = traj_disp(V, traj_taps(V, bb, px, py), g);
    out[n] = make_float2(add_rn(px, d.x), add_rn(py, d.y));
  }
}

// Reverse step through one sample of d at p (basis g, incoming dL/dd = (ux, uy)): scatters the coefficient
// gradient and returns J_d(p)^T (ux, uy).
__device__ __forceinline__ float2 traj_disp_bwd(const TrajView& V, const Taps& T, const float* g, float ux, float uy,
                                                float* __restrict__ gC) {
  // d(sample)/d(ax), d(sample)/d(ay) per channel, from the weights' derivatives
  float jxx = 0.f, jxy = 0.f, jyx = 0.f, jyy = 0.f;  // J = [[d dx/d px, d dx/d py], [d dy/d px, d dy/d py]]
  const float oax = 1.f - T.ax, oay = 1.f - T.ay;
  for (int k = 0; k < V.K; ++k) {
    float f[4][2];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      f[q][0] = __ldg(V.C + T.base[q] + V.K + k);  // x channel
      f[q][1] = __ldg(V.C + T.base[q] + k);        // y channel
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const float dax = (f[1][c] - f[0][c]) * oay + (f[3][c] - f[2][c]) * T.ay;
      const float day = (f[2][c] - f[0][c]) * oax + (f[3][c] - f[1][c]) * T.ax;
      if (c == 0) { jxx += g[k] * dax; jxy += g[k] * day; } else { jyx += g[k] * dax; jyy += g[k] * day; }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float wg = T.w[q] * g[k];
      if (uy != 0.f) red_add_f1(gC + T.base[q] + k, wg * uy);
      if (ux != 0.f) red_add_f1(gC + T.base[q] + V.K + k, wg * ux);
    }
  }
  const float sx = T.gx_in ? 1.f / V.tile : 0.f, sy = T.gy_in ? 1.f / V.tile : 0.f;
  return make_float2((jxx * ux + jyx * uy) * sx, (jxy * ux + jyy * uy) * sy);
}

__global__ void __launch_bounds__(kTThreads) k_traj_bwd(TrajView V, const float2* __restrict__ gy,
                                                        const float2* __restrict__ xy, const float* __restrict__ t,
                                                        const float* __restrict__ tdst, float tdst_s,
                                                        const long long* __restrict__ b, long long N,
                                                        float* __restrict__ gC) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 u = gy[n];
    if ((u.x == 0.f && u.y == 0.f) || b[n] < 0 || b[n] >= V.B) continue;
    const float2 x = xy[n];
    const int bb = (int)b[n];
    float g[kTrajKMax], gd[kTrajKMax];
    traj_basis(V, t[n], g);
    traj_basis(V, tdst ? tdst[n] : tdst_s, gd);
    float P[kTrajKMax + 1][2];  // iterates p_0 .. p_n (n_fp <= kTrajKMax)
    P[0][0] = x.x;
    P[0][1] = x.y;
    for (int i = 0; i < V.n_fp; ++i) {
      const float2 d = traj_disp(V, traj_taps(V, bb, P[i][0], P[i][1]), g);
      P[i + 1][0] = sub_rn(x.x, d.x);
      P[i + 1][1] = sub_rn(x.y, d.y);
    }
    // y = p_n + d(p_n, t')
    const float2 jt = traj_disp_bwd(V, traj_taps(V, bb, P[V.n_fp][0], P[V.n_fp][1]), gd, u.x, u.y, gC);
    float gpx = u.x + jt.x, gpy = u.y + jt.y;
    // p_{i+1} = x - d(p_i, t)
    for (int i = V.n_fp - 1; i >= 0; --i) {
      const float2 j = traj_disp_bwd(V, traj_taps(V, bb, P[i][0], P[i][1]), g, -gpx, -gpy, gC);
      gpx = j.x;
      gpy = j.y;
    }
  }
}

inline int tgrid(long long n) { return clamp_grid(blocks_for(n, kTThreads)); }

}  // namespace

int traj_transport(const TrajView& V, const float* xy, const float* t, const float* tdst, float tdst_s,
                   const long long* b, long long N, float* out, cudaStream_t s) {
  if (N > 0)
    launch(k_traj_fwd, tgrid(N), kTThreads, 0, s, V, (const float2*)xy, t, tdst, tdst_s, b, N, (float2*)out);
  return launch_status("traj_transport");
}

int traj_transport_bwd(const TrajView& V, const float* gy, const float* xy, const float* t, const float* tdst,
                       float tdst_s, const long long* b, long long N, float* gC, cudaStream_t s) {
  if (N > 0)
    launch(k_traj_bwd, tgrid(N), kTThreads, 0, s, V, (const float2*)gy, (const float2*)xy, t, tdst, tdst_s, b, N,
           gC);
  return launch_status("traj_transport_bwd");
}

}  // namespace atlb
