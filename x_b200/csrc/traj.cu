// Continuous-time pixel trajectories (atl/motion/trajectories.py:40-90): transport of events and its
// backward to the tile coefficients, one thread per event.
//
//   q(p, t) = p + sum_k c_k(p) g_k(t),   c(p) = bilinear sample (border clamp) of the tile coefficient grid
//                                              at ((p - offset) / tile)            (parametric.py:296-312)
//   transport(x, t -> t'):  p_0 = x,  p_{i+1} = x - d(p_i, t)  (n_fp times),  y = p_n + d(p_n, t')
//
// The coefficients are read channels-last (B, Hq, Wq, 2K) with channels [y_1..y_K, x_1..x_K], so one tap of
// a sample is 2K consecutive floats (16-byte vector loads when 2K is a multiple of 4).  The kernels are
// instantiated per K (1..16) so that the per-event basis and channel sums live in registers.  The final
// sample follows the reference's order (the coefficient sample, taps in order, then the sum over k); the
// fixed-point iterations sum tap by tap with fused multiply-adds (traj_disp_it, half the arithmetic); the
// basis powers are products (t^k by repeated multiplication instead of pow).  Values differ from the
// reference's in the last bits.
// The backward recomputes the iterates and runs reverse mode through them: dL/dp_i = -J_d(p_i)^T dL/dp_{i+1}.
// The coefficient gradient w_tap * g_k(t) * dL/dp of the samples of one coefficient cell is accumulated per
// tap (the iterates of one event rarely leave their cell) and leaves with vector reds when the cell changes.
#include <type_traits>

#include "common.cuh"
#include "traj.cuh"

namespace atlb {
namespace {

constexpr int kTThreads = 256;

// g_k(t) - g_k(0), k = 1..K (trajectories.py:26-37): t^k, or (c_k t^k) (1 - t)^(K - k).
template <int K>
__device__ __forceinline__ void traj_basis(const TrajView& V, float t, float (&g)[K]) {
  float om[K];  // (1 - t)^j, j = 0..K-1
  const float u = sub_rn(1.f, t);
  om[0] = 1.f;
#pragma unroll
  for (int j = 1; j < K; ++j) om[j] = om[j - 1] * u;
  float tk = t;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    g[k] = V.basis == 0 ? tk : (V.bc[k] * tk) * om[K - 1 - k];
    tk *= t;
  }
}

struct Taps {
  int base[4];  // element offsets of the four taps (channels-last; the grid holds < 2^31 floats)
  float w[4];         // bilinear weights (1-ax)(1-ay), ax(1-ay), (1-ax)ay, ax ay
  float ax, ay;
  bool gx_in, gy_in;  // inside the clamp range (the clamp passes gradient)
};

__device__ __forceinline__ Taps traj_taps(const TrajView& V, int b, float px, float py) {
  Taps T;
  // (p - offset) / tile; for a power-of-two tile the product with its reciprocal is the same number
  const float ox = sub_rn(px, V.offset), oy = sub_rn(py, V.offset);
  const float gxr = V.tile_pow2 ? mul_rn(ox, V.rtile) : div_rn(ox, V.tile);
  const float gyr = V.tile_pow2 ? mul_rn(oy, V.rtile) : div_rn(oy, V.tile);
  const float wq = (float)(V.Wq - 1), hq = (float)(V.Hq - 1);
  T.gx_in = gxr >= 0.f && gxr <= wq;
  T.gy_in = gyr >= 0.f && gyr <= hq;
  const float gx = fminf(fmaxf(gxr, 0.f), wq), gy = fminf(fmaxf(gyr, 0.f), hq);
  const float x0 = fminf(floorf(gx), (float)max(V.Wq - 2, 0)), y0 = fminf(floorf(gy), (float)max(V.Hq - 2, 0));
  T.ax = sub_rn(gx, x0);
  T.ay = sub_rn(gy, y0);
  const int ix0 = (int)x0, iy0 = (int)y0, ix1 = min(ix0 + 1, V.Wq - 1), iy1 = min(iy0 + 1, V.Hq - 1);
  const int C2 = 2 * V.K, plane = b * V.Hq * V.Wq;
  T.base[0] = (plane + iy0 * V.Wq + ix0) * C2;
  T.base[1] = (plane + iy0 * V.Wq + ix1) * C2;
  T.base[2] = (plane + iy1 * V.Wq + ix0) * C2;
  T.base[3] = (plane + iy1 * V.Wq + ix1) * C2;
  const float oax = sub_rn(1.f, T.ax), oay = sub_rn(1.f, T.ay);
  T.w[0] = mul_rn(oax, oay);
  T.w[1] = mul_rn(T.ax, oay);
  T.w[2] = mul_rn(oax, T.ay);
  T.w[3] = mul_rn(T.ax, T.ay);
  return T;
}

// The 2K channels of one tap into registers.
template <int K>
__device__ __forceinline__ void load_tap(const float* __restrict__ p, float (&f)[2 * K]) {
  if constexpr ((2 * K) % 4 == 0) {
#pragma unroll
    for (int c = 0; c < 2 * K; c += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p + c));
      f[c] = v.x; f[c + 1] = v.y; f[c + 2] = v.z; f[c + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 2 * K; c += 2) {
      const float2 v = __ldg(reinterpret_cast<const float2*>(p + c));
      f[c] = v.x; f[c + 1] = v.y;
    }
  }
}

// The coefficient sample at the taps T: c = sum_q w_q c_q (taps summed in order, as sample_grid does).
template <int K>
__device__ __forceinline__ void traj_sample(const TrajView& V, const Taps& T, float (&c)[2 * K]) {
#pragma unroll
  for (int ch = 0; ch < 2 * K; ++ch) c[ch] = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float f[2 * K];
    load_tap<K>(V.C + T.base[q], f);
#pragma unroll
    for (int ch = 0; ch < 2 * K; ++ch) c[ch] = add_rn(c[ch], mul_rn(f[ch], T.w[q]));
  }
}

// sum_k (cx_k, cy_k) g_k of a coefficient sample
template <int K>
__device__ __forceinline__ float2 traj_dot(const float (&c)[2 * K], const float (&g)[K]) {
  float dx = 0.f, dy = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dx = add_rn(dx, mul_rn(c[K + k], g[k]));
    dy = add_rn(dy, mul_rn(c[k], g[k]));
  }
  return make_float2(dx, dy);
}

// displacement d(p, t) = sum_k (cx_k, cy_k) g_k with c the bilinear sample at p (the final sample of a
// transport; a caller moving one point to several times samples once and takes one dot per time)
template <int K>
__device__ __forceinline__ float2 traj_disp(const TrajView& V, const Taps& T, const float (&g)[K]) {
  float c[2 * K];
  traj_sample<K>(V, T, c);
  return traj_dot<K>(c, g);
}

// The displacement inside the fixed-point iterations, tap-major with fused multiply-adds:
// d = sum_q w_q(p) D_q, D_q = sum_k c_{q,k} g_k (x and y channels) -- half the arithmetic of traj_disp (which
// forms the coefficient sample first, as the reference's sample_grid does); the iterates differ from that
// order in the last bits only.  D depends on the cell (the four taps) and the basis only, and the iterates
// of one event rarely leave their cell, so D is kept in a CellDisp and the taps are read again only when
// the cell changes.  Every kernel iterates with this function, so a backward that solves the iterates
// again, and the records / targets kernels, reproduce the forward's iterates exactly.
struct CellDisp {
  int base0;           // first tap of the cell whose sums are held; -1: none
  float dx[4], dy[4];  // per tap q: D_q for the x and the y channels
};

template <int K>
__device__ __forceinline__ void cell_fill(const TrajView& V, const Taps& T, const float (&g)[K], CellDisp& D) {
  if (D.base0 == T.base[0]) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float f[2 * K];
    load_tap<K>(V.C + T.base[q], f);
    float sx = 0.f, sy = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      sx = fmaf(f[K + k], g[k], sx);
      sy = fmaf(f[k], g[k], sy);
    }
    D.dx[q] = sx;
    D.dy[q] = sy;
  }
  D.base0 = T.base[0];
}

template <int K>
__device__ __forceinline__ float2 traj_disp_it(const TrajView& V, const Taps& T, const float (&g)[K], CellDisp& D) {
  cell_fill<K>(V, T, g, D);
  float dx = 0.f, dy = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    dx = fmaf(T.w[q], D.dx[q], dx);
    dy = fmaf(T.w[q], D.dy[q], dy);
  }
  return make_float2(dx, dy);
}

// mode 0: x -> transport(x, t -> t');  1: x -> origin p (the fixed point, t' unused);  2: p -> p + d(p, t')
// (the input is an origin; t unused);  3: x -> the velocity of the degree-1 trajectory, the first coefficient
// pair c_1 sampled at the origin (trajectories.py:79-83; t' unused), with the origin iterated in the
// reference's order (traj_disp), so that the velocity -- which decides the exact path's pair tests -- is the
// reference's to the bit.  Modes 1 then 2 give exactly mode 0.
template <int K>
__global__ void __launch_bounds__(kTThreads) k_traj_fwd(TrajView V, int mode, const float2* __restrict__ xy,
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
    float g[K];
    float px = x.x, py = x.y;
    if (mode != 2) {
      traj_basis<K>(V, t[n], g);
      CellDisp D;
      D.base0 = -1;
      for (int i = 0; i < V.n_fp; ++i) {
        // the velocity feeds the exact pair test, so its origin is iterated in the reference's own order
        const Taps T = traj_taps(V, bb, px, py);
        const float2 d = mode == 3 ? traj_disp<K>(V, T, g) : traj_disp_it<K>(V, T, g, D);
        px = sub_rn(x.x, d.x);
        py = sub_rn(x.y, d.y);
      }
    }
    if (mode == 1) {
      out[n] = make_float2(px, py);
      continue;
    }
    if (mode == 3) {  // the first coefficient pair sampled at the origin (the basis e_1: c_1 exactly)
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = k == 0 ? 1.f : 0.f;
      out[n] = traj_disp<K>(V, traj_taps(V, bb, px, py), g);
      continue;
    }
    traj_basis<K>(V, tdst ? tdst[n] : tdst_s, g);
    const float2 d = traj_disp<K>(V, traj_taps(V, bb, px, py), g);
    out[n] = make_float2(add_rn(px, d.x), add_rn(py, d.y));
  }
}

// J_d(p)^T for per-channel weights (Ux_k, Uy_k) (the transposed bilinear Jacobian; the clamp passes
// gradient inside its range, floor none): (sum_q dw_q/dpx s_q, sum_q dw_q/dpy s_q) / tile with
// s_q = sum_k (Ux_k cx_{q,k} + Uy_k cy_{q,k}).
template <int K>
__device__ __forceinline__ float2 traj_jt_u(const TrajView& V, const Taps& T, const float (&Ux)[K],
                                            const float (&Uy)[K]) {
  const float oax = 1.f - T.ax, oay = 1.f - T.ay;
  const float dwx[4] = {-oay, oay, -T.ay, T.ay}, dwy[4] = {-oax, -T.ax, oax, T.ax};
  float jx = 0.f, jy = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float f[2 * K];
    load_tap<K>(V.C + T.base[q], f);
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) sq += Ux[k] * f[K + k] + Uy[k] * f[k];
    jx += dwx[q] * sq;
    jy += dwy[q] * sq;
  }
  const float sx = T.gx_in ? V.rtile : 0.f, sy = T.gy_in ? V.rtile : 0.f;
  return make_float2(jx * sx, jy * sy);
}

// J_d(p)^T (ux, uy) for one sample of d at p with basis g (the transposed bilinear Jacobian; the clamp passes
// gradient inside its range, floor none).  d = sum_q w_q(p) sum_k g_k c_{q,k}, so with
// s_q = sum_k g_k (ux cx_{q,k} + uy cy_{q,k}) the result is (sum_q dw_q/dpx s_q, sum_q dw_q/dpy s_q) / tile:
// one tap's coefficients are live at a time.
template <int K>
__device__ __forceinline__ float2 traj_jt(const TrajView& V, const Taps& T, const float (&g)[K], float ux,
                                          float uy) {
  float Ux[K], Uy[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    Ux[k] = g[k] * ux;
    Uy[k] = g[k] * uy;
  }
  return traj_jt_u<K>(V, T, Ux, Uy);
}

// traj_jt for the basis of a CellDisp (the iterations' basis g), from its per-tap sums:
// s_q = ux Dx_q + uy Dy_q; the taps are read only when the cell changes.
template <int K>
__device__ __forceinline__ float2 traj_jt_it(const TrajView& V, const Taps& T, const float (&g)[K], CellDisp& D,
                                             float ux, float uy) {
  cell_fill<K>(V, T, g, D);
  const float oax = 1.f - T.ax, oay = 1.f - T.ay;
  const float dwx[4] = {-oay, oay, -T.ay, T.ay}, dwy[4] = {-oax, -T.ax, oax, T.ax};
  float jx = 0.f, jy = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float sq = ux * D.dx[q] + uy * D.dy[q];
    jx += dwx[q] * sq;
    jy += dwy[q] * sq;
  }
  const float sx = T.gx_in ? V.rtile : 0.f, sy = T.gy_in ? V.rtile : 0.f;
  return make_float2(jx * sx, jy * sy);
}

// Coefficient gradient of the samples that fall in one coefficient cell.  For samples with basis g the
// gradient of (tap q, channel k) is g_k * sum_i w_q(p_i) u_i, so per cell only the per-tap sums
// a_q = sum_i w_q u_i (basis of the origin iterations) and f_q (basis of the final sample) are kept; they are
// flushed as g_k a_q + gd_k f_q into the 2K channels of each tap (vector reds) when the cell changes.
struct CellAcc {
  int base[4];
  float a[4][2], f[4][2];  // [tap][x, y]
  bool live;
};

template <int K>
__device__ __forceinline__ void acc_flush(CellAcc& A, const float (&g)[K], const float (&gd)[K],
                                          float* __restrict__ gC) {
  if (!A.live) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float v[2 * K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      v[k] = g[k] * A.a[q][1] + gd[k] * A.f[q][1];
      v[K + k] = g[k] * A.a[q][0] + gd[k] * A.f[q][0];
    }
    float* dst = gC + A.base[q];
    if constexpr ((2 * K) % 4 == 0) {
#pragma unroll
      for (int c = 0; c < 2 * K; c += 4) red_add_f4(dst + c, v[c], v[c + 1], v[c + 2], v[c + 3]);
    } else {
#pragma unroll
      for (int c = 0; c < 2 * K; c += 2) red_add_f2(dst + c, v[c], v[c + 1]);
    }
  }
  A.live = false;
}

template <int K>
__device__ __forceinline__ void acc_add(CellAcc& A, const Taps& T, bool final_basis, float ux, float uy,
                                        const float (&g)[K], const float (&gd)[K], float* __restrict__ gC) {
  if (A.live && A.base[0] != T.base[0]) acc_flush<K>(A, g, gd, gC);
  if (!A.live) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      A.base[q] = T.base[q];
      A.a[q][0] = A.a[q][1] = A.f[q][0] = A.f[q][1] = 0.f;
    }
    A.live = true;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (final_basis) {
      A.f[q][0] += T.w[q] * ux;
      A.f[q][1] += T.w[q] * uy;
    } else {
      A.a[q][0] += T.w[q] * ux;
      A.a[q][1] += T.w[q] * uy;
    }
  }
}

// Backward of k_traj_fwd's modes for u = dL/d(output): mode 0 and 1 scatter the coefficient gradient (mode 1:
// u is dL/dp of the origin); mode 2 also writes gp = dL/dp of its input origin.
template <int K>
__global__ void __launch_bounds__(kTThreads) k_traj_bwd(TrajView V, int mode, const float2* __restrict__ gy,
                                                        const float2* __restrict__ xy, const float* __restrict__ t,
                                                        const float* __restrict__ tdst, float tdst_s,
                                                        const long long* __restrict__ b, long long N,
                                                        float* __restrict__ gC, float2* __restrict__ gp_out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 u = gy[n];
    if ((u.x == 0.f && u.y == 0.f) || b[n] < 0 || b[n] >= V.B) {
      if (mode == 2) gp_out[n] = make_float2(0.f, 0.f);
      continue;
    }
    const float2 x = xy[n];
    const int bb = (int)b[n];
    float g[K], gd[K];
    const int nfp = mode == 2 ? 0 : V.n_fp;
    if (mode != 2) traj_basis<K>(V, t[n], g);
    if (mode == 0 || mode == 2) traj_basis<K>(V, tdst ? tdst[n] : tdst_s, gd);
    if (mode == 3)  // out = d(p, e_1): the final basis is e_1 and there is no identity term
#pragma unroll
      for (int k = 0; k < K; ++k) gd[k] = k == 0 ? 1.f : 0.f;
    if (mode == 2)
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = 0.f;
    if (mode == 1)
#pragma unroll
      for (int k = 0; k < K; ++k) gd[k] = 0.f;
    float P[kTrajKMax + 1][2];  // iterates p_0 .. p_n (n_fp <= kTrajKMax), as the forward computes them
    P[0][0] = x.x;
    P[0][1] = x.y;
    CellDisp D;
    D.base0 = -1;
    for (int i = 0; i < nfp; ++i) {
      const Taps T = traj_taps(V, bb, P[i][0], P[i][1]);
      const float2 d = mode == 3 ? traj_disp<K>(V, T, g) : traj_disp_it<K>(V, T, g, D);  // as the forward
      P[i + 1][0] = sub_rn(x.x, d.x);
      P[i + 1][1] = sub_rn(x.y, d.y);
    }
    CellAcc A;
    A.live = false;
    float gpx = u.x, gpy = u.y;
    if (mode != 1) {  // y = p_n + d(p_n, t')  (mode 3: y = d(p_n, e_1))
      const Taps T = traj_taps(V, bb, P[nfp][0], P[nfp][1]);
      acc_add<K>(A, T, true, u.x, u.y, g, gd, gC);
      const float2 jt = traj_jt<K>(V, T, gd, u.x, u.y);
      gpx = (mode == 3 ? 0.f : u.x) + jt.x;
      gpy = (mode == 3 ? 0.f : u.y) + jt.y;
    }
    // p_{i+1} = x - d(p_i, t)
    for (int i = nfp - 1; i >= 0; --i) {
      const Taps T = traj_taps(V, bb, P[i][0], P[i][1]);
      acc_add<K>(A, T, false, -gpx, -gpy, g, gd, gC);
      const float2 j = traj_jt_it<K>(V, T, g, D, -gpx, -gpy);
      gpx = j.x;
      gpy = j.y;
    }
    acc_flush<K>(A, g, gd, gC);
    if (mode == 2) gp_out[n] = make_float2(gpx, gpy);
  }
}

// Exposure correction (atl/objectives/ats.py:31-50) under the trajectories: for each anchor, the share of
// its window's events recorded while the anchor's trajectory was inside the image, over n_check slice
// centres.  The origin of the anchor's trajectory is solved once and reused for every centre (the
// reference transports the anchor to each centre separately; the origin does not depend on the centre).
template <int K>
__global__ void __launch_bounds__(kTThreads) k_traj_vis(TrajView V, const float2* __restrict__ xa,
                                                        const float* __restrict__ ta, const long long* __restrict__ ba,
                                                        long long M, const float* __restrict__ counts,
                                                        const float* __restrict__ centres, int n_check, float tau,
                                                        float wmax, float hmax, float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const float2 x = xa[i];
    if (ba[i] < 0 || ba[i] >= V.B) {
      out[i] = __int_as_float(0x7fc00000);
      continue;
    }
    const int bb = (int)ba[i];
    const float t = ta[i];
    float g[K];
    traj_basis<K>(V, t, g);
    float px = x.x, py = x.y;
    CellDisp D;
    D.base0 = -1;
    for (int it = 0; it < V.n_fp; ++it) {
      const float2 d = traj_disp_it<K>(V, traj_taps(V, bb, px, py), g, D);
      px = sub_rn(x.x, d.x);
      py = sub_rn(x.y, d.y);
    }
    float cs[2 * K];  // the coefficient sample at the origin, shared by every check time
    traj_sample<K>(V, traj_taps(V, bb, px, py), cs);
    float vis = 0.f, tot = 0.f;
    for (int k = 0; k < n_check; ++k) {
      const float c = __ldg(centres + k);
      const float near = fabsf(sub_rn(t, c)) <= tau ? 1.f : 0.f;
      traj_basis<K>(V, c, g);
      const float2 d = traj_dot<K>(cs, g);
      const float yx = add_rn(px, d.x), yy = add_rn(py, d.y);
      const float inside = (yx >= 0.f && yx <= wmax && yy >= 0.f && yy <= hmax) ? 1.f : 0.f;
      const float w = mul_rn(__ldg(counts + (long long)bb * n_check + k), near);
      vis = add_rn(vis, mul_rn(w, inside));
      tot = add_rn(tot, w);
    }
    const float r = div_rn(vis, tot < 1.f ? 1.f : tot);
    out[i] = r < 1e-3f ? 1e-3f : r;
  }
}

// Records: R positions per event (xy (N, R, 2), all at the event's time t) moved to one target time each
// (t_dst per event or t_dst_s): out (N, R, 2), each record exactly as mode 0 moves it.  One thread per record,
// so the records of an event sit in neighbouring lanes and their coefficient taps (close together, usually
// in one cell) are served by the same load instructions.  The backward merges the final per-tap gradient
// sums of neighbouring lanes of one event and one coefficient cell (segmented shuffle reduction) before a
// single lane flushes them.
template <int K>
__global__ void __launch_bounds__(kTThreads, 4) k_traj_records_fwd(TrajView V, int R, const float2* __restrict__ xy,
                                                                const float* __restrict__ t,
                                                                const float* __restrict__ tdst, float tdst_s,
                                                                const long long* __restrict__ b, long long N,
                                                                float2* __restrict__ out, float2* __restrict__ iters) {
  const long long NR = N * R;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < NR; i += stride) {
    const long long n = i / R;
    if (b[n] < 0 || b[n] >= V.B) {
      out[i] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      continue;
    }
    const int bb = (int)b[n];
    float g[K];
    traj_basis<K>(V, t[n], g);
    const float2 x = xy[i];
    float px = x.x, py = x.y;
    CellDisp D;
    D.base0 = -1;
    for (int it = 0; it < V.n_fp; ++it) {
      const float2 d = traj_disp_it<K>(V, traj_taps(V, bb, px, py), g, D);
      px = sub_rn(x.x, d.x);
      py = sub_rn(x.y, d.y);
      if (iters) iters[(long long)it * NR + i] = make_float2(px, py);  // iterate-major: coalesced
    }
    traj_basis<K>(V, tdst ? tdst[n] : tdst_s, g);
    const float2 d = traj_disp<K>(V, traj_taps(V, bb, px, py), g);
    out[i] = make_float2(add_rn(px, d.x), add_rn(py, d.y));
  }
}

// STORED: the forward's iterates are read back from `iters` inside the reverse loop (no per-thread array of
// iterates, which would live in local memory); otherwise the iterates are solved again into such an array.
template <int K, bool STORED>
__global__ void __launch_bounds__(kTThreads, 3) k_traj_records_bwd(TrajView V, int R, const float2* __restrict__ gy,
                                                                const float2* __restrict__ xy,
                                                                const float* __restrict__ t,
                                                                const float* __restrict__ tdst, float tdst_s,
                                                                const long long* __restrict__ b, long long N,
                                                                const float2* __restrict__ iters,
                                                                float* __restrict__ gC) {
  const long long NR = N * R;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  // warp-uniform loop: every lane reaches the merge below on every pass
  for (long long i0 = blockIdx.x * (long long)blockDim.x; i0 < NR; i0 += stride) {
    const long long i = i0 + threadIdx.x;
    const long long n = i < NR ? i / R : -1;
    float g[K], gd[K];
    CellAcc A;
    A.live = false;
    const float2 u = n >= 0 ? gy[i] : make_float2(0.f, 0.f);
    if (n >= 0 && (u.x != 0.f || u.y != 0.f) && b[n] >= 0 && b[n] < V.B) {
      const int bb = (int)b[n];
      traj_basis<K>(V, t[n], g);
      traj_basis<K>(V, tdst ? tdst[n] : tdst_s, gd);
      const float2 x = xy[i];
      CellDisp D;
      D.base0 = -1;
      if constexpr (STORED) {
        // iterate k (k = 1..n_fp) sits at iters[(k - 1) NR + i]; iterate 0 is x
        const float2 pn = V.n_fp > 0 ? iters[(long long)(V.n_fp - 1) * NR + i] : x;
        const Taps T = traj_taps(V, bb, pn.x, pn.y);
        acc_add<K>(A, T, true, u.x, u.y, g, gd, gC);
        const float2 jt = traj_jt<K>(V, T, gd, u.x, u.y);
        float gpx = u.x + jt.x, gpy = u.y + jt.y;
        float2 p = V.n_fp > 1 ? iters[(long long)(V.n_fp - 2) * NR + i] : x;
        for (int it = V.n_fp - 1; it >= 0; --it) {
          // the next (earlier) iterate is loaded before this one's work
          const float2 pnext = it > 1 ? iters[(long long)(it - 2) * NR + i] : x;
          const Taps Ti = traj_taps(V, bb, p.x, p.y);
          acc_add<K>(A, Ti, false, -gpx, -gpy, g, gd, gC);
          const float2 j = traj_jt_it<K>(V, Ti, g, D, -gpx, -gpy);
          gpx = j.x;
          gpy = j.y;
          p = pnext;
        }
      } else {
        float P[kTrajKMax + 1][2];
        P[0][0] = x.x;
        P[0][1] = x.y;
        for (int it = 0; it < V.n_fp; ++it) {
          const float2 d = traj_disp_it<K>(V, traj_taps(V, bb, P[it][0], P[it][1]), g, D);
          P[it + 1][0] = sub_rn(x.x, d.x);
          P[it + 1][1] = sub_rn(x.y, d.y);
        }
        const Taps T = traj_taps(V, bb, P[V.n_fp][0], P[V.n_fp][1]);
        acc_add<K>(A, T, true, u.x, u.y, g, gd, gC);
        const float2 jt = traj_jt<K>(V, T, gd, u.x, u.y);
        float gpx = u.x + jt.x, gpy = u.y + jt.y;
        for (int it = V.n_fp - 1; it >= 0; --it) {
          const Taps Ti = traj_taps(V, bb, P[it][0], P[it][1]);
          acc_add<K>(A, Ti, false, -gpx, -gpy, g, gd, gC);
          const float2 j = traj_jt_it<K>(V, Ti, g, D, -gpx, -gpy);
          gpx = j.x;
          gpy = j.y;
        }
      }
    }
    // runs of neighbouring lanes with the same event and the same open cell add up their per-tap sums
    const long long key_n = A.live ? n : -1 - lane;
    const long long key_c = A.live ? A.base[0] : -1;
    const long long prev_n = __shfl_up_sync(0xffffffffu, key_n, 1), prev_c = __shfl_up_sync(0xffffffffu, key_c, 1);
    const bool head = lane == 0 || prev_n != key_n || prev_c != key_c;
    const unsigned heads = __ballot_sync(0xffffffffu, head);
    const int run = __popc(heads & (0xffffffffu >> (31 - lane)));
    for (int off = 1; off < R && off < 32; off <<= 1) {
      const int orun = __shfl_down_sync(0xffffffffu, run, off);
      const bool take = lane + off < 32 && orun == run;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float oa = __shfl_down_sync(0xffffffffu, A.a[q][c], off);
          const float of = __shfl_down_sync(0xffffffffu, A.f[q][c], off);
          if (take) {
            A.a[q][c] += oa;
            A.f[q][c] += of;
          }
        }
    }
    if (head && A.live) acc_flush<K>(A, g, gd, gC);
  }
}

// Targets: every event moved to each of T shared target times (targets, T <= kTrajTargetsMax): the origin
// is solved once, the coefficients are sampled once at it, and each target costs one basis dot product.
// out (T, N, 2), each entry exactly as mode 0 computes it.  Backward: with u_j = dL/dout[j] and
// U_k = sum_j g_k(c_j) u_j, the coefficient gradient of the final samples is w_q U_k and dL/dp is
// sum_j u_j + J^T(U), one Jacobian evaluation for all targets; then reverse mode through the iterations.
constexpr int kTrajTargetsMax = 64;

template <int K>
__device__ __forceinline__ void load_target_bases(const TrajView& V, const float* __restrict__ targets, int T,
                                                  float* s_gd) {
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    float gd[K];
    traj_basis<K>(V, targets[j], gd);
#pragma unroll
    for (int k = 0; k < K; ++k) s_gd[j * K + k] = gd[k];
  }
  __syncthreads();
}

template <int K>
__global__ void __launch_bounds__(kTThreads) k_traj_targets_fwd(TrajView V, const float2* __restrict__ xy,
                                                                const float* __restrict__ t,
                                                                const long long* __restrict__ b, long long N,
                                                                const float* __restrict__ targets, int T,
                                                                float2* __restrict__ out) {
  __shared__ float s_gd[kTrajTargetsMax * K];
  load_target_bases<K>(V, targets, T, s_gd);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    if (b[n] < 0 || b[n] >= V.B) {
      for (int j = 0; j < T; ++j) out[j * N + n] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      continue;
    }
    const int bb = (int)b[n];
    const float2 x = xy[n];
    float g[K];
    traj_basis<K>(V, t[n], g);
    float px = x.x, py = x.y;
    CellDisp D;
    D.base0 = -1;
    for (int i = 0; i < V.n_fp; ++i) {
      const float2 d = traj_disp_it<K>(V, traj_taps(V, bb, px, py), g, D);
      px = sub_rn(x.x, d.x);
      py = sub_rn(x.y, d.y);
    }
    // the coefficient sample at the origin (as traj_disp forms it), one dot product per target
    float c[2 * K];
    traj_sample<K>(V, traj_taps(V, bb, px, py), c);
    for (int j = 0; j < T; ++j) {
      const float* gd = s_gd + j * K;
      float dx = 0.f, dy = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        dx = add_rn(dx, mul_rn(c[K + k], gd[k]));
        dy = add_rn(dy, mul_rn(c[k], gd[k]));
      }
      out[j * N + n] = make_float2(add_rn(px, dx), add_rn(py, dy));
    }
  }
}

template <int K>
__global__ void __launch_bounds__(kTThreads, 2) k_traj_targets_bwd(TrajView V, const float2* __restrict__ gy,
                                                                const float2* __restrict__ xy,
                                                                const float* __restrict__ t,
                                                                const long long* __restrict__ b, long long N,
                                                                const float* __restrict__ targets, int T,
                                                                float* __restrict__ gC) {
  __shared__ float s_gd[kTrajTargetsMax * K];
  load_target_bases<K>(V, targets, T, s_gd);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    if (b[n] < 0 || b[n] >= V.B) continue;
    float Ux[K], Uy[K];
#pragma unroll
    for (int k = 0; k < K; ++k) Ux[k] = Uy[k] = 0.f;
    float sux = 0.f, suy = 0.f;
    for (int j = 0; j < T; ++j) {
      const float2 u = gy[j * N + n];
      const float* gd = s_gd + j * K;
      sux += u.x;
      suy += u.y;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        Ux[k] += gd[k] * u.x;
        Uy[k] += gd[k] * u.y;
      }
    }
    if (sux == 0.f && suy == 0.f) {
      bool any = false;
#pragma unroll
      for (int k = 0; k < K; ++k) any |= (Ux[k] != 0.f) | (Uy[k] != 0.f);
      if (!any) continue;
    }
    const int bb = (int)b[n];
    const float2 x = xy[n];
    float g[K];
    traj_basis<K>(V, t[n], g);
    float P[kTrajKMax + 1][2];
    P[0][0] = x.x;
    P[0][1] = x.y;
    CellDisp D;
    D.base0 = -1;
    for (int i = 0; i < V.n_fp; ++i) {
      const float2 d = traj_disp_it<K>(V, traj_taps(V, bb, P[i][0], P[i][1]), g, D);
      P[i + 1][0] = sub_rn(x.x, d.x);
      P[i + 1][1] = sub_rn(x.y, d.y);
    }
    const Taps Tp = traj_taps(V, bb, P[V.n_fp][0], P[V.n_fp][1]);
    // final samples: coefficient gradient w_q U_k, and dL/dp = sum_j u_j + J^T(U)
    const float2 jU = traj_jt_u<K>(V, Tp, Ux, Uy);
    float gpx = sux + jU.x, gpy = suy + jU.y;
    // the fixed-point part accumulates per tap (basis g); the final samples' w_q U_k joins the flush of the
    // origin's cell (the cell of the last iterate, where the reverse pass starts)
    CellAcc A;
    A.live = false;
    bool final_pending = true;
    auto flush = [&]() {
      if (!A.live) return;
      const bool fin = final_pending && A.base[0] == Tp.base[0];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v[2 * K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
          v[k] = g[k] * A.a[q][1] + (fin ? Tp.w[q] * Uy[k] : 0.f);
          v[K + k] = g[k] * A.a[q][0] + (fin ? Tp.w[q] * Ux[k] : 0.f);
        }
        float* dst = gC + A.base[q];
        if constexpr ((2 * K) % 4 == 0) {
#pragma unroll
          for (int c = 0; c < 2 * K; c += 4) red_add_f4(dst + c, v[c], v[c + 1], v[c + 2], v[c + 3]);
        } else {
#pragma unroll
          for (int c = 0; c < 2 * K; c += 2) red_add_f2(dst + c, v[c], v[c + 1]);
        }
      }
      if (fin) final_pending = false;
      A.live = false;
    };
    // open the accumulator on the origin's cell so that the final samples always find it
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      A.base[q] = Tp.base[q];
      A.a[q][0] = A.a[q][1] = 0.f;
    }
    A.live = true;
    for (int i = V.n_fp - 1; i >= 0; --i) {
      const Taps Ti = traj_taps(V, bb, P[i][0], P[i][1]);
      if (A.live && A.base[0] != Ti.base[0]) flush();
      if (!A.live) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          A.base[q] = Ti.base[q];
          A.a[q][0] = A.a[q][1] = 0.f;
        }
        A.live = true;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        A.a[q][0] -= Ti.w[q] * gpx;
        A.a[q][1] -= Ti.w[q] * gpy;
      }
      const float2 j = traj_jt_it<K>(V, Ti, g, D, -gpx, -gpy);
      gpx = j.x;
      gpy = j.y;
    }
    flush();
    if (final_pending) {  // the iterations left the origin's cell: the final samples flush on their own
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        A.base[q] = Tp.base[q];
        A.a[q][0] = A.a[q][1] = 0.f;
      }
      A.live = true;
      flush();
    }
  }
}

inline int tgrid(long long n) { return clamp_grid(blocks_for(n, kTThreads)); }

template <typename F>
void dispatch_k(int K, F&& f) {
  switch (K) {
#define ATLB_K(k) \
  case k: f(std::integral_constant<int, k>{}); break;
    ATLB_K(1) ATLB_K(2) ATLB_K(3) ATLB_K(4) ATLB_K(5) ATLB_K(6) ATLB_K(7) ATLB_K(8)
    ATLB_K(9) ATLB_K(10) ATLB_K(11) ATLB_K(12) ATLB_K(13) ATLB_K(14) ATLB_K(15) ATLB_K(16)
#undef ATLB_K
    default: break;
  }
}

}  // namespace

int traj_transport(const TrajView& V, int mode, const float* xy, const float* t, const float* tdst, float tdst_s,
                   const long long* b, long long N, float* out, cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_fwd<K>, tgrid(N), kTThreads, 0, s, V, mode, (const float2*)xy, t, tdst, tdst_s, b, N,
             (float2*)out);
    });
    timing_end("k_traj_fwd", s, e0);
  }
  return launch_status("traj_transport");
}

int traj_transport_bwd(const TrajView& V, int mode, const float* gy, const float* xy, const float* t,
                       const float* tdst, float tdst_s, const long long* b, long long N, float* gC, float* gp,
                       cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_bwd<K>, tgrid(N), kTThreads, 0, s, V, mode, (const float2*)gy, (const float2*)xy, t, tdst, tdst_s,
             b, N, gC, (float2*)gp);
    });
    timing_end("k_traj_bwd", s, e0);
  }
  return launch_status("traj_transport_bwd");
}

int traj_records(const TrajView& V, int R, const float* xy, const float* t, const float* tdst, float tdst_s,
                 const long long* b, long long N, float* out, float* iters, cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_records_fwd<K>, tgrid(N * R), kTThreads, 0, s, V, R, (const float2*)xy, t, tdst, tdst_s, b, N,
             (float2*)out, (float2*)iters);
    });
    timing_end("k_traj_records_fwd", s, e0);
  }
  return launch_status("traj_records");
}

int traj_records_bwd(const TrajView& V, int R, const float* gy, const float* xy, const float* t, const float* tdst,
                     float tdst_s, const long long* b, long long N, const float* iters, float* gC, cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      if (iters)
        launch(k_traj_records_bwd<K, true>, tgrid(N * R), kTThreads, 0, s, V, R, (const float2*)gy,
               (const float2*)xy, t, tdst, tdst_s, b, N, (const float2*)iters, gC);
      else
        launch(k_traj_records_bwd<K, false>, tgrid(N * R), kTThreads, 0, s, V, R, (const float2*)gy,
               (const float2*)xy, t, tdst, tdst_s, b, N, (const float2*)nullptr, gC);
    });
    timing_end("k_traj_records_bwd", s, e0);
  }
  return launch_status("traj_records_bwd");
}

int traj_targets(const TrajView& V, const float* xy, const float* t, const long long* b, long long N,
                 const float* targets, int T, float* out, cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_targets_fwd<K>, tgrid(N), kTThreads, 0, s, V, (const float2*)xy, t, b, N, targets, T,
             (float2*)out);
    });
    timing_end("k_traj_targets_fwd", s, e0);
  }
  return launch_status("traj_targets");
}

int traj_targets_bwd(const TrajView& V, const float* gy, const float* xy, const float* t, const long long* b,
                     long long N, const float* targets, int T, float* gC, cudaStream_t s) {
  if (N > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_targets_bwd<K>, tgrid(N), kTThreads, 0, s, V, (const float2*)gy, (const float2*)xy, t, b, N,
             targets, T, gC);
    });
    timing_end("k_traj_targets_bwd", s, e0);
  }
  return launch_status("traj_targets_bwd");
}

int traj_targets_max() { return kTrajTargetsMax; }

int traj_visible_fraction(const TrajView& V, const float* xa, const float* ta, const long long* ba, long long M,
                          const float* counts, const float* centres, int n_check, float tau, float wmax, float hmax,
                          float* out, cudaStream_t s) {
  if (M > 0) {
    cudaEvent_t e0 = timing_begin(s);
    dispatch_k(V.K, [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      launch(k_traj_vis<K>, tgrid(M), kTThreads, 0, s, V, (const float2*)xa, ta, ba, M, counts, centres, n_check, tau,
             wmax, hmax, out);
    });
    timing_end("k_traj_vis", s, e0);
  }
  return launch_status("traj_visible_fraction");
}

}  // namespace atlb
