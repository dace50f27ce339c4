// Exact transport of affine velocity fields (atl/motion/parametric.py:60-71, mode="exact"): the flow of
// v(x) = A (x - c) + t over a time step dt is the affine map of the augmented matrix exponential
//     E = exp(Z),  Z = dt [[A, t], [0, 0]]  (3 x 3),     y = c + E[:2, :2] (x - c) + E[:2, 2].
// Translation (A = 0) and Affine (theta = (tx, ty, a11, a12, a21, a22)) use it.
//
// exp is evaluated by scaling and squaring with a Taylor polynomial (Horner), in fp32.  The number of halvings
// j is chosen from the linear part X = A dt alone (||X / 2^j||_1 <= 1/2): the powers of Z are
// [[X^k, X^(k-1) u], [0, 0]], so the translation column u = t dt enters every term linearly and the series
// converges at the rate of ||X|| whatever |u| is -- scaling by the whole matrix (|u| is tens of pixels) would
// square several times and multiply the rounding of the translation.  With |A dt| below 1/2 (the usual case) no
// squaring is needed at all.  Measured against float64: 2e-6 px, where torch's fp32 matrix_exp of the same
// matrix (the reference's call) deviates by up to 1.3e-4 px.
// Backward: with G = dL/dE (from dL/dy: G[i][j] = gy_i (x - c)_j, G[i][2] = gy_i), dL/dZ is the Frechet
// derivative of exp at Z^T in the direction G, the upper-right block of exp([[Z^T, G], [0, Z^T]]); the same
// scaling and squaring runs on (P, Q) pairs that stand for the block matrix [[P, Q], [0, P]]:
//     (P1, Q1) (P2, Q2) = (P1 P2, P1 Q2 + Q1 P2).
// Then dL/dA = dt dL/dZ[:2, :2], dL/dt = dt dL/dZ[:2, 2]; reduced per batch into dL/dtheta.
#include "common.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;
constexpr int kTaylor = 10;

struct M3 {
  float a[9];  // row-major
};

__device__ __forceinline__ M3 m3_zero() {
  M3 r;
#pragma unroll
  for (int i = 0; i < 9; ++i) r.a[i] = 0.f;
  return r;
}
__device__ __forceinline__ M3 m3_eye() {
  M3 r = m3_zero();
  r.a[0] = r.a[4] = r.a[8] = 1.f;
  return r;
}
__device__ __forceinline__ M3 m3_mul(const M3& x, const M3& y) {
  M3 r;
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      r.a[3 * i + j] = fmaf(x.a[3 * i], y.a[j], fmaf(x.a[3 * i + 1], y.a[3 + j], x.a[3 * i + 2] * y.a[6 + j]));
  return r;
}
__device__ __forceinline__ M3 m3_add(const M3& x, const M3& y) {
  M3 r;
#pragma unroll
  for (int i = 0; i < 9; ++i) r.a[i] = x.a[i] + y.a[i];
  return r;
}
__device__ __forceinline__ M3 m3_scale(const M3& x, float s) {
  M3 r;
#pragma unroll
  for (int i = 0; i < 9; ++i) r.a[i] = x.a[i] * s;
  return r;
}
__device__ __forceinline__ M3 m3_transpose(const M3& x) {
  M3 r;
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) r.a[3 * i + j] = x.a[3 * j + i];
  return r;
}

// ||.||_1 of the linear (upper-left 2 x 2) block.
__device__ __forceinline__ float lin_norm1(const M3& x) {
  return fmaxf(fabsf(x.a[0]) + fabsf(x.a[3]), fabsf(x.a[1]) + fabsf(x.a[4]));
}

// Number of halvings j with nrm / 2^j <= 1/2 (0 for a small or non-finite norm: the result is then
// non-finite as the reference's would be).
__device__ __forceinline__ int squarings(float nrm) {
  if (!(nrm > 0.5f) || !(nrm < 1e30f)) return 0;
  int e;
  frexpf(nrm, &e);  // nrm = f 2^e, f in [1/2, 1)
  return min(e + 1, 120);
}

// exp(Z).
__device__ __forceinline__ M3 expm3(M3 Z) {
  const int j = squarings(lin_norm1(Z));
  Z = m3_scale(Z, ldexpf(1.f, -j));
  M3 E = m3_eye();  // Horner: E = I + Z/k E, k = K..1
#pragma unroll
  for (int k = kTaylor; k >= 1; --k) E = m3_add(m3_eye(), m3_scale(m3_mul(Z, E), 1.f / (float)k));
  for (int i = 0; i < j; ++i) E = m3_mul(E, E);
  return E;
}

// The upper-right block L of exp([[P, Q], [0, P]]): the Frechet derivative of exp at P in the direction Q, for
// P = Z^T of an augmented matrix.  The upper-right block of the k-th power is sum_i P^i Q P^(k-1-i), whose
// terms decay like ||X||^(k-2) |u|^2 |Q|: the halvings follow ||X|| again, with two more Taylor terms.
constexpr int kTaylorFrechet = kTaylor + 2;
__device__ __forceinline__ M3 expm3_frechet(M3 P, M3 Q) {
  const int j = squarings(lin_norm1(P));
  const float s = ldexpf(1.f, -j);
  P = m3_scale(P, s);
  Q = m3_scale(Q, s);
  M3 EP = m3_eye(), EQ = m3_zero();  // (EP, EQ) = I + (P, Q)/k (EP, EQ)
#pragma unroll
  for (int k = kTaylorFrechet; k >= 1; --k) {
    const float ik = 1.f / (float)k;
    const M3 nP = m3_mul(P, EP);
    const M3 nQ = m3_add(m3_mul(P, EQ), m3_mul(Q, EP));
    EP = m3_add(m3_eye(), m3_scale(nP, ik));
    EQ = m3_scale(nQ, ik);
  }
  for (int i = 0; i < j; ++i) {
    const M3 q = m3_add(m3_mul(EP, EQ), m3_mul(EQ, EP));
    EP = m3_mul(EP, EP);
    EQ = q;
  }
  return EQ;
}

struct FlowView {
  int kind;  // ATLB_MOTION_TRANSLATION / _AFFINE
  const float* theta;
  long long B;
  float cx, cy;
};

// Z = dt [[A, t], [0, 0]] of event n's batch (the reference forms the product with dt in fp32).
__device__ __forceinline__ M3 flow_z(const FlowView& V, long long b, float dt) {
  M3 Z = m3_zero();
  const int np = V.kind == ATLB_MOTION_TRANSLATION ? 2 : 6;
  const float* th = V.theta + b * np;
  Z.a[2] = th[0] * dt;
  Z.a[5] = th[1] * dt;
  if (V.kind == ATLB_MOTION_AFFINE) {
    Z.a[0] = th[2] * dt;
    Z.a[1] = th[3] * dt;
    Z.a[3] = th[4] * dt;
    Z.a[4] = th[5] * dt;
  }
  return Z;
}

__global__ void __launch_bounds__(kThreads) k_flow_fwd(FlowView V, const float2* __restrict__ xy,
                                                       const float* __restrict__ t, const float* __restrict__ tdst,
                                                       float tdst_s, const long long* __restrict__ b, long long N,
                                                       float2* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const long long bb = b[n];
    if (bb < 0 || bb >= V.B) {
      out[n] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      continue;
    }
    const float dt = (tdst ? tdst[n] : tdst_s) - t[n];
    const M3 E = expm3(flow_z(V, bb, dt));
    const float2 p = xy[n];
    const float dx = p.x - V.cx, dy = p.y - V.cy;
    out[n] = make_float2(V.cx + (E.a[0] * dx + E.a[1] * dy) + E.a[2], V.cy + (E.a[3] * dx + E.a[4] * dy) + E.a[5]);
  }
}

// dL/dtheta (per batch, atomics after a warp reduction over runs of one batch) and dL/dxy (gxy, optional).
__global__ void __launch_bounds__(kThreads) k_flow_bwd(FlowView V, const float2* __restrict__ gy,
                                                       const float2* __restrict__ xy, const float* __restrict__ t,
                                                       const float* __restrict__ tdst, float tdst_s,
                                                       const long long* __restrict__ b, long long N,
                                                       float* __restrict__ gtheta, float2* __restrict__ gxy) {
  const int np = V.kind == ATLB_MOTION_TRANSLATION ? 2 : 6;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n0 = blockIdx.x * (long long)blockDim.x; n0 < N; n0 += stride) {  // warp-uniform trips
    const long long n = n0 + threadIdx.x;
    float c[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    long long bb = -1;
    if (n < N) {
      bb = b[n];
      if (bb >= 0 && bb < V.B) {
        const float dt = (tdst ? tdst[n] : tdst_s) - t[n];
        const M3 Z = flow_z(V, bb, dt);
        const float2 g = gy[n], p = xy[n];
        const float dx = p.x - V.cx, dy = p.y - V.cy;
        M3 G = m3_zero();
        G.a[0] = g.x * dx; G.a[1] = g.x * dy; G.a[2] = g.x;
        G.a[3] = g.y * dx; G.a[4] = g.y * dy; G.a[5] = g.y;
        const M3 D = expm3_frechet(m3_transpose(Z), G);  // dL/dZ
        c[0] = D.a[2] * dt;
        c[1] = D.a[5] * dt;
        c[2] = D.a[0] * dt; c[3] = D.a[1] * dt; c[4] = D.a[3] * dt; c[5] = D.a[4] * dt;
        if (gxy) {
          const M3 E = expm3(Z);
          gxy[n] = make_float2(E.a[0] * g.x + E.a[3] * g.y, E.a[1] * g.x + E.a[4] * g.y);
        }
      } else {
        bb = -1;
        if (gxy) gxy[n] = make_float2(0.f, 0.f);
      }
    }
    const long long b0 = __shfl_sync(0xffffffffu, bb, 0);
    if (__all_sync(0xffffffffu, bb == b0)) {
      for (int q = 0; q < np; ++q) c[q] = warp_sum(c[q]);
      if ((threadIdx.x & 31) == 0 && b0 >= 0)
        for (int q = 0; q < np; ++q) atomicAdd(gtheta + b0 * np + q, c[q]);
    } else if (bb >= 0) {
      for (int q = 0; q < np; ++q) atomicAdd(gtheta + bb * np + q, c[q]);
    }
  }
}

}  // namespace

int flow_exact(int kind, const float* theta, long long B, long long H, long long W, const float* xy, const float* t,
               const float* t_dst, double t_dst_s, const long long* b, long long N, float* out, cudaStream_t s) {
  const FlowView V{kind, theta, B, (float)((W - 1) / 2.0), (float)((H - 1) / 2.0)};
  if (N > 0)
    launch(k_flow_fwd, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, V, (const float2*)xy, t, t_dst,
           (float)t_dst_s, b, N, (float2*)out);
  return launch_status("flow_exact");
}

int flow_exact_bwd(int kind, const float* gy, const float* theta, long long B, long long H, long long W,
                   const float* xy, const float* t, const float* t_dst, double t_dst_s, const long long* b, long long N,
                   float* gtheta, float* gxy, cudaStream_t s) {
  const FlowView V{kind, theta, B, (float)((W - 1) / 2.0), (float)((H - 1) / 2.0)};
  cudaMemsetAsync(gtheta, 0, (size_t)(B * (kind == ATLB_MOTION_TRANSLATION ? 2 : 6)) * 4, s);
  if (N > 0)
    launch(k_flow_bwd, clamp_grid(blocks_for(N, kThreads)), kThreads, 0, s, V, (const float2*)gy, (const float2*)xy,
           t, t_dst, (float)t_dst_s, b, N, gtheta, (float2*)gxy);
  return launch_status("flow_exact_bwd");
}

}  // namespace atlb
