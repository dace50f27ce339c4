// Bilinear splat, gather and voxel kernels of the sliced path (csrc/atl_cpu.cpp:17-76, 134-172, 256-286); the
// Gaussian splat is in gauss_tiled.cu.
//
// Each output keeps the reference's per-element rounding sequence.  Scatters go to L2 with
// fire-and-forget red.global (no return value, no retry loop); gathers are one thread per event.
#include "common.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;

// bilinear_corners (atl_cpu.cpp:17-33): f(yy, xx, weight, dweight/dx, dweight/dy) for the in-image corners.
template <typename F>
__device__ __forceinline__ void bilinear_corners(float x, float y, long long H, long long W, F&& f) {
  if (!(fabsf(x) < 1e18f && fabsf(y) < 1e18f)) return;  // no in-image corner (and no int64 overflow)
  const float fx0 = floorf(x), fy0 = floorf(y);
  const long long x0 = (long long)fx0, y0 = (long long)fy0;
  const float ax = sub_rn(x, fx0), ay = sub_rn(y, fy0);
  const float wx0 = sub_rn(1.f, ax), wy0 = sub_rn(1.f, ay);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const long long yy = y0 + j;
    if (yy < 0 || yy >= H) continue;
    const float wy = j ? ay : wy0, dwy = j ? 1.f : -1.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const long long xx = x0 + i;
      if (xx < 0 || xx >= W) continue;
      const float wx = i ? ax : wx0, dwx = i ? 1.f : -1.f;
      f(yy, xx, mul_rn(wx, wy), mul_rn(dwx, wy), mul_rn(wx, dwy));
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_splat_bilinear_fwd(const float2* __restrict__ P,
                                                                 const float* __restrict__ Wt,
                                                                 const long long* __restrict__ Bi, long long N,
                                                                 long long B, long long H, long long W,
                                                                 float* __restrict__ I) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float wn = Wt[n];
    if (wn == 0.f || Bi[n] < 0 || Bi[n] >= B) continue;
    const float2 p = P[n];
    float* base = I + Bi[n] * H * W;
    bilinear_corners(p.x, p.y, H, W, [&](long long yy, long long xx, float c, float, float) {
      red_add_f1(base + yy * W + xx, mul_rn(wn, c));
    });
  }
}

__global__ void __launch_bounds__(kThreads) k_splat_bilinear_bwd(const float* __restrict__ G,
                                                                 const float2* __restrict__ P,
                                                                 const float* __restrict__ Wt,
                                                                 const long long* __restrict__ Bi, long long N,
                                                                 long long B, long long H, long long W,
                                                                 float2* __restrict__ GP, float* __restrict__ GW) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 p = P[n];
    const long long bb = Bi[n];
    const float* base = G + bb * H * W;
    float sx = 0.f, sy = 0.f, sw = 0.f;
    if (bb >= 0 && bb < B) bilinear_corners(p.x, p.y, H, W, [&](long long yy, long long xx, float c, float dcx, float dcy) {
      const float g = __ldg(base + yy * W + xx);
      sw = add_rn(sw, mul_rn(g, c));
      sx = add_rn(sx, mul_rn(g, dcx));
      sy = add_rn(sy, mul_rn(g, dcy));
    });
    const float wn = Wt[n];
    GW[n] = sw;
    GP[n] = make_float2(mul_rn(wn, sx), mul_rn(wn, sy));
  }
}

__global__ void __launch_bounds__(kThreads) k_gather_fwd(const float* __restrict__ I, const float2* __restrict__ P,
                                                         const long long* __restrict__ Bi, long long N, long long B,
                                                         long long H, long long W, float* __restrict__ O) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 p = P[n];
    const long long bb = Bi[n];
    const float* base = I + bb * H * W;
    float s = 0.f;
    if (bb >= 0 && bb < B) bilinear_corners(p.x, p.y, H, W, [&](long long yy, long long xx, float c, float, float) {
      s = add_rn(s, mul_rn(c, __ldg(base + yy * W + xx)));
    });
    O[n] = s;
  }
}

__global__ void __launch_bounds__(kThreads) k_gather_bwd(const float* __restrict__ GV, const float* __restrict__ I,
                                                         const float2* __restrict__ P,
                                                         const long long* __restrict__ Bi, long long N, long long B,
                                                         long long H, long long W, float* __restrict__ GI,
                                                         float2* __restrict__ GP) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float g = GV[n];
    const float2 p = P[n];
    const long long bb = Bi[n];
    const float* base = I + bb * H * W;
    float* gbase = GI + bb * H * W;
    float sx = 0.f, sy = 0.f;
    if (bb >= 0 && bb < B) bilinear_corners(p.x, p.y, H, W, [&](long long yy, long long xx, float c, float dcx, float dcy) {
      const float v = __ldg(base + yy * W + xx);
      sx = add_rn(sx, mul_rn(dcx, v));
      sy = add_rn(sy, mul_rn(dcy, v));
      red_add_f1(gbase + yy * W + xx, mul_rn(g, c));
    });
    GP[n] = make_float2(mul_rn(g, sx), mul_rn(g, sy));
  }
}

__global__ void __launch_bounds__(kThreads) k_voxel(const float2* __restrict__ P, const float* __restrict__ T,
                                                    const float* __restrict__ Pol, const long long* __restrict__ Bi,
                                                    long long N, long long B, long long C, long long H, long long W,
                                                    float* __restrict__ V) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long n = blockIdx.x * (long long)blockDim.x + threadIdx.x; n < N; n += stride) {
    const float2 p = P[n];
    const float tn = mul_rn(T[n], (float)(C - 1));
    const long long bb = Bi[n];
    if (bb < 0 || bb >= B || !(fabsf(p.x) < 1e18f && fabsf(p.y) < 1e18f && fabsf(tn) < 1e18f)) continue;
    const long long x0 = (long long)floorf(p.x), y0 = (long long)floorf(p.y), t0 = (long long)floorf(tn);
    const float pol = Pol[n];
    for (int dt = 0; dt < 2; ++dt) {
      const long long tt = t0 + dt;
      if (tt < 0 || tt >= C) continue;
      const float wt = sub_rn(1.f, fabsf(sub_rn((float)tt, tn)));
      for (int dy = 0; dy < 2; ++dy) {
        const long long yy = y0 + dy;
        if (yy < 0 || yy >= H) continue;
        const float wy = sub_rn(1.f, fabsf(sub_rn((float)yy, p.y)));
        for (int dx = 0; dx < 2; ++dx) {
          const long long xx = x0 + dx;
          if (xx < 0 || xx >= W) continue;
          const float wx = sub_rn(1.f, fabsf(sub_rn((float)xx, p.x)));
          red_add_f1(V + ((bb * C + tt) * H + yy) * W + xx, mul_rn(mul_rn(mul_rn(pol, wt), wy), wx));
        }
      }
    }
  }
}

inline int grid_for(long long n) { return clamp_grid(blocks_for(n, kThreads)); }

}  // namespace

int splat_bilinear_fwd(const float* pos, const float* w, const long long* b, long long N, long long B, long long H,
                       long long W, float* img, cudaStream_t s) {
  cudaMemsetAsync(img, 0, (size_t)(B * H * W) * sizeof(float), s);
  if (N > 0) launch(k_splat_bilinear_fwd, grid_for(N), kThreads, 0, s, (const float2*)pos, w, b, N, B, H, W, img);
  return launch_status("splat_bilinear_fwd");
}

int splat_bilinear_bwd(const float* g, const float* pos, const float* w, const long long* b, long long N, long long B,
                       long long H, long long W, float* gpos, float* gw, cudaStream_t s) {
  if (N > 0)
    launch(k_splat_bilinear_bwd, grid_for(N), kThreads, 0, s, g, (const float2*)pos, w, b, N, B, H, W, (float2*)gpos, gw);
  return launch_status("splat_bilinear_bwd");
}

int gather_fwd(const float* img, const float* pos, const long long* b, long long N, long long B, long long H,
               long long W, float* out, cudaStream_t s) {
  if (N > 0) launch(k_gather_fwd, grid_for(N), kThreads, 0, s, img, (const float2*)pos, b, N, B, H, W, out);
  return launch_status("gather_bilinear_fwd");
}

int gather_bwd(const float* g, const float* img, const float* pos, const long long* b, long long N, long long B,
               long long H, long long W, float* gimg, float* gpos, cudaStream_t s) {
  cudaMemsetAsync(gimg, 0, (size_t)(B * H * W) * sizeof(float), s);
  if (N > 0)
    launch(k_gather_bwd, grid_for(N), kThreads, 0, s, g, img, (const float2*)pos, b, N, B, H, W, gimg, (float2*)gpos);
  return launch_status("gather_bilinear_bwd");
}

int voxel_grid(const float* pos, const float* t, const float* p, const long long* b, long long N, long long B,
               long long C, long long H, long long W, float* vox, cudaStream_t s) {
  cudaMemsetAsync(vox, 0, (size_t)(B * C * H * W) * sizeof(float), s);
  if (N > 0) launch(k_voxel, grid_for(N), kThreads, 0, s, (const float2*)pos, t, p, b, N, B, C, H, W, vox);
  return launch_status("voxel_grid");
}

}  // namespace atlb
