// Device pair plan: the B200 replacement of build_pair_plan (atl/ops/functional.py:132-178).
//
// The reference builds the plan with ~15 torch ops on the host side (repeat_interleave, argsort of
// N*S int64 keys, bincount, cumsum).  Here it is a counting sort: one pass counts the (source, slice)
// entries per cell with L2 atomics, a scan turns the counts into CSR offsets, a second pass
// scatters the entries.  Nothing is sorted by comparison; the keys are recomputed in each pass
// (a few FLOPs) instead of being stored (8 bytes per entry).
#include <stdio.h>

#include <cmath>

#include "common.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;

// scratch ints: [0] vmax bits, [1] min x, [2] min y, [3] max x, [4] max y (ordered ints),
// [5] set when an anchor index lies outside [0, N)
__global__ void k_geom_init(int* r) {
  if (threadIdx.x == 0) {
    r[0] = 0;
    r[1] = 0x7fffffff; r[2] = 0x7fffffff;
    r[3] = (int)0x80000000; r[4] = (int)0x80000000;
    r[5] = 0;
  }
}

// Anchor positions: anchor_xy[i] if given, else x[anchors[i]] (functional.py:142).
__global__ void __launch_bounds__(kThreads) k_geom_reduce(const float2* __restrict__ v, long long N,
                                                          const float2* __restrict__ x,
                                                          const long long* __restrict__ anchors,
                                                          const float2* __restrict__ anchor_xy, long long M, int* r) {
  float vm = 0.f;
  int mnx = 0x7fffffff, mny = 0x7fffffff, mxx = (int)0x80000000, mxy = (int)0x80000000;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N || j < M; j += stride) {
    if (j < N) {
      const float2 q = v[j];
      const float n = row_norm(q.x, q.y);
      vm = (n > vm || n != n) ? n : vm;
    }
    if (j < M) {
      const long long ai = anchors[j];
      if (ai < 0 || ai >= N) {
        r[5] = 1;
      } else {
        const float2 a = anchor_xy ? anchor_xy[j] : x[ai];
        const int ox = float_to_ordered(a.x), oy = float_to_ordered(a.y);
        mnx = min(mnx, ox); mny = min(mny, oy); mxx = max(mxx, ox); mxy = max(mxy, oy);
      }
    }
  }
  // vm >= 0 (or NaN, whose bits exceed every finite value): int max on the raw bits is the float max
  int vb = __float_as_int(vm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    vb = max(vb, __shfl_xor_sync(0xffffffffu, vb, o));
    mnx = min(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
    mny = min(mny, __shfl_xor_sync(0xffffffffu, mny, o));
    mxx = max(mxx, __shfl_xor_sync(0xffffffffu, mxx, o));
    mxy = max(mxy, __shfl_xor_sync(0xffffffffu, mxy, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(r + 0, vb);
    atomicMin(r + 1, mnx); atomicMin(r + 2, mny);
    atomicMax(r + 3, mxx); atomicMax(r + 4, mxy);
  }
}

// Slice-major passes: blockIdx.y walks the slices, so at any moment the writes of the scatter pass
// land in one slice's part of the plan (~1/S of it), which stays in L2 until its sectors are full.
__global__ void __launch_bounds__(kThreads) k_plan_count(PlanConsts P, const float2* __restrict__ x,
                                                         const float* __restrict__ t, const float2* __restrict__ v,
                                                         const long long* __restrict__ b, long long N,
                                                         int* __restrict__ counts) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (int s = blockIdx.y; s < P.S; s += gridDim.y) {
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
      const float tj = t[j];
      int s_lo, s_hi;
      slice_range(P, tj, &s_lo, &s_hi);
      if (s < s_lo || s > s_hi) continue;
      const float2 xj = x[j], vj = v[j];
      float yx, yy;
      const long long key = source_key(P, xj.x, xj.y, vj.x, vj.y, tj, b[j], s, &yx, &yy);
      if (key >= 0) atomicAdd(counts + key, 1);
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_plan_scatter(PlanConsts P, const float2* __restrict__ x,
                                                           const float* __restrict__ t, const float2* __restrict__ v,
                                                           const long long* __restrict__ b, long long N,
                                                           const long long* __restrict__ cell_start,
                                                           int* __restrict__ cursor, float2* __restrict__ src_y,
                                                           float2* __restrict__ src_v, float* __restrict__ src_t,
                                                           long long* __restrict__ src_id) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (int s = blockIdx.y; s < P.S; s += gridDim.y) {
    for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
      const float tj = t[j];
      int s_lo, s_hi;
      slice_range(P, tj, &s_lo, &s_hi);
      if (s < s_lo || s > s_hi) continue;
      const float2 xj = x[j], vj = v[j];
      float yx, yy;
      const long long key = source_key(P, xj.x, xj.y, vj.x, vj.y, tj, b[j], s, &yx, &yy);
      if (key < 0) continue;
      const long long p = cell_start[key] + atomicAdd(cursor + key, 1);
      src_y[p] = make_float2(yx, yy);
      src_v[p] = vj;
      src_t[p] = tj;
      src_id[p] = j;
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_plan_anchors(PlanConsts P, const float2* __restrict__ x,
                                                           const float* __restrict__ t,
                                                           const long long* __restrict__ b,
                                                           const long long* __restrict__ anchors,
                                                           const float2* __restrict__ anchor_xy, long long M,
                                                           long long N, float2* __restrict__ anc_x, float* __restrict__ anc_t,
                                                           long long* __restrict__ anc_cell,
                                                           long long* __restrict__ anc_id, float* __restrict__ slice_c) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i0 < P.S) slice_c[i0] = slice_centre(P, (int)i0);
  for (long long i = i0; i < M; i += stride) {
    const long long a = anchors[i];
    if (a < 0 || a >= N) {  // invalid anchor index: no cell (the pair kernels report NaN for it)
      anc_x[i] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      anc_t[i] = __int_as_float(0x7fc00000);
      anc_cell[3 * i] = -1; anc_cell[3 * i + 1] = -1; anc_cell[3 * i + 2] = -1;
      anc_id[i] = a;
      continue;
    }
    const float ta = t[a];
    const float2 xa = anchor_xy ? anchor_xy[i] : x[a];
    long long g, cx, cy;
    anchor_cell(P, xa.x, xa.y, ta, b[a], &g, &cx, &cy);
    anc_x[i] = xa;
    anc_t[i] = ta;
    anc_cell[3 * i] = g; anc_cell[3 * i + 1] = cx; anc_cell[3 * i + 2] = cy;
    anc_id[i] = a;
  }
}

}  // namespace

// (x over events, y over slices): enough CTAs to fill the GPU, slices striding by gridDim.y.
dim3 slice_grid(long long N, int S) {
  const long long bx = blocks_for(N, kThreads);
  const long long by = S < 65535 ? S : 65535;
  const long long cap = 148LL * 32;
  long long gx = bx;
  if (gx * by > cap) gx = (cap + by - 1) / by;
  return dim3((unsigned)(gx < 1 ? 1 : gx), (unsigned)by, 1);
}

static inline float __int_as_float_host(int i) {
  float f;
  memcpy(&f, &i, 4);
  return f;
}

// Host-side geometry, functional.py:139-149, in double exactly as the reference's Python computes it.
void plan_geometry_host(float vmax, bool have_anchors, float mnx, float mny, float mxx, float mxy, long long H,
                        long long W, double h, double cut, long long S, atlb_plan_geom* g) {
  const double delta = 1.0 / (double)S;
  double cell = cut * h + (double)vmax * delta / 2 + 1e-3;
  if (!(cell >= 1.0)) cell = (cell != cell) ? cell : 1.0;
  double ox, oy, ex, ey;
  if (have_anchors) {
    ox = (double)mnx - cell; oy = (double)mny - cell;
    ex = (double)mxx + cell; ey = (double)mxy + cell;
  } else {
    ox = -cell; oy = -cell; ex = (double)W + cell; ey = (double)H + cell;
  }
  g->cell = cell; g->ox = ox; g->oy = oy;
  g->GW = (int64_t)std::ceil((ex - ox) / cell) + 1;
  g->GH = (int64_t)std::ceil((ey - oy) / cell) + 1;
  g->vmax = vmax;
  g->S = (int32_t)S;
  g->t_lo = __int_as_float_host(0x7fc00000);
  g->t_hi = __int_as_float_host(0x7fc00000);
}

PlanConsts make_plan_consts(const atlb_plan_geom& g, double tau, long long B) {
  PlanConsts P;
  const double delta = 1.0 / (double)g.S;
  P.tau_f = (float)tau;
  P.hd_f = (float)(delta / 2);
  P.delta_f = (float)delta;
  P.ox_f = (float)g.ox;
  P.oy_f = (float)g.oy;
  P.cell_f = (float)g.cell;
  volatile float one = 1.f;  // an fp32 division on the host: RN(1 / cell_f)
  P.rcell_f = one / P.cell_f;
  P.GW = g.GW;
  P.GH = g.GH;
  P.S = g.S;
  P.B = B;
  P.src0 = 0;
  P.src1 = LLONG_MAX;
  P.rfine_f = (float)((double)kFine / g.cell);
  P.GWf = g.GW * kFine;
  P.GHf = g.GH * kFine;
  return P;
}

int plan_geometry(const float* x, const float* v, long long N, const long long* anchors, const float* anchor_xy,
                  long long M, long long H, long long W, double h, double cut, long long S, void* scratch,
                  atlb_plan_geom* out, cudaStream_t s) {
  int* r = (int*)scratch;
  launch(k_geom_init, 1, 32, 0, s, r);
  const long long n = N > M ? N : M;
  if (n > 0) {
    launch(k_geom_reduce, clamp_grid(blocks_for(n, kThreads)), kThreads, 0, s, (const float2*)v, N, (const float2*)x,
           anchors, (const float2*)anchor_xy, M, r);
  }
  int host[6];
  if (cudaMemcpyAsync(host, r, sizeof(host), cudaMemcpyDeviceToHost, s) != cudaSuccess) return launch_status("plan_geometry copy");
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("plan_geometry sync");
  if (host[5]) {
    set_error("build_pair_plan: an anchor index lies outside [0, %lld)", N);
    return ATLB_ERR_ARG;
  }
  float vmax;
  memcpy(&vmax, &host[0], 4);
  plan_geometry_host(N > 0 ? vmax : 0.f, M > 0, ordered_to_float(host[1]), ordered_to_float(host[2]),
                     ordered_to_float(host[3]), ordered_to_float(host[4]), H, W, h, cut, S, out);
  return launch_status("plan_geometry");
}

size_t plan_workspace_bytes(long long ncell) {
  return align_up((size_t)ncell * sizeof(int)) + align_up(scan_partials_bytes(ncell)) + 256;
}

int plan_count(const float* x, const float* t, const float* v, const long long* b, long long N, long long B,
               double tau, const atlb_plan_geom* g, long long* cell_start, void* ws, long long* n_entries,
               cudaStream_t s) {
  const long long ncell = B * (long long)g->S * g->GH * g->GW;
  char* p = (char*)align_ptr(ws);
  int* counts = (int*)p;
  long long* partials = (long long*)(p + align_up((size_t)ncell * sizeof(int)));
  cudaMemsetAsync(counts, 0, (size_t)ncell * sizeof(int), s);
  const PlanConsts P = make_plan_consts(*g, tau, B);
  if (N > 0) launch(k_plan_count, slice_grid(N, P.S), kThreads, 0, s, P, (const float2*)x, t, (const float2*)v, b, N, counts);
  exclusive_scan<long long>(counts, ncell, partials, cell_start, s);
  if (cudaMemcpyAsync(n_entries, cell_start + ncell, sizeof(long long), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return launch_status("plan_count copy");
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("plan_count sync");
  return launch_status("plan_count");
}

int plan_fill(const float* x, const float* t, const float* v, const long long* b, long long N, long long B, double tau,
              const atlb_plan_geom* g, const long long* anchors, const float* anchor_xy, long long M,
              const long long* cell_start, void* ws, float* src_y, float* src_v, float* src_t, long long* src_id,
              float* anc_x, float* anc_t, long long* anc_cell, long long* anc_id, float* slice_c, cudaStream_t s) {
  char* p = (char*)align_ptr(ws);
  int* cursor = (int*)p;  // zeroed by the scan of plan_count
  const PlanConsts P = make_plan_consts(*g, tau, B);
  if (N > 0)
    launch(k_plan_scatter, slice_grid(N, P.S), kThreads, 0, s, P, (const float2*)x, t, (const float2*)v, b, N,
           cell_start, cursor, (float2*)src_y, (float2*)src_v, src_t, src_id);
  const long long na = M > P.S ? M : P.S;
  launch(k_plan_anchors, clamp_grid(blocks_for(na, kThreads)), kThreads, 0, s, 
      P, (const float2*)x, t, b, anchors, (const float2*)anchor_xy, M, N, (float2*)anc_x, anc_t, anc_cell, anc_id,
      slice_c);
  return launch_status("plan_fill");
}

}  // namespace atlb
