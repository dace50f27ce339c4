// Fused AnchoredExact (atl/objectives/ats.py:75-96) for the motion fields of motion_math.cuh.
//
// The reference runs ~40 torch ops and four extension calls per score evaluation, with the plan built
// by host-orchestrated torch ops.  Here one score is:
//   prepare   one pass over the events: dequantised position xs = xy + (u - 1/2), velocity v(xs),
//             packed (xs, v) record, vmax and (b, t)-order checks; one pass over the anchors:
//             xa = xs[a] + h z and the anchors' bounding box                       [1 host read]
//   forward   count + scan + scatter of the (source, slice) entries into a compact 24-byte layout (the
//             events walked in mid-slice cell order, warp-aggregated cursors; optionally a range of the
//             events as sources, for one window split over GPUs), anchors bucketed by cell, per-anchor
//             normaliser W_i * vis_i * 2 pi h^2
//             (window count + exposure correction fused), pair sums with the log score written
//             directly (log(eps + S / den)).
//   backward  dL/dS from the upstream dL/dls, source-centric pair gradient, velocity-field gradient.
// Every step keeps the reference's rounding, so scores match it to float accuracy and the plan's
// cells are the reference's cells.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <mutex>

#include "common.cuh"
#include "motion_math.cuh"
#include "pair_kernels.cuh"
#include "pair_fine.cuh"
#include "pair_tiled.cuh"
#include "plan_math.cuh"
#include "rng.cuh"
#include "scan.cuh"

namespace atlb {

void plan_geometry_host(float vmax, bool have_anchors, float mnx, float mny, float mxx, float mxy, long long H,
                        long long W, double h, double cut, long long S, atlb_plan_geom* g);
PlanConsts make_plan_consts(const atlb_plan_geom& g, double tau, long long B);
dim3 slice_grid(long long N, int S);

namespace {

constexpr int kThreads = 256;
inline int grid_for(long long n) { return clamp_grid(blocks_for(n, kThreads)); }

// scratch ints: [0] vmax bits, [1..4] anchor bbox (ordered ints), [5] bad anchor index,
// [6] events not sorted by (b, t), [7] batch index outside [0, B), [8] / [9] min / max t (ordered ints)
__global__ void k_exact_init(int* r) {
  if (threadIdx.x == 0) {
    r[0] = 0;
    r[1] = 0x7fffffff; r[2] = 0x7fffffff;
    r[3] = (int)0x80000000; r[4] = (int)0x80000000;
    r[5] = 0; r[6] = 0; r[7] = 0;
    r[8] = 0x7fffffff; r[9] = (int)0x80000000;
  }
}

// rng: u == NULL and rng set -> the dequantisation jitter is drawn on the device (stream 0 of rng.cuh)
// 5 CTAs per SM (51 registers, no spills; 4 at the uncapped 64): the kernel waits on its loads and the flow taps
template <bool RNG>  // compiled with and without the device draw, which needs registers of its own
__global__ void __launch_bounds__(kThreads, 5) k_exact_events(MotionView Mv, const float2* __restrict__ xy,
                                                           const float2* __restrict__ u, const float* __restrict__ t,
                                                           const long long* __restrict__ b, long long N, long long B,
                                                           RngKey K, float4* __restrict__ ev4, int* r) {
  float vm = 0.f;
  int unsorted = 0, badb = 0, tmn = 0x7fffffff, tmx = (int)0x80000000;
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const int ot = float_to_ordered(t[j]);
    tmn = min(tmn, ot);
    tmx = max(tmx, ot);
    float2 p = xy[j];
    if (u || RNG) {  // ats.py:84-85: xs = xy + (u - 0.5)
      const float2 q = (RNG && !u) ? rng_uniform2(K, (unsigned long long)j) : u[j];
      p = make_float2(add_rn(p.x, sub_rn(q.x, 0.5f)), add_rn(p.y, sub_rn(q.y, 0.5f)));
    }
    const long long bj = b[j];
    float2 v;
    if (bj >= 0 && bj < B && bj < Mv.B) {
      v = motion_field(Mv, p.x, p.y, bj);
    } else {
      v = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
      badb = 1;
    }
    ev4[j] = make_float4(p.x, p.y, v.x, v.y);
    const float n = row_norm(v.x, v.y);
    vm = (n > vm || n != n) ? n : vm;
    if (j + 1 < N) {
      const double k0 = (double)bj * 4.0 + (double)t[j], k1 = (double)b[j + 1] * 4.0 + (double)t[j + 1];
      if (!(k0 <= k1)) unsorted = 1;
    }
  }
  int vb = __float_as_int(vm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    vb = max(vb, __shfl_xor_sync(0xffffffffu, vb, o));
    unsorted |= __shfl_xor_sync(0xffffffffu, unsorted, o);
    badb |= __shfl_xor_sync(0xffffffffu, badb, o);
    tmn = min(tmn, __shfl_xor_sync(0xffffffffu, tmn, o));
    tmx = max(tmx, __shfl_xor_sync(0xffffffffu, tmx, o));
  }
  // one atomic per CTA and quantity (warp results combined in shared memory first)
  __shared__ int red[5];
  if (threadIdx.x == 0) {
    red[0] = 0; red[1] = 0; red[2] = 0; red[3] = 0x7fffffff; red[4] = (int)0x80000000;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    atomicMax(red + 0, vb);
    atomicOr(red + 1, unsorted);
    atomicOr(red + 2, badb);
    atomicMin(red + 3, tmn);
    atomicMax(red + 4, tmx);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicMax(r + 0, red[0]);
    if (red[1]) atomicOr(r + 6, 1);
    if (red[2]) atomicOr(r + 7, 1);
    atomicMin(r + 8, red[3]);
    atomicMax(r + 9, red[4]);
  }
}

template <bool RNG>  // compiled with and without the device draw, as k_exact_events
__global__ void __launch_bounds__(kThreads) k_exact_anchors(const float4* __restrict__ ev4,
                                                            const float* __restrict__ t,
                                                            const long long* __restrict__ b, long long N,
                                                            const long long* __restrict__ anchors,
                                                            const float2* __restrict__ z, RngKey K,
                                                            float h_f, long long M,
                                                            float4* __restrict__ anc4, long long* __restrict__ anc_b,
                                                            int* r) {
  int mnx = 0x7fffffff, mny = 0x7fffffff, mxx = (int)0x80000000, mxy = (int)0x80000000, bad = 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const long long a = anchors ? anchors[i] : i;
    if (a < 0 || a >= N) {
      bad = 1;
      anc4[i] = make_float4(0.f, 0.f, 0.f, __int_as_float(-1));
      anc_b[i] = -1;
      continue;
    }
    const float4 e = ev4[a];
    float xa = e.x, ya = e.y;
    if (z || RNG) {  // ats.py:87-88: xa = xs[a] + h * z (z drawn on the device: stream 1 of rng.cuh)
      const float2 q = (RNG && !z) ? rng_normal2(K, (unsigned long long)i) : z[i];
      xa = add_rn(xa, mul_rn(h_f, q.x));
      ya = add_rn(ya, mul_rn(h_f, q.y));
    }
    anc4[i] = make_float4(xa, ya, t[a], __int_as_float((int)a));
    anc_b[i] = b[a];
    const int ox = float_to_ordered(xa), oy = float_to_ordered(ya);
    mnx = min(mnx, ox); mny = min(mny, oy); mxx = max(mxx, ox); mxy = max(mxy, oy);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mnx = min(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
    mny = min(mny, __shfl_xor_sync(0xffffffffu, mny, o));
    mxx = max(mxx, __shfl_xor_sync(0xffffffffu, mxx, o));
    mxy = max(mxy, __shfl_xor_sync(0xffffffffu, mxy, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  __shared__ int red[5];
  if (threadIdx.x == 0) {
    red[0] = 0x7fffffff; red[1] = 0x7fffffff; red[2] = (int)0x80000000; red[3] = (int)0x80000000; red[4] = 0;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    atomicMin(red + 0, mnx); atomicMin(red + 1, mny);
    atomicMax(red + 2, mxx); atomicMax(red + 3, mxy);
    atomicOr(red + 4, bad);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicMin(r + 1, red[0]); atomicMin(r + 2, red[1]);
    atomicMax(r + 3, red[2]); atomicMax(r + 4, red[3]);
    if (red[4]) atomicOr(r + 5, 1);
  }
}

// ---- compact plan -------------------------------------------------------------------------------------
// ---- spatial order of the events for the plan passes ------------------------------------------------
// The count and scatter passes walk the events in the order of their sub-cell at the middle slice, i.e. of
// where each event sits at mid-window under its own motion.  Under a smooth motion field, events that
// share that sub-cell stay within a few sub-cells of one another at every slice, so the 32 lanes of a warp
// fall into a handful of sub-cells: one cursor atomic per distinct sub-cell (warp-aggregated with
// match.any), and the lanes of one sub-cell write consecutive slots.  The order only decides where inside a
// sub-cell an entry lands; the keys themselves come from source_fine_key, unchanged.
__device__ __forceinline__ int order_key(const PlanConsts& P, float4 e, float t, int b) {
  const float dtc = slice_centre(P, P.S / 2) - t;
  const float qx = floorf((e.x + e.z * dtc - P.ox_f) * P.rfine_f);
  const float qy = floorf((e.y + e.w * dtc - P.oy_f) * P.rfine_f);
  const int cx = (int)fminf(fmaxf(qx, 0.f), (float)(P.GWf - 1));  // NaN -> 0
  const int cy = (int)fminf(fmaxf(qy, 0.f), (float)(P.GHf - 1));
  const int bb = (b >= 0 && b < P.B) ? b : 0;
  return (bb * (int)P.GHf + cy) * (int)P.GWf + cx;
}

__global__ void __launch_bounds__(kThreads) k_order_count(PlanConsts P, const float4* __restrict__ ev4,
                                                          const float* __restrict__ t,
                                                          const long long* __restrict__ b, long long N,
                                                          int* __restrict__ ocount) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride)
    atomicAdd(ocount + order_key(P, ev4[j], t[j], (int)b[j]), 1);
}

// XVo[i] = (x, y, vx, vy) and TBo[i] = (t bits, b, original index, 0) of the i-th event in that order;
// the arrays passed start at event id0.
__global__ void __launch_bounds__(kThreads) k_order_scatter(PlanConsts P, const float4* __restrict__ ev4,
                                                            const float* __restrict__ t,
                                                            const long long* __restrict__ b, long long N,
                                                            long long id0, int* __restrict__ ocursor,
                                                            float4* __restrict__ XVo,
                                                            int4* __restrict__ TBo) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const float4 e = ev4[j];
    const float tj = t[j];
    const int bj = (int)b[j];
    const int key = order_key(P, e, tj, bj);
    const int pos = atomicAdd(ocursor + key, 1);  // the cursors start at the offsets
    XVo[pos] = e;
    TBo[pos] = make_int4(__float_as_int(tj), bj, (int)(id0 + j), 0);
  }
}

// Plan entry counts over the ordered events; one atomic per distinct cell of a warp.  Keys fit in int
// (the cell count is checked against the int32 range by the caller).  One event per lane, its slices in an
// inner loop: the event is read and its slice range computed once, not once per slice.
__global__ void __launch_bounds__(kThreads) k_fast_count_ordered(PlanConsts P, const float4* __restrict__ XVo,
                                                                 const int4* __restrict__ TBo, long long N,
                                                                 int* __restrict__ counts, int* __restrict__ KEY) {
  const int lane = threadIdx.x & 31;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = blockIdx.x * (long long)blockDim.x + (threadIdx.x & ~31);
#pragma unroll 1
  for (long long i0 = first; i0 < N; i0 += stride) {  // warp-uniform loop
    const long long i = i0 + lane;
    const bool live = i < N;
    int s_lo = 1, s_hi = 0;  // empty range for lanes past the end
    float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
    float tj = 0.f;
    long long bj = 0;
    if (live) {
      const int4 tb = TBo[i];
      tj = __int_as_float(tb.x);
      bj = tb.y;
      slice_range(P, tj, &s_lo, &s_hi);
      e = XVo[i];
    }
    for (int s = 0; s < P.S; ++s) {
      int key = -1;
      if (s >= s_lo && s <= s_hi) key = source_fine_key(P, e.x, e.y, e.z, e.w, tj, bj, s);
      if (live) KEY[(long long)s * N + i] = key;
      const unsigned grp = __match_any_sync(0xffffffffu, key);
      if (key >= 0 && lane == __ffs(grp) - 1) atomicAdd(counts + key, __popc(grp));
    }
  }
}

// Entries of the ordered events: the count pass's keys, one cursor atomic per distinct cell of a warp, and
// the lanes of a cell writing consecutive slots.  One event per lane, its slices in an inner loop.  The
// cursors start at zero and the leader adds the cell's offset (cursors started at the offsets, so that an
// atomic returns the slot itself, measured 16 % slower: 167 against 144 us at configuration 2).
__global__ void __launch_bounds__(kThreads) k_fast_scatter_ordered(PlanConsts P, const float4* __restrict__ XVo,
                                                                   const int4* __restrict__ TBo, long long N,
                                                                   const int* __restrict__ KEY,
                                                                   const int* __restrict__ start,
                                                                   int* __restrict__ cursor, float4* __restrict__ YV,
                                                                   float2* __restrict__ TI) {
  const int lane = threadIdx.x & 31;
  const unsigned below = (1u << lane) - 1u;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = blockIdx.x * (long long)blockDim.x + (threadIdx.x & ~31);
#pragma unroll 1
  for (long long i0 = first; i0 < N; i0 += stride) {  // warp-uniform loop
    const long long i = i0 + lane;
    const bool live = i < N;
    float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
    float tj = 0.f;
    int id = 0;
    if (live) {
      const int4 tb = TBo[i];
      tj = __int_as_float(tb.x);
      id = tb.z;
      e = XVo[i];
    }
    // slices in batches of kSB: the batch's cursor atomics are issued back to back before any result is
    // used, so a warp waits for one round trip to L2 per batch rather than per slice
    constexpr int kSB = 8;
    for (int s0 = 0; s0 < P.S; s0 += kSB) {
      int key[kSB], base[kSB];
      unsigned grp[kSB];
#pragma unroll
      for (int u = 0; u < kSB; ++u)
        key[u] = live && s0 + u < P.S ? KEY[(long long)(s0 + u) * N + i] : -1;  // the count pass's keys
#pragma unroll
      for (int u = 0; u < kSB; ++u) {
        grp[u] = __match_any_sync(0xffffffffu, key[u]);
        base[u] = 0;
        if (key[u] >= 0 && lane == __ffs(grp[u]) - 1) base[u] = atomicAdd(cursor + key[u], __popc(grp[u]));
      }
#pragma unroll
      for (int u = 0; u < kSB; ++u) {
        const int leader = __ffs(grp[u]) - 1;
        int b = 0;
        if (key[u] >= 0 && lane == leader) b = start[key[u]] + base[u];
        b = __shfl_sync(0xffffffffu, b, leader);
        if (key[u] >= 0) {
          float yx, yy;
          transported(P, e.x, e.y, e.z, e.w, tj, s0 + u, &yx, &yy);
          const int p = b + __popc(grp[u] & below);
          YV[p] = make_float4(yx, yy, e.z, e.w);
          TI[p] = make_float2(tj, __int_as_float(id));
        }
      }
    }
  }
}

// Sub-cell key of an anchor (its plan cell as anchor_cell computes it, then the sub-cell inside), -1 if it has
// no cell.  *g, *fy, *fx: its plane and sub-cell; *cx, *cy: its plan cell.
__device__ __forceinline__ long long fast_anchor_key(const PlanConsts& P, float4 a, long long ba, int* g, int* fy,
                                                     int* fx, int* cx, int* cy) {
  if (__float_as_int(a.w) < 0 || ba < 0 || ba >= P.B) return -1;
  long long gg, qx, qy;
  anchor_cell(P, a.x, a.y, a.z, ba, &gg, &qx, &qy);
  *g = (int)gg;
  *cx = (int)qx;
  *cy = (int)qy;
  *fx = fine_index(a.x, P.ox_f, P.rfine_f, (int)qx);
  *fy = fine_index(a.y, P.oy_f, P.rfine_f, (int)qy);
  return (gg * P.GHf + *fy) * P.GWf + *fx;
}

__global__ void __launch_bounds__(kThreads) k_fast_anchor_count(PlanConsts P, const float4* __restrict__ anc4,
                                                                const long long* __restrict__ anc_b, long long M,
                                                                int* __restrict__ counts) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    int g, fy, fx, cx, cy;
    const long long key = fast_anchor_key(P, anc4[i], anc_b[i], &g, &fy, &fx, &cx, &cy);
    if (key >= 0) atomicAdd(counts + key, 1);
  }
}

// Anchor records in sub-cell order: XT = (x, y, t, the anchor's own pair value) and XK = (original index, plane,
// sub-cell row, sub-cell column).  The own pair (leave-one-out) is evaluated here once per anchor, with every
// lane busy, rather than in the pair kernel.
__global__ void __launch_bounds__(kThreads) k_fast_anchor_scatter(PlanConsts P, PairConsts C,
                                                                  const float4* __restrict__ anc4,
                                                                  const long long* __restrict__ anc_b, long long M,
                                                                  const float4* __restrict__ ev4,
                                                                  const float* __restrict__ SC,
                                                                  int* __restrict__ cursor, float4* __restrict__ XT,
                                                                  int4* __restrict__ XK) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const float4 a = anc4[i];
    const long long ba = anc_b[i];
    int g, fy, fx, cx, cy;
    const long long key = fast_anchor_key(P, a, ba, &g, &fy, &fx, &cx, &cy);
    if (key < 0) continue;
    const int p = atomicAdd(cursor + key, 1);  // the cursors start at the offsets
    const int s = (int)(g - ba * P.S);
    const float self = self_term(P, C, ev4, __float_as_int(a.w), a.x, a.y, a.z, sub_rn(a.z, SC[s]), (int)ba, s, cx, cy);
    XT[p] = make_float4(a.x, a.y, a.z, self);
    XK[p] = make_int4((int)i, g, fy, fx);
  }
}

// ---- per-anchor normaliser: den = W * vis * 2 pi h^2 (ats.py:92-96, functional.py:210-217) ----------
__device__ __forceinline__ double ev_key(const float* t, const long long* b, long long j) {
  return (double)b[j] * 4.0 + (double)t[j];
}

__device__ __forceinline__ long long key_search(const float* t, const long long* b, long long N, double q, bool right) {
  long long lo = 0, hi = N;
  while (lo < hi) {
    const long long m = (lo + hi) >> 1;
    const double k = ev_key(t, b, m);
    if (right ? (k <= q) : (k < q)) lo = m + 1; else hi = m;
  }
  return lo;
}

struct NormConsts {
  double tau;
  float tau_f, pi_f, h2_f, wmax, hmax;
  int n_check, visibility;
  long long B;  // rows of the slice histogram
};

// Exposure-check tables staged per CTA: the check-slice centres and the per-batch slice counts as floats.
constexpr int kNormMaxCheck = 64;
constexpr int kNormMaxCounts = 2048;

// visible_fraction_one with the centres and float counts read from tables: the same operations in the same
// order, without recomputing each centre (an IEEE division and the linspace formula) and converting each
// count per anchor.
__device__ __forceinline__ float visible_fraction_tab(float2 v, float xa, float ya, float ta, const float* cen,
                                                      const float* cnt_b, int n_check, float tau, float wmax,
                                                      float hmax) {
  float vis = 0.f, tot = 0.f;
#pragma unroll 16
  for (int k = 0; k < n_check; ++k) {
    const float c = cen[k];
    const float near = fabsf(sub_rn(ta, c)) <= tau ? 1.f : 0.f;
    const float dt = sub_rn(c, ta);
    const float yx = add_rn(xa, mul_rn(v.x, dt)), yy = add_rn(ya, mul_rn(v.y, dt));
    const float inside = (yx >= 0.f && yx <= wmax && yy >= 0.f && yy <= hmax) ? 1.f : 0.f;
    const float w = mul_rn(cnt_b[k], near);
    vis = add_rn(vis, mul_rn(w, inside));
    tot = add_rn(tot, w);
  }
  const float r = div_rn(vis, tot < 1.f ? 1.f : tot);
  return r < 1e-3f ? 1e-3f : r;
}

// bstart[k] = first event of batch k (events sorted by b, b in [0, B)), bstart[B] = N.
__global__ void __launch_bounds__(kThreads) k_batch_bounds(const long long* __restrict__ b, long long N, long long B,
                                                           long long* __restrict__ bstart) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j <= N; j += stride) {
    const long long lo = j == 0 ? 0 : b[j - 1] + 1, hi = j == N ? B : b[j];
    for (long long k = lo; k <= hi && k <= B; ++k) bstart[k] = j;
  }
}

// Normaliser den = Wn * vis * 2 pi h^2.  bstart != nullptr: tau exceeds the events' time span (with margin)
// and tau + span < 4, so the window of every anchor is its whole batch and the count is n_b - 1 (the
// reference's float64 key search gives the same, functional.py:210-217).
__global__ void __launch_bounds__(kThreads) k_exact_norm(MotionView Mv, NormConsts K, const float4* __restrict__ anc4,
                                                         const long long* __restrict__ anc_b, long long M,
                                                         const float* __restrict__ t, const long long* __restrict__ b,
                                                         long long N, const long long* __restrict__ bstart,
                                                         const int* __restrict__ counts, float* __restrict__ den) {
  __shared__ float cen[kNormMaxCheck];
  __shared__ float cntf[kNormMaxCounts];
  const int nc = K.n_check;
  const bool tab = K.visibility && nc <= kNormMaxCheck && K.B * nc <= kNormMaxCounts;  // CTA-uniform
  if (tab) {
    for (int k = threadIdx.x; k < nc; k += blockDim.x) cen[k] = check_centre(k, nc);
    for (int k = threadIdx.x; k < (int)(K.B * nc); k += blockDim.x) cntf[k] = (float)counts[k];
  }
  __syncthreads();
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const float4 a = anc4[i];
    const int ai = __float_as_int(a.w);
    const long long ba = anc_b[i];
    if (ai < 0 || ba < 0 || ba >= Mv.B || ba >= K.B) {
      den[i] = __int_as_float(0x7fc00000);
      continue;
    }
    long long c;
    if (bstart) {
      c = bstart[ba + 1] - bstart[ba] - 1;
    } else {
      const double ki = ev_key(t, b, ai);
      c = key_search(t, b, N, ki + K.tau, true) - key_search(t, b, N, ki - K.tau, false) - 1;
    }
    float wn = (float)(c > 0 ? c : 0);
    wn = wn < 1.f ? 1.f : wn;  // .clamp(min=1)
    if (tab)
      wn = mul_rn(wn, visible_fraction_tab(motion_field(Mv, a.x, a.y, ba), a.x, a.y, a.z, cen, cntf + ba * nc, nc,
                                           K.tau_f, K.wmax, K.hmax));
    else if (K.visibility)
      wn = mul_rn(wn, visible_fraction_one(Mv, a.x, a.y, a.z, ba, counts + ba * K.n_check, K.n_check, K.tau_f,
                                           K.wmax, K.hmax));
    den[i] = mul_rn(mul_rn(mul_rn(wn, 2.f), K.pi_f), K.h2_f);  // Wn * 2 * math.pi * h ** 2
  }
}


// The log score ls_i = log(eps + S_i / den_i) (ats.py:95), one thread per anchor after the pair sums: the
// division and the logarithm cost a full warp instruction stream per anchor group inside the pair kernel.
__global__ void __launch_bounds__(kThreads) k_exact_ls(const float* __restrict__ S, const float* __restrict__ den,
                                                       float eps, long long M, float* __restrict__ ls) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride)
    ls[i] = logf(add_rn(eps, div_rn(S[i], den[i])));  // log(eps + S / den)
}


// dL/dS in bucket order from the upstream dL/dls (torch's LogBackward then DivBackward).
// The backward's anchor records in bucket order: AB = (x, y, t, dL/dS / h^2), with
// dL/dS = dL/dls / (eps + S / den) / den (the Log then Div backward of ls = log(eps + S / den)).
__global__ void __launch_bounds__(kThreads) k_exact_gs_records(const float4* __restrict__ XT,
                                                               const int4* __restrict__ XK, long long M,
                                                               const float* __restrict__ grad_ls,
                                                               const float* __restrict__ S,
                                                               const float* __restrict__ den, float eps, float invh2,
                                                               float4* __restrict__ AB) {
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < M; p += stride) {
    const int i = XK[p].x;
    const float q = div_rn(S[i], den[i]);
    const float g = div_rn(div_rn(grad_ls[i], add_rn(eps, q)), den[i]);
    const float4 a = XT[p];
    AB[p] = make_float4(a.x, a.y, a.z, g * invh2);
  }
}

__global__ void __launch_bounds__(kThreads) k_slice_hist(const float* __restrict__ t, const long long* __restrict__ b,
                                                         long long N, long long B, int n_check,
                                                         int* __restrict__ counts) {
  __shared__ int hist[4096];
  const long long nbins = B * n_check;
  const bool sm = nbins <= 4096;
  if (sm)
    for (long long i = threadIdx.x; i < nbins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const long long bj = b[j];
    if (bj < 0 || bj >= B) continue;
    long long s = (long long)mul_rn(t[j], (float)n_check);
    s = s < 0 ? 0 : (s > n_check - 1 ? n_check - 1 : s);
    if (sm) atomicAdd(hist + bj * n_check + s, 1);
    else atomicAdd(counts + bj * n_check + s, 1);
  }
  __syncthreads();
  if (sm)
    for (long long i = threadIdx.x; i < nbins; i += blockDim.x)
      if (hist[i]) atomicAdd(counts + i, hist[i]);
}

// sc[s] = centre of slice s (S values), then scg[g] = centre of the slice of plane g = b S + s (B S values)
__global__ void k_slice_centres(PlanConsts P, float* sc, float* scg) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i < P.S) sc[i] = slice_centre(P, (int)i);
  if (i < P.B * P.S) scg[i] = slice_centre(P, (int)(i % P.S));
}

// velocity-field gradient at the dequantised positions stored in ev4 (x, y in the first two lanes)
__global__ void __launch_bounds__(kThreads) k_exact_vbwd_dense(MotionView Mv, const float2* __restrict__ gv,
                                                               const float4* __restrict__ ev4,
                                                               const long long* __restrict__ b, long long N,
                                                               float* __restrict__ ggrid) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long plane = Mv.Hg * Mv.Wg;
#pragma unroll 1
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < N; j += stride) {
    const float2 g = gv[j];
    if ((g.x == 0.f && g.y == 0.f) || b[j] < 0 || b[j] >= Mv.B) continue;
    const float4 e = ev4[j];
    DenseTaps T;
    dense_taps(Mv, e.x, e.y, &T);
    float* G = ggrid + b[j] * 2 * plane;
    // per channel and tap row, the taps (x0, x1) are adjacent floats: one red.v2 when they form an 8-byte
    // aligned pair, else one red per non-zero tap
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const float gc = c ? g.y : g.x;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float* row = G + c * plane + (r ? T.y1 : T.y0) * Mv.Wg;
        const float w0 = T.w[2 * r], w1 = T.w[2 * r + 1];
        if (T.x1 == T.x0 + 1 && ((reinterpret_cast<uintptr_t>(row + T.x0) & 7) == 0)) {
          red_add_f2(row + T.x0, gc * w0, gc * w1);
        } else {
          if (w0 != 0.f) red_add_f1(row + T.x0, gc * w0);
          if (w1 != 0.f) red_add_f1(row + T.x1, gc * w1);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) k_exact_vbwd_param(MotionView Mv, const float2* __restrict__ gv,
                                                               const float4* __restrict__ ev4,
                                                               const long long* __restrict__ b, long long N,
                                                               float* __restrict__ gtheta) {
  // per-warp partial sums for batch 0..B-1 are rare to mix: accumulate per event with atomics on the
  // (B, 2|6) parameters after a warp reduction over runs of equal batch index
  const int np = Mv.kind == ATLB_MOTION_TRANSLATION ? 2 : 6;
  const long long stride = (long long)gridDim.x * blockDim.x;
#pragma unroll 1
  for (long long j0 = blockIdx.x * (long long)blockDim.x; j0 < N; j0 += stride) {
    const long long j = j0 + threadIdx.x;
    float c[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    long long bj = -1;
    if (j < N) {
      bj = b[j];
      const float2 g = gv[j];
      const float4 e = ev4[j];
      const float d0 = sub_rn(e.x, Mv.cx), d1 = sub_rn(e.y, Mv.cy);
      c[0] = g.x; c[1] = g.y; c[2] = g.x * d0; c[3] = g.x * d1; c[4] = g.y * d0; c[5] = g.y * d1;
      if (bj < 0 || bj >= Mv.B) bj = -1;
    }
    const long long b0 = __shfl_sync(0xffffffffu, bj, 0);
    const bool uniform = __all_sync(0xffffffffu, bj == b0);
    if (uniform) {
      for (int q = 0; q < np; ++q) c[q] = warp_sum(c[q]);
      if ((threadIdx.x & 31) == 0 && b0 >= 0)
        for (int q = 0; q < np; ++q) atomicAdd(gtheta + b0 * np + q, c[q]);
    } else if (bj >= 0) {
      for (int q = 0; q < np; ++q) atomicAdd(gtheta + bj * np + q, c[q]);
    }
  }
}

struct ExactWs {
  int* counts;
  int* start;
  long long* partials;
  float4* YV;
  float2* TI;
  int* acounts;
  int* astart;
  long long* apartials;  // scan scratch of the anchor buckets (their scan runs on the second stream)
  float4* XT;
  int4* XK;      // (original index, plane, sub-cell row, sub-cell column) of the bucketed anchors
  int* slice_hist;
  float* SC;
  float* SCg;    // slice centre of every plane (B S)
  long long* bstart;  // first event of each batch (B + 1)
  int* KEY;      // cell key of each (slice, source event) of the count pass, -1 = no entry
  float4* AB;    // backward anchor records (x, y, t, dL/dS / h^2), bucket order
  int* ocount;   // events per mid-slice cell (B*GH*GW), then the order cursor
  int* ostart;
  float4* XVo;   // events in spatial order: (x, y, vx, vy)
  int4* TBo;     // (t bits, b, original index, 0)
  int* scratch;
};

size_t ws_layout(long long N, long long M, long long ncell, long long S, long long B, long long n_check,
                 long long nkey, ExactWs* w, void* base) {
  const long long nent = N * S;
  size_t off = 0;
  char* p = (char*)align_ptr(base ? base : (void*)256);
  auto take = [&](size_t bytes) {
    char* q = p + off;
    off += align_up(bytes);
    return (void*)q;
  };
  ExactWs x;
  x.counts = (int*)take((size_t)ncell * 4);
  x.start = (int*)take((size_t)(ncell + 1) * 4);
  x.partials = (long long*)take(scan_partials_bytes(ncell));
  x.YV = (float4*)take((size_t)(nent + kFwdPad) * 16);  // padding: read, never used, by k_pair_fwd_fine
  x.TI = (float2*)take((size_t)(nent + kFwdPad) * 8);
  x.acounts = (int*)take((size_t)ncell * 4);
  x.astart = (int*)take((size_t)(ncell + 1) * 4);
  x.apartials = (long long*)take(scan_partials_bytes(ncell));
  x.XT = (float4*)take((size_t)M * 16);
  x.XK = (int4*)take((size_t)M * 16);
  x.slice_hist = (int*)take((size_t)(B * n_check) * 4);
  x.SC = (float*)take((size_t)S * 4);
  x.SCg = (float*)take((size_t)(B * S) * 4);
  x.bstart = (long long*)take((size_t)(B + 1) * 8);
  x.KEY = (int*)take((size_t)nent * 4);
  x.AB = (float4*)take((size_t)M * 16);
  x.ocount = (int*)take((size_t)nkey * 4);
  x.ostart = (int*)take((size_t)(nkey + 1) * 4);
  x.XVo = (float4*)take((size_t)N * 16);
  x.TBo = (int4*)take((size_t)N * 16);
  x.scratch = (int*)take(64);
  if (w) *w = x;
  return off + 256;
}

int warp_grid(long long nwarps) { return clamp_grid(blocks_for(nwarps * 32, kThreads)); }


// A second stream of the calling host thread on the current device, with the events that fork work onto it
// from the caller's stream and join it back (null if it cannot be created: the caller's stream is used).
// Per thread, so that concurrent callers never record into each other's events.  Under stream capture the
// fork / join pair brings the second stream into the caller's graph.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
SideStream* side_stream() {
  thread_local SideStream per_dev[64];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  SideStream& x = per_dev[dev];
  if (!x.s) {
    cudaStream_t st = nullptr;
    cudaEvent_t f = nullptr, j = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&f, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&j, cudaEventDisableTiming) != cudaSuccess) {
      if (j) cudaEventDestroy(j);
      if (f) cudaEventDestroy(f);
      if (st) cudaStreamDestroy(st);
      cudaGetLastError();  // not sticky: clear it, the caller's stream does the work instead
      return nullptr;
    }
    x.s = st;
    x.fork = f;
    x.join = j;
  }
  return &x;
}

// Every pair passes |t_i - t_j| <= tau when tau covers the events' time range: fl(t_i - t_j) never exceeds
// fl(t_hi - t_lo) (rounding is monotonic).  NaN bounds (unknown range) fail the test.
// The events that are sources of the pair sums: [src_begin, src_end) of the configuration, all if src_end <= 0.
void src_range(const atlb_exact_cfg& c, long long N, long long* j0, long long* j1) {
  *j0 = c.src_end > 0 ? c.src_begin : 0;
  *j1 = c.src_end > 0 ? c.src_end : N;
}

bool tau_covers(const atlb_plan_geom& g, double tau) {
  const float span = g.t_hi - g.t_lo;
  return span <= (float)tau;
}

}  // namespace

// Sub-cells of the fused plan: every plan cell split kFine x kFine.
static long long fine_cells(const atlb_exact_cfg& c, const atlb_plan_geom& g) {
  return c.B * (long long)g.S * (g.GH * kFine) * (g.GW * kFine);
}

// Window constants of the pair kernels (pair_fine.cuh).  The margin covers the rounding of the positions, of
// the sub-cell bounds and of the window arithmetic: 0.01 px plus 16 ulp of the largest coordinate of the grid.
static FineConsts fine_consts(const atlb_exact_cfg& c, const atlb_plan_geom& g, const PlanConsts& P) {
  FineConsts F;
  F.ox = P.ox_f;
  F.oy = P.oy_f;
  F.f = (float)(g.cell / kFine);
  F.rf = P.rfine_f;
  const double r2 = (double)make_pair_consts(c.h, c.tau, c.cut).r2max;
  F.rcut = (float)(std::sqrt(r2) * (1.0 + 1e-6));
  F.vmax = (float)((double)g.vmax * (1.0 + 1e-6));
  const double maxc = std::max(std::max(std::fabs(g.ox), std::fabs(g.oy)),
                               std::max(std::fabs(g.ox + g.GW * g.cell), std::fabs(g.oy + g.GH * g.cell)));
  F.margin = (float)(0.01 + 16.0 * maxc * std::ldexp(1.0, -23));
  // max |t_a - c_s| over anchors (events): half a slice inside [0, 1], more for times outside it
  const double delta = 1.0 / (double)g.S;
  double dtmax = delta / 2;
  if (g.t_lo == g.t_lo) dtmax = std::max(dtmax, delta / 2 - (double)g.t_lo);
  if (g.t_hi == g.t_hi) dtmax = std::max(dtmax, (double)g.t_hi - (1.0 - delta / 2));
  F.rho_max = (float)(((double)F.rcut + (double)F.vmax * dtmax * (1.0 + 1e-6) + F.margin) * (1.0 + 1e-6));
  F.GWf = (int)(g.GW * kFine);
  F.GHf = (int)(g.GH * kFine);
  const bool finite_t = g.t_lo == g.t_lo && g.t_hi == g.t_hi;
  F.clip = (std::isfinite(F.rho_max) && finite_t) ? 1 : 0;
  return F;
}

size_t exact_workspace_bytes(const atlb_exact_cfg& c, long long N, long long M, const atlb_plan_geom& g) {
  const long long ncell = fine_cells(c, g);
  long long j0, j1;
  src_range(c, N, &j0, &j1);
  return ws_layout(j1 - j0, M, ncell, g.S, c.B, c.n_check, c.B * g.GH * g.GW * kFine * kFine, nullptr, nullptr);
}

static MotionView motion_of(const atlb_exact_cfg& c) {
  return make_motion_view(c.kind, c.theta, c.Bt, c.Hg, c.Wg, c.H, c.W);
}

// The prepare's read-back buffer: 64 bytes of pinned host memory per host thread, allocated on the thread's first
// call and kept for the thread (null if pinned memory cannot be had: the caller then copies into its stack).  A
// copy into pageable memory is staged by the driver and handed to the stream only once the stream reaches it;
// into pinned memory it is an ordinary stream operation queued right behind the prepare kernels.
static int* pinned_readback() {
  thread_local struct Holder {
    int* p = nullptr;
    bool tried = false;
    ~Holder() {
      if (p) cudaFreeHost(p);  // at thread exit; an error during process teardown is of no consequence
    }
  } h;
  if (!h.tried) {
    h.tried = true;
    if (cudaHostAlloc((void**)&h.p, 64, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();  // not sticky: clear it, the stack buffer is used instead
      h.p = nullptr;
    }
  }
  return h.p;
}

int exact_prepare(const atlb_exact_cfg& c, const float* xy, const float* u, const float* t, const long long* b,
                  long long N, const long long* anchors, const float* z, long long M, float* ev4, float* anc4,
                  long long* anc_b, void* scratch, atlb_plan_geom* geom, cudaStream_t s) {
  int* r = (int*)scratch;
  launch(k_exact_init, 1, 32, 0, s, r);
  const MotionView Mv = motion_of(c);
  const bool rng_u = (c.rng & 1) != 0, rng_z = (c.rng & 2) != 0;
  const RngKey K = make_rng_key(c.rng_seed, c.rng_call);
  if (N > 0)
    launch(rng_u ? k_exact_events<true> : k_exact_events<false>, grid_for(N), kThreads, 0, s, Mv, (const float2*)xy,
           (const float2*)u, t, b, N, c.B, K, (float4*)ev4, r);
  if (M > 0)
    launch(rng_z ? k_exact_anchors<true> : k_exact_anchors<false>, grid_for(M), kThreads, 0, s, (const float4*)ev4, t,
           b, N, anchors, (const float2*)z, K, (float)c.h, M, (float4*)anc4, anc_b, r);
  int stack_host[10];
  int* pinned = pinned_readback();
  int* host = pinned ? pinned : stack_host;
  if (cudaMemcpyAsync(host, r, sizeof(stack_host), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return launch_status("exact_prepare copy");
  if (cudaStreamSynchronize(s) != cudaSuccess) return launch_status("exact_prepare sync");
  if (int st = launch_status("exact_prepare")) return st;
  if (host[5]) { set_error("exact_prepare: an anchor index lies outside [0, %lld)", N); return ATLB_ERR_ARG; }
  if (host[7]) { set_error("exact_prepare: a batch index lies outside [0, %lld)", (long long)c.B); return ATLB_ERR_ARG; }
  if (host[6]) { set_error("exact_prepare: events are not sorted by (b, t)"); return ATLB_ERR_UNSORTED; }
  float vmax;
  memcpy(&vmax, &host[0], 4);
  plan_geometry_host(N > 0 ? vmax : 0.f, M > 0, ordered_to_float(host[1]), ordered_to_float(host[2]),
                     ordered_to_float(host[3]), ordered_to_float(host[4]), c.H, c.W, c.h, c.cut, c.S, geom);
  if (N > 0) {
    geom->t_lo = ordered_to_float(host[8]);
    geom->t_hi = ordered_to_float(host[9]);
  }
  return ATLB_OK;
}

int exact_forward(const atlb_exact_cfg& c, const float* t, const long long* b, long long N, long long M,
                  const float* ev4, const float* anc4, const long long* anc_b, const atlb_plan_geom& g, void* ws,
                  float* S_out, float* den_out, float* ls_out, cudaStream_t s) {
  const long long ncell = fine_cells(c, g);
  long long j0, j1;
  src_range(c, N, &j0, &j1);
  const long long ns = j1 - j0;  // source events of this call
  ExactWs w;
  ws_layout(ns, M, ncell, g.S, c.B, c.n_check, c.B * g.GH * g.GW * kFine * kFine, &w, ws);
  PlanConsts P = make_plan_consts(g, c.tau, c.B);
  P.src0 = j0;
  P.src1 = j1;
  // slice centres: read by the anchor records and the pair kernels
  launch(k_slice_centres, (unsigned)((c.B * g.S + 127) / 128), 128, 0, s, P, w.SC, w.SCg);
  // the normaliser (window counts, exposure correction) and the anchor buckets depend on the prepared events
  // and anchors only, so they run on a second stream beside the entry plan build below
  SideStream* side = side_stream();
  const cudaStream_t norm_s = side ? side->s : s;
  if (side) {
    cudaEventRecord(side->fork, s);
    cudaStreamWaitEvent(side->s, side->fork, 0);
  }
  const MotionView Mv = motion_of(c);
  NormConsts K;
  K.tau = c.tau;
  K.tau_f = (float)c.tau;
  K.pi_f = (float)M_PI;
  K.h2_f = (float)(c.h * c.h);
  K.wmax = (float)(c.W - 1);
  K.hmax = (float)(c.H - 1);
  K.n_check = (int)c.n_check;
  K.visibility = c.visibility;
  K.B = c.B;
  cudaMemsetAsync(w.slice_hist, 0, (size_t)(c.B * c.n_check) * 4, norm_s);
  if (c.visibility && N > 0)
    launch(k_slice_hist, clamp_grid(blocks_for(N, kThreads * 16)), kThreads, 0, norm_s, t, b, N, c.B, (int)c.n_check,
           w.slice_hist);
  // Window counts are batch size - 1 when every event of a batch lies within tau of every other and no other
  // batch does: span <= tau (then key_i - tau <= key_j <= key_i + tau holds for the float64 keys b*4 + t of one
  // batch, which are exact, after the monotone rounding of key_i +- tau) and tau + span < 4 with a margin
  // (keys of the neighbouring batch stay outside).  span is exact: two floats subtracted in double.  NaN
  // (unknown range) fails both tests.
  const double span = (double)g.t_hi - (double)g.t_lo;
  const bool whole_batch = c.tau >= span && c.tau + span < 4.0 - 1e-6;
  if (whole_batch) launch(k_batch_bounds, grid_for(N + 1), kThreads, 0, norm_s, b, N, c.B, w.bstart);
  if (M > 0)
    launch(k_exact_norm, grid_for(M), kThreads, 0, norm_s, Mv, K, (const float4*)anc4, anc_b, M, t, b, N,
           whole_batch ? (const long long*)w.bstart : nullptr, (const int*)w.slice_hist, den_out);
  // anchors into sub-cells, each with its own pair value (second stream)
  cudaMemsetAsync(w.acounts, 0, (size_t)ncell * 4, norm_s);
  if (M > 0)
    launch(k_fast_anchor_count, grid_for(M), kThreads, 0, norm_s, P, (const float4*)anc4, anc_b, M, w.acounts);
  exclusive_scan<int>(w.acounts, ncell, w.apartials, w.astart, norm_s, /*cursors=*/true);
  if (M > 0)
    launch(k_fast_anchor_scatter, grid_for(M), kThreads, 0, norm_s, P, make_pair_consts(c.h, c.tau, c.cut),
           (const float4*)anc4, anc_b, M, (const float4*)ev4, (const float*)w.SC, w.acounts, w.XT, w.XK);
  // entries
  cudaMemsetAsync(w.counts, 0, (size_t)ncell * 4, s);
  if (ns > 0) {  // source events in mid-slice cell order (see k_order_count)
    const long long nkey = c.B * g.GH * g.GW * kFine * kFine;  // mid-slice sub-cells
    const float4* ev = (const float4*)ev4 + j0;
    cudaMemsetAsync(w.ocount, 0, (size_t)nkey * 4, s);
    launch(k_order_count, grid_for(ns), kThreads, 0, s, P, ev, t + j0, b + j0, ns, w.ocount);
    exclusive_scan<int>(w.ocount, nkey, w.partials, w.ostart, s, /*cursors=*/true);
    launch(k_order_scatter, grid_for(ns), kThreads, 0, s, P, ev, t + j0, b + j0, ns, j0, w.ocount, w.XVo, w.TBo);
    launch(k_fast_count_ordered, grid_for(ns), kThreads, 0, s, P, (const float4*)w.XVo, (const int4*)w.TBo,
           ns, w.counts, w.KEY);
  }
  exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);  // relative cursors: measured faster here
  if (ns > 0)
    launch(k_fast_scatter_ordered, grid_for(ns), kThreads, 0, s, P, (const float4*)w.XVo, (const int4*)w.TBo,
           ns, (const int*)w.KEY, (const int*)w.start, w.counts, w.YV, w.TI);
  if (side) {  // the pair kernels below read den and the anchor buckets
    cudaEventRecord(side->join, norm_s);
    cudaStreamWaitEvent(s, side->join, 0);
  }
  // pair sums + log scores
  const FastEntries E{w.YV, w.TI};
  const PairConsts C = make_pair_consts(c.h, c.tau, c.cut);
  const float eps = (float)(c.eps_frac / (double)(c.H * c.W));
  if (M > 0 && ncell > 0) {
    const FineConsts F = fine_consts(c, g, P);
    const dim3 grid((unsigned)((F.GWf + kFwdTileX - 1) / kFwdTileX), (unsigned)((F.GHf + kFwdTileY - 1) / kFwdTileY),
                    (unsigned)(c.B * g.S));
    cudaEvent_t e0 = timing_begin(s);
    const int n_ent = (int)(ns * (long long)g.S);  // an upper bound of the entries; only read through cstart
    if (ns == 0)  // no sources, no pairs: every sum is 0 (and so is every own pair value)
      cudaMemsetAsync(S_out, 0, (size_t)M * sizeof(float), s);
    else if (tau_covers(g, c.tau))
      launch(k_pair_fwd_fine<true>, grid, kFwdWarps * 32, 0, s, E, (const float4*)w.XT, (const int4*)w.XK,
             (const int*)w.astart, (const int*)w.start, F, (const float*)w.SCg, C, n_ent, S_out);
    else
      launch(k_pair_fwd_fine<false>, grid, kFwdWarps * 32, 0, s, E, (const float4*)w.XT, (const int4*)w.XK,
             (const int*)w.astart, (const int*)w.start, F, (const float*)w.SCg, C, n_ent, S_out);
    timing_end("k_pair_fwd", s, e0);
    launch(k_exact_ls, grid_for(M), kThreads, 0, s, (const float*)S_out, (const float*)den_out, eps, M, ls_out);
  }
  return launch_status("exact_forward");
}

int exact_backward(const atlb_exact_cfg& c, const float* grad_ls, const long long* b, long long N, long long M,
                   const float* ev4, const atlb_plan_geom& g, void* ws, const float* S, const float* den, float* gv,
                   float* gtheta, cudaStream_t s) {
  const long long ncell = fine_cells(c, g);
  long long j0, j1;
  src_range(c, N, &j0, &j1);
  const long long ns = j1 - j0;
  ExactWs w;
  ws_layout(ns, M, ncell, g.S, c.B, c.n_check, c.B * g.GH * g.GW * kFine * kFine, &w, ws);
  const float eps = (float)(c.eps_frac / (double)(c.H * c.W));
  cudaMemsetAsync(gv, 0, (size_t)N * 2 * sizeof(float), s);
  const FastEntries E{w.YV, w.TI};
  const PairConsts C = make_pair_consts(c.h, c.tau, c.cut);
  if (M > 0 && ncell > 0) {
    const PlanConsts P = make_plan_consts(g, c.tau, c.B);
    launch(k_exact_gs_records, grid_for(M), kThreads, 0, s, (const float4*)w.XT, (const int4*)w.XK, M, grad_ls, S,
           den, eps, C.invh2, w.AB);
    const FineConsts F = fine_consts(c, g, P);
    const int nrows = (int)(c.B * g.S * g.GH);  // plan cell rows of all planes
    const dim3 grid((unsigned)((g.GW + kBwdWarps - 1) / kBwdWarps), (unsigned)min(nrows, 65535));
    cudaEvent_t e0 = timing_begin(s);
    if (tau_covers(g, c.tau))
      launch(k_pair_bwd_fine<true>, grid, kBwdWarps * 32, 0, s, E, (const float4*)w.AB, (const float*)w.SCg,
             (const int*)w.astart, (const int*)w.start, F, (int)g.GW, nrows, C, N, gv);
    else
      launch(k_pair_bwd_fine<false>, grid, kBwdWarps * 32, 0, s, E, (const float4*)w.AB, (const float*)w.SCg,
             (const int*)w.astart, (const int*)w.start, F, (int)g.GW, nrows, C, N, gv);
    timing_end("k_pair_bwd", s, e0);
  }
  const MotionView Mv = motion_of(c);
  const size_t nth = c.kind == ATLB_MOTION_DENSE ? (size_t)(c.Bt * 2 * c.Hg * c.Wg)
                                                 : (size_t)(c.Bt * (c.kind == ATLB_MOTION_TRANSLATION ? 2 : 6));
  cudaMemsetAsync(gtheta, 0, nth * sizeof(float), s);
  if (ns > 0) {  // the motion gradient of this call's source events
    const float2* g2 = (const float2*)gv + j0;
    const float4* e4 = (const float4*)ev4 + j0;
    if (c.kind == ATLB_MOTION_DENSE)
      launch(k_exact_vbwd_dense, grid_for(ns), kThreads, 0, s, Mv, g2, e4, b + j0, ns, gtheta);
    else
      launch(k_exact_vbwd_param, grid_for(ns), kThreads, 0, s, Mv, g2, e4, b + j0, ns, gtheta);
  }
  return launch_status("exact_backward");
}

}  // namespace atlb
