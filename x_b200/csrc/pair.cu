// Anchored pair sums over the reference plan layout: the B200 replacement of ats_pair_fwd /
// ats_pair_bwd (csrc/atl_cpu.cpp:176-253).
//
// Reference: one thread per anchor walks its 3x3 cells; the backward scatters 2 global float
// atomics per pair.  Here:
//   * anchors are first bucketed by cell (counting sort, same key as the sources), so one WARP owns
//     one anchor cell: its anchors sit in registers and the 32 lanes stream the candidate sources of
//     the 3 neighbouring cell rows (each row is one contiguous CSR range), coalesced;
//   * the backward is source-centric over the same bucketing: one warp owns one source cell, each
//     lane one source, and the anchors of the 3x3 neighbourhood are broadcast -- the gradient of a
//     source entry is summed in registers and leaves with ONE vector red.global per entry instead of
//     two atomics per pair.
// The pair test (|dt| <= tau, d^2 <= (cut h)^2, leave-one-out by id) is evaluated with the exact
// rounding sequence of the reference, so the set of contributing pairs is identical.
#include "common.cuh"
#include "pair_math.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;
constexpr int kAnchorChunk = 8;

struct PlanView {
  const float2* SY;
  const float2* SV;
  const float* ST;
  const long long* SID;
  const long long* CS;
  long long S, GH, GW, ncell;
};

// Anchors bucketed by cell: sorted copies of what the kernels read.
struct AnchorBuckets {
  const int* start;    // [ncell + 1]
  const float2* xy;    // [M]
  const float* t;      // [M]
  const long long* id; // [M]
  const int* idx;      // [M] original anchor index
};

__device__ __forceinline__ long long anchor_key(const long long* AC, long long i, long long S, long long GH,
                                                long long GW, long long ncell) {
  const long long g = AC[3 * i], cx = AC[3 * i + 1], cy = AC[3 * i + 2];
  if (g < 0 || cx < 0 || cx >= GW || cy < 0 || cy >= GH) return -1;
  const long long key = (g * GH + cy) * GW + cx;
  return key < ncell ? key : -1;
}

__global__ void __launch_bounds__(kThreads) k_anchor_count(const long long* __restrict__ AC, long long M, long long S,
                                                           long long GH, long long GW, long long ncell,
                                                           int* __restrict__ counts) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const long long key = anchor_key(AC, i, S, GH, GW, ncell);
    if (key >= 0) atomicAdd(counts + key, 1);
  }
}

__global__ void __launch_bounds__(kThreads) k_anchor_scatter(const long long* __restrict__ AC,
                                                             const float2* __restrict__ AX,
                                                             const float* __restrict__ AT,
                                                             const long long* __restrict__ AID, long long M,
                                                             long long S, long long GH, long long GW, long long ncell,
                                                             const int* __restrict__ start, int* __restrict__ cursor,
                                                             float2* __restrict__ bxy, float* __restrict__ bt,
                                                             long long* __restrict__ bid, int* __restrict__ bidx,
                                                             float* __restrict__ out_invalid) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const long long key = anchor_key(AC, i, S, GH, GW, ncell);
    if (key < 0) {
      // a cell outside the grid: the reference would read out of bounds; flag the anchor with NaN
      if (out_invalid) out_invalid[i] = __int_as_float(0x7fc00000);
      continue;
    }
    const int p = start[key] + atomicAdd(cursor + key, 1);
    bxy[p] = AX[i];
    bt[p] = AT[i];
    bid[p] = AID[i];
    bidx[p] = (int)i;
  }
}

// One warp per anchor cell.  Lanes stride over the candidate sources of the 3 neighbouring cell rows.
__global__ void __launch_bounds__(kThreads) k_pair_fwd(PlanView P, AnchorBuckets A, const float* __restrict__ SC,
                                                       PairConsts C, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long c = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; c < P.ncell; c += nwarps) {
    const int a0 = A.start[c], a1 = A.start[c + 1];
    if (a0 == a1) continue;
    const long long cx = c % P.GW, cy = (c / P.GW) % P.GH, g = c / (P.GW * P.GH);
    const float cs = SC[g % P.S];
    const long long xlo = cx > 0 ? cx - 1 : 0, xhi = cx + 1 < P.GW ? cx + 1 : P.GW - 1;
    for (int base = a0; base < a1; base += kAnchorChunk) {
      const int na = min(kAnchorChunk, a1 - base);
      float ax[kAnchorChunk], ay[kAnchorChunk], at[kAnchorChunk], adt[kAnchorChunk], acc[kAnchorChunk];
      long long aid[kAnchorChunk];
#pragma unroll
      for (int q = 0; q < kAnchorChunk; ++q) {
        const int p = base + (q < na ? q : 0);
        const float2 xy = A.xy[p];
        ax[q] = xy.x; ay[q] = xy.y; at[q] = A.t[p]; aid[q] = q < na ? A.id[p] : -1;
        adt[q] = sub_rn(at[q], cs);
        acc[q] = 0.f;
      }
      for (long long yy = cy > 0 ? cy - 1 : 0; yy <= cy + 1 && yy < P.GH; ++yy) {
        const long long row = (g * P.GH + yy) * P.GW;
        const long long k0 = P.CS[row + xlo], k1 = P.CS[row + xhi + 1];
        for (long long k = k0 + lane; k < k1; k += 32) {
          const float2 sy = P.SY[k], sv = P.SV[k];
          const float st = P.ST[k];
          const long long sid = P.SID[k];
#pragma unroll
          for (int q = 0; q < kAnchorChunk; ++q) {
            float rx, ry, d2, dt;
            if (q < na && sid != aid[q] && pair_test(C, ax[q], ay[q], at[q], adt[q], sy, sv, st, &rx, &ry, &d2, &dt))
              acc[q] += pair_kernel(C, d2);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < kAnchorChunk; ++q) {
        if (q < na) {
          const double s = warp_sum((double)acc[q]);
          if (lane == 0) out[A.idx[base + q]] = (float)s;
        }
      }
    }
  }
}

// One warp per source cell.  Lane = one source entry; the anchors of the 3x3 neighbourhood are
// broadcast.  Gradient of sum_i gS_i S_i w.r.t. v_j (csrc/atl_cpu.cpp:241-250).
__global__ void __launch_bounds__(kThreads) k_pair_bwd(PlanView P, AnchorBuckets A, const float* __restrict__ SC,
                                                       const float* __restrict__ gS, PairConsts C,
                                                       long long N, float* __restrict__ gv) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long c = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; c < P.ncell; c += nwarps) {
    const long long k0 = P.CS[c], k1 = P.CS[c + 1];
    if (k0 == k1) continue;
    const long long cx = c % P.GW, cy = (c / P.GW) % P.GH, g = c / (P.GW * P.GH);
    const float cs = SC[g % P.S];
    const long long xlo = cx > 0 ? cx - 1 : 0, xhi = cx + 1 < P.GW ? cx + 1 : P.GW - 1;
    for (long long kb = k0; kb < k1; kb += 32) {
      const long long k = kb + lane;
      const bool valid = k < k1;
      const long long kk = valid ? k : k0;
      const float2 sy = P.SY[kk], sv = P.SV[kk];
      const float st = P.ST[kk];
      const long long sid = P.SID[kk];
      float gx = 0.f, gy = 0.f;
      for (long long yy = cy > 0 ? cy - 1 : 0; yy <= cy + 1 && yy < P.GH; ++yy) {
        const long long row = (g * P.GH + yy) * P.GW;
        const int p0 = A.start[row + xlo], p1 = A.start[row + xhi + 1];
        for (int p = p0; p < p1; ++p) {
          const float gi = gS[A.idx[p]];
          if (gi == 0.f) continue;
          const float2 xy = A.xy[p];
          const float at = A.t[p];
          const float adt = sub_rn(at, cs);
          float rx, ry, d2, dt;
          if (sid != A.id[p] && pair_test(C, xy.x, xy.y, at, adt, sy, sv, st, &rx, &ry, &d2, &dt)) {
            const float f = pair_grad_factor(C, gi, pair_kernel(C, d2), dt);
            gx += mul_rn(f, rx);
            gy += mul_rn(f, ry);
          }
        }
      }
      if (valid && (gx != 0.f || gy != 0.f) && sid >= 0 && sid < N) red_add_f2(gv + 2 * sid, gx, gy);
    }
  }
}

}  // namespace

size_t pair_workspace_bytes(long long M, long long ncell) {
  size_t n = 0;
  n += align_up((size_t)ncell * sizeof(int));              // counts / cursor
  n += align_up((size_t)(ncell + 1) * sizeof(int));        // start
  n += align_up(scan_partials_bytes(ncell));               // scan partials
  n += align_up((size_t)M * sizeof(float2));               // xy
  n += align_up((size_t)M * sizeof(float));                // t
  n += align_up((size_t)M * sizeof(long long));            // id
  n += align_up((size_t)M * sizeof(int));                  // idx
  return n + 256;
}

namespace {
struct PairWs {
  int* counts;
  int* start;
  long long* partials;
  float2* xy;
  float* t;
  long long* id;
  int* idx;
};
PairWs carve(void* ws, long long M, long long ncell) {
  char* p = (char*)align_ptr(ws);
  PairWs w;
  w.counts = (int*)p; p += align_up((size_t)ncell * sizeof(int));
  w.start = (int*)p; p += align_up((size_t)(ncell + 1) * sizeof(int));
  w.partials = (long long*)p; p += align_up(scan_partials_bytes(ncell));
  w.xy = (float2*)p; p += align_up((size_t)M * sizeof(float2));
  w.t = (float*)p; p += align_up((size_t)M * sizeof(float));
  w.id = (long long*)p; p += align_up((size_t)M * sizeof(long long));
  w.idx = (int*)p;
  return w;
}

AnchorBuckets bucket_anchors(const PairWs& w, const long long* AC, const float* AX, const float* AT,
                             const long long* AID, long long M, long long S, long long GH, long long GW,
                             long long ncell, float* out_invalid, cudaStream_t s) {
  cudaMemsetAsync(w.counts, 0, (size_t)ncell * sizeof(int), s);
  if (M > 0)
    launch(k_anchor_count, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, M, S, GH, GW, ncell, w.counts);
  exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);
  if (M > 0)
    launch(k_anchor_scatter, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, 
        AC, (const float2*)AX, AT, AID, M, S, GH, GW, ncell, w.start, w.counts, w.xy, w.t, w.id, w.idx, out_invalid);
  AnchorBuckets A;
  A.start = w.start; A.xy = w.xy; A.t = w.t; A.id = w.id; A.idx = w.idx;
  return A;
}

int warp_grid(long long nwarps) { return clamp_grid(blocks_for(nwarps * 32, kThreads)); }
}  // namespace

int pair_fwd(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
             const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC, long long M,
             long long ncell, long long S, long long GH, long long GW, double h, double tau, double cut, float* out,
             void* ws, cudaStream_t s) {
  const PairWs w = carve(ws, M, ncell);
  const AnchorBuckets A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, out, s);
  const PlanView P{(const float2*)SY, (const float2*)SV, ST, SID, CS, S, GH, GW, ncell};
  const PairConsts C = make_pair_consts(h, tau, cut);
  if (M > 0 && ncell > 0) {
    cudaEvent_t e0 = timing_begin(s);
    launch(k_pair_fwd, warp_grid(ncell), kThreads, 0, s, P, A, SC, C, out);
    timing_end("k_pair_fwd", s, e0);
  }
  return launch_status("ats_pair_fwd");
}

int pair_bwd(const float* gS, const float* SY, const float* SV, const float* ST, const long long* SID,
             const long long* CS, const float* AX, const float* AT, const long long* AC, const long long* AID,
             const float* SC, long long M, long long ncell, long long S, long long GH, long long GW, double h,
             double tau, double cut, long long N, float* gv, void* ws, cudaStream_t s) {
  const PairWs w = carve(ws, M, ncell);
  cudaMemsetAsync(gv, 0, (size_t)N * 2 * sizeof(float), s);
  const AnchorBuckets A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, nullptr, s);
  const PlanView P{(const float2*)SY, (const float2*)SV, ST, SID, CS, S, GH, GW, ncell};
  const PairConsts C = make_pair_consts(h, tau, cut);
  if (M > 0 && ncell > 0) {
    cudaEvent_t e0 = timing_begin(s);
    launch(k_pair_bwd, warp_grid(ncell), kThreads, 0, s, P, A, SC, gS, C, N, gv);
    timing_end("k_pair_bwd", s, e0);
  }
  return launch_status("ats_pair_bwd");
}

}  // namespace atlb
