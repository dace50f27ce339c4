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
#include <mutex>

#include "common.cuh"
#include "pair_kernels.cuh"
#include "pair_math.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;
constexpr int kAnchorChunk = 8;

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

struct RefOut {
  float* out;
  const int* idx;
  __device__ __forceinline__ void operator()(int p, double v) const { out[idx[p]] = (float)v; }
};

__global__ void __launch_bounds__(kThreads) k_gather_bucketed(const float* __restrict__ g, const int* __restrict__ idx,
                                                              long long M, float* __restrict__ gb) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < M; p += stride) gb[p] = g[idx[p]];
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
  n += align_up((size_t)M * sizeof(float));                // gS in bucket order
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
  float* gb;
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
  w.idx = (int*)p; p += align_up((size_t)M * sizeof(int));
  w.gb = (float*)p;
  return w;
}

RefAnchors bucket_anchors(const PairWs& w, const long long* AC, const float* AX, const float* AT,
                             const long long* AID, long long M, long long S, long long GH, long long GW,
                             long long ncell, float* out_invalid, cudaStream_t s) {
  cudaMemsetAsync(w.counts, 0, (size_t)ncell * sizeof(int), s);
  if (M > 0)
    launch(k_anchor_count, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, M, S, GH, GW, ncell, w.counts);
  exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);
  if (M > 0)
    launch(k_anchor_scatter, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, 
        AC, (const float2*)AX, AT, AID, M, S, GH, GW, ncell, w.start, w.counts, w.xy, w.t, w.id, w.idx, out_invalid);
  RefAnchors A;
  A.xy = w.xy; A.t = w.t; A.id = w.id; A.idx = w.idx;
  return A;
}

int warp_grid(long long nwarps) { return clamp_grid(blocks_for(nwarps * 32, kThreads)); }
}  // namespace

int pair_fwd(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
             const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC, long long M,
             long long ncell, long long S, long long GH, long long GW, double h, double tau, double cut, float* out,
             void* ws, cudaStream_t s) {
  const PairWs w = carve(ws, M, ncell);
  const RefAnchors A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, out, s);
  const RefEntries E{(const float2*)SY, (const float2*)SV, ST, SID};
  const CellGrid G{GW, GH, S, ncell};
  const PairConsts C = make_pair_consts(h, tau, cut);
  if (M > 0 && ncell > 0) {
    cudaEvent_t e0 = timing_begin(s);
    launch(k_pair_fwd_t<RefEntries, RefAnchors, long long, RefOut>, warp_grid(ncell), kThreads, 0, s, E, A,
           (const int*)w.start, CS, G, SC, C, RefOut{out, w.idx});
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
  const RefAnchors A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, nullptr, s);
  const RefEntries E{(const float2*)SY, (const float2*)SV, ST, SID};
  const CellGrid G{GW, GH, S, ncell};
  const PairConsts C = make_pair_consts(h, tau, cut);
  if (M > 0 && ncell > 0) {
    launch(k_gather_bucketed, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, gS, (const int*)w.idx, M, w.gb);
    cudaEvent_t e0 = timing_begin(s);
    launch(k_pair_bwd_t<RefEntries, RefAnchors, long long>, warp_grid(ncell), kThreads, 0, s, E, A,
           (const int*)w.start, (const float*)w.gb, CS, G, SC, C, N, gv);
    timing_end("k_pair_bwd", s, e0);
  }
  return launch_status("ats_pair_bwd");
}

// ---- allocation-free forward ---------------------------------------------------------------------
// Some callers cannot call cudaMalloc at the point where they need the pair sums: code running while
// a stream is being captured into a CUDA graph by someone else, hosts that hand the library a fixed
// device-memory budget (a custom allocator, an embedded runtime, a real-time loop that forbids
// allocation after start-up), or FFI layers with no device allocator of their own.  For them the
// forward's anchor buckets live in this file-scope device array instead of a caller workspace.  Every
// device that loads the library holds these bytes until the process exits.  In host code the array's
// name is a stand-in for the symbol, not a device address: its address on the current device comes
// from cudaGetSymbolAddress, looked up once per device on that device's first call.
constexpr size_t kNoAllocScratchBytes = ATLB_PAIR_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_pair_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_pair_scratch on the current device (looked up on the first call per device).
int pair_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("ats_pair_fwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return ATLB_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("ats_pair_fwd_noalloc: device ordinal %d beyond the %d supported", dev, kMaxDevices);
    return ATLB_ERR_ARG;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pair_scratch);
    if (e != cudaSuccess || !p) {
      set_error("ats_pair_fwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return ATLB_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return ATLB_OK;
}
}  // namespace

// Same kernels and result as pair_fwd; the workspace is g_pair_scratch.  The per-cell counters are
// zeroed on the stream by every call (bucket_anchors), and every other byte used is written before it
// is read, so what an earlier call left in the array does not matter.  Calls whose work overlaps on the
// GPU (two streams, or two host threads) share the array and race.  Not timed by atlb_timing_*, whose
// events would be created here.
int pair_fwd_noalloc(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
                     const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC,
                     long long M, long long ncell, long long S, long long GH, long long GW, double h, double tau,
                     double cut, float* out, cudaStream_t s) {
  const size_t need = pair_workspace_bytes(M, ncell);
  if (need > kNoAllocScratchBytes) {
    set_error("atlb_ats_pair_fwd_noalloc: %lld anchors over %lld cells need %zu scratch bytes, above the fixed %zu",
              M, ncell, need, kNoAllocScratchBytes);
    return ATLB_ERR_WORKSPACE;
  }
  void* ws = nullptr;
  if (int st = pair_scratch_address(&ws)) return st;
  const PairWs w = carve(ws, M, ncell);
  const RefAnchors A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, out, s);
  const RefEntries E{(const float2*)SY, (const float2*)SV, ST, SID};
  const CellGrid G{GW, GH, S, ncell};
  const PairConsts C = make_pair_consts(h, tau, cut);
  if (M > 0 && ncell > 0)
    launch(k_pair_fwd_t<RefEntries, RefAnchors, long long, RefOut>, warp_grid(ncell), kThreads, 0, s, E, A,
           (const int*)w.start, CS, G, SC, C, RefOut{out, w.idx});
  return launch_status("ats_pair_fwd_noalloc");
}

}  // namespace atlb
