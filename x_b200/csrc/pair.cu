// Anchored pair sums over the reference plan layout: the B200 replacement of ats_pair_fwd /
// ats_pair_bwd (csrc/atl_cpu.cpp:176-253).
//
// Reference: one thread per anchor walks its 3x3 cells; the backward scatters 2 global float atomics per
// pair.  Here the anchors are first bucketed by cell (counting sort, same key as the sources) into 16-byte
// records, and the plan's entries are read where the caller holds them (SoA, int64 ids and CSR offsets):
//   * forward: the shared-memory tiled kernel of the fused path (pair_tiled.cuh).  Per tile of 8 x 4 cells
//     the entries of the surrounding cells are staged with cp.async and assembled there into (y, v) and
//     (t, id) records.  Leave-one-out compares the entry's id with the anchor's, per pair, on the low 32
//     bits; when some id does not fit in 32 bits (the count pass flags it) every cell takes the untiled
//     kernel instead, which compares all 64;
//   * backward: one warp per source cell, one entry per lane, the anchors of the 3x3 neighbourhood read as
//     warp-uniform broadcast records: the gradient of an entry is summed in registers and leaves with ONE
//     vector red.global instead of two atomics per pair.
// The acceptance test (|dt| <= tau, d^2 <= (cut h)^2, leave-one-out by id) follows the reference's exact
// rounding sequence, so the set of contributing pairs is identical; the kernel value (ex2) and the order of
// summation differ from the reference in the last bits.  Grids the tiled kernels cannot index (2^31 entries
// or more, a cell count that is not a whole number of S x GH x GW grids, more than 65535 slices) take the
// per-cell-warp kernels of pair_kernels.cuh.
#include <mutex>

#include "common.cuh"
#include "pair_kernels.cuh"
#include "pair_math.cuh"
#include "pair_tiled.cuh"
#include "plan_math.cuh"
#include "scan.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ long long anchor_key(const long long* AC, long long i, long long S, long long GH,
                                                long long GW, long long ncell) {
  const long long g = AC[3 * i], cx = AC[3 * i + 1], cy = AC[3 * i + 2];
  if (g < 0 || cx < 0 || cx >= GW || cy < 0 || cy >= GH) return -1;
  const long long key = (g * GH + cy) * GW + cx;
  return key < ncell ? key : -1;
}

__device__ __forceinline__ bool wide_id(long long id) { return ((unsigned long long)id >> 32) != 0; }

// Anchors per cell.  With `flags`, also raises kOverflowAll when an anchor id (AID) or an entry id (SID) is
// negative or not below 2^32, the range in which the tiled forward's 32-bit comparison is exact.
__global__ void __launch_bounds__(kThreads) k_anchor_count(const long long* __restrict__ AC,
                                                           const long long* __restrict__ AID, long long M,
                                                           const long long* __restrict__ SID, long long Ns,
                                                           long long S, long long GH, long long GW, long long ncell,
                                                           int* __restrict__ counts, int* __restrict__ flags) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long n = M > Ns ? M : Ns;
  bool wide = false;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    if (i < M) {
      const long long key = anchor_key(AC, i, S, GH, GW, ncell);
      if (key >= 0) atomicAdd(counts + key, 1);
      if (flags) wide |= wide_id(AID[i]);
    }
    if (flags && i < Ns) wide |= wide_id(SID[i]);
  }
  if (wide) atomicOr(flags, kOverflowAll);
}

// Generic kernels' anchor buckets: SoA copies.
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

// Tiled forward's anchor records: XT = (x, y, t, low 32 bits of the id), BI = original index.
__global__ void __launch_bounds__(kThreads) k_anchor_records_fwd(const long long* __restrict__ AC,
                                                                 const float2* __restrict__ AX,
                                                                 const float* __restrict__ AT,
                                                                 const long long* __restrict__ AID, long long M,
                                                                 long long S, long long GH, long long GW,
                                                                 long long ncell, const int* __restrict__ start,
                                                                 int* __restrict__ cursor, float4* __restrict__ XT,
                                                                 int* __restrict__ BI, float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const long long key = anchor_key(AC, i, S, GH, GW, ncell);
    if (key < 0) {
      out[i] = __int_as_float(0x7fc00000);  // a cell outside the grid, as the generic path
      continue;
    }
    const int p = start[key] + atomicAdd(cursor + key, 1);
    const float2 x = AX[i];
    XT[p] = make_float4(x.x, x.y, AT[i], __int_as_float((int)AID[i]));
    BI[p] = (int)i;
  }
}

// Cell-per-warp backward's anchor records: AB = (x, y, t - c_s, t - c_s), GT = (dL/dS / h^2, t), GID = id.
__global__ void __launch_bounds__(kThreads) k_anchor_records_bwd(const long long* __restrict__ AC,
                                                                 const float2* __restrict__ AX,
                                                                 const float* __restrict__ AT,
                                                                 const long long* __restrict__ AID,
                                                                 const float* __restrict__ gS,
                                                                 const float* __restrict__ SC, long long M,
                                                                 long long S, long long GH, long long GW,
                                                                 long long ncell, float invh2,
                                                                 const int* __restrict__ start,
                                                                 int* __restrict__ cursor, float4* __restrict__ AB,
                                                                 float2* __restrict__ GT, long long* __restrict__ GID) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M; i += stride) {
    const long long key = anchor_key(AC, i, S, GH, GW, ncell);
    if (key < 0) continue;
    const int p = start[key] + atomicAdd(cursor + key, 1);
    const float2 x = AX[i];
    const float t = AT[i];
    const float dts = sub_rn(t, __ldg(SC + AC[3 * i] % S));
    AB[p] = make_float4(x.x, x.y, dts, dts);
    GT[p] = make_float2(gS[i] * invh2, t);
    GID[p] = AID[i];
  }
}

struct RefOut {
  float* out;
  const int* idx;
  __device__ __forceinline__ void operator()(int p, double v) const { out[idx[p]] = (float)v; }
};

// Output of the tiled forward: it passes the original anchor index.
struct DirectOut {
  float* out;
  __device__ __forceinline__ void operator()(int i, double v) const { out[i] = (float)v; }
};

__global__ void __launch_bounds__(kThreads) k_gather_bucketed(const float* __restrict__ g, const int* __restrict__ idx,
                                                              long long M, float* __restrict__ gb) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < M; p += stride) gb[p] = g[idx[p]];
}

}  // namespace

// Per anchor: a 16-byte record (tiled kernels; the generic kernels keep x and t there), the id, and 8 bytes
// that hold the original index and dL/dS (generic kernels, tiled forward) or the tiled backward's
// (dL/dS / h^2, t).  Per cell: a count / cursor and a CSR offset.  Two ints after the counts hold the
// forward's overflow word.
size_t pair_workspace_bytes(long long M, long long ncell) {
  size_t n = 0;
  n += align_up((size_t)(ncell + 2) * sizeof(int));        // counts / cursor, overflow word
  n += align_up((size_t)(ncell + 1) * sizeof(int));        // start
  n += align_up(scan_partials_bytes(ncell));               // scan partials
  n += align_up((size_t)M * sizeof(float4));               // records (generic: xy, then t)
  n += align_up((size_t)M * sizeof(long long));            // id
  n += align_up((size_t)M * 2 * sizeof(float));            // idx + gS in bucket order, or (gS / h^2, t)
  return n + 256;
}

namespace {
struct PairWs {
  int* counts;
  int* flags;
  int* start;
  long long* partials;
  float4* rec;
  float2* xy;  // generic kernels: inside rec
  float* t;
  long long* id;
  int* idx;
  float* gb;   // follows idx
  float2* gt;  // the tiled backward's (gS / h^2, t): the idx and gb bytes
};
PairWs carve(void* ws, long long M, long long ncell) {
  char* p = (char*)align_ptr(ws);
  PairWs w;
  w.counts = (int*)p; p += align_up((size_t)(ncell + 2) * sizeof(int));
  w.flags = w.counts + ncell;
  w.start = (int*)p; p += align_up((size_t)(ncell + 1) * sizeof(int));
  w.partials = (long long*)p; p += align_up(scan_partials_bytes(ncell));
  w.rec = (float4*)p; p += align_up((size_t)M * sizeof(float4));
  w.xy = (float2*)w.rec;
  w.t = (float*)(w.xy + M);
  w.id = (long long*)p; p += align_up((size_t)M * sizeof(long long));
  w.idx = (int*)p;
  w.gb = (float*)(w.idx + M);
  w.gt = (float2*)p;
  return w;
}

RefAnchors bucket_anchors(const PairWs& w, const long long* AC, const float* AX, const float* AT,
                          const long long* AID, long long M, long long S, long long GH, long long GW,
                          long long ncell, float* out_invalid, cudaStream_t s) {
  cudaMemsetAsync(w.counts, 0, (size_t)ncell * sizeof(int), s);
  if (M > 0)
    launch(k_anchor_count, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, AID, M, (const long long*)nullptr,
           0LL, S, GH, GW, ncell, w.counts, (int*)nullptr);
  exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);
  if (M > 0)
    launch(k_anchor_scatter, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, (const float2*)AX, AT, AID, M,
           S, GH, GW, ncell, w.start, w.counts, w.xy, w.t, w.id, w.idx, out_invalid);
  RefAnchors A;
  A.xy = w.xy; A.t = w.t; A.id = w.id; A.idx = w.idx;
  return A;
}

int warp_grid(long long nwarps) { return clamp_grid(blocks_for(nwarps * 32, kThreads)); }

// The tiled kernels' grid when the plan fits their 32-bit indexing: ncell = B x S x GH x GW.
bool tiled_grid(long long Ns, long long ncell, long long S, long long GH, long long GW, TileGrid* T) {
  if (Ns >= INT_MAX || GH <= 0 || GW <= 0 || S < 1 || S > 65535) return false;
  const long long per = S * GH * GW;
  if (ncell % per != 0 || (GH + kTileY - 1) / kTileY > 65535) return false;
  *T = TileGrid{(int)GW, (int)GH, (int)S, (int)(ncell / per)};
  return true;
}

unsigned long long g_ref_fwd_attr = 0;  // devices on which the tiled forward's shared-memory opt-in is set

// Forward into `out` with the buckets in `ws`; `timed`: report the pair kernels to atlb_timing_*.
int pair_fwd_ws(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
                const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC,
                long long Ns, long long M, long long ncell, long long S, long long GH, long long GW, double h,
                double tau, double cut, float* out, void* ws, bool timed, cudaStream_t s) {
  const PairWs w = carve(ws, M, ncell);
  const RefEntries E{(const float2*)SY, (const float2*)SV, ST, SID};
  const PairConsts C = make_pair_consts(h, tau, cut);
  TileGrid T;
  if (M > 0 && ncell > 0 && tiled_grid(Ns, ncell, S, GH, GW, &T)) {
    using Tiled = void (*)(RefEntries, FastAnchors, const int*, const long long*, TileGrid, const float*, PairConsts,
                           DirectOut, int*);
    const Tiled tiled = k_pair_fwd_tiled<false, true, RefEntries, long long, DirectOut>;
    if (first_use_on_device(g_ref_fwd_attr))  // the opt-in above 48 KB is a per-device attribute
      cudaFuncSetAttribute(tiled, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TileSmemFwd));
    cudaMemsetAsync(w.counts, 0, (size_t)(ncell + 2) * sizeof(int), s);  // counts and the overflow word
    launch(k_anchor_count, clamp_grid(blocks_for(M > Ns ? M : Ns, kThreads)), kThreads, 0, s, AC, AID, M, SID, Ns, S,
           GH, GW, ncell, w.counts, w.flags);
    exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);
    launch(k_anchor_records_fwd, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, (const float2*)AX, AT, AID,
           M, S, GH, GW, ncell, (const int*)w.start, w.counts, w.rec, w.idx, out);
    const FastAnchors A{w.rec, w.idx};
    const dim3 grid((unsigned)((GW + kTileX - 1) / kTileX), (unsigned)((GH + kTileY - 1) / kTileY), (unsigned)S);
    cudaEvent_t e0 = timed ? timing_begin(s) : nullptr;
    launch(tiled, grid, kTileThreads, sizeof(TileSmemFwd), s, E, A, (const int*)w.start, CS, T, SC, C, DirectOut{out},
           w.flags);
    launch(k_pair_fwd_overflow<false, true, RefEntries, long long, DirectOut>, warp_grid(ncell), 256, 0, s, E, A, AID,
           (const int*)w.start, CS, T, SC, C, DirectOut{out}, (const int*)w.flags);
    if (timed) timing_end("k_pair_fwd", s, e0);
    return ATLB_OK;
  }
  const RefAnchors A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, out, s);
  const CellGrid G{GW, GH, S, ncell};
  if (M > 0 && ncell > 0) {
    cudaEvent_t e0 = timed ? timing_begin(s) : nullptr;
    launch(k_pair_fwd_t<RefEntries, RefAnchors, long long, RefOut>, warp_grid(ncell), kThreads, 0, s, E, A,
           (const int*)w.start, CS, G, SC, C, RefOut{out, w.idx});
    if (timed) timing_end("k_pair_fwd", s, e0);
  }
  return ATLB_OK;
}
}  // namespace

int pair_fwd(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
             const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC, long long Ns,
             long long M, long long ncell, long long S, long long GH, long long GW, double h, double tau, double cut,
             float* out, void* ws, cudaStream_t s) {
  pair_fwd_ws(SY, SV, ST, SID, CS, AX, AT, AC, AID, SC, Ns, M, ncell, S, GH, GW, h, tau, cut, out, ws, true, s);
  return launch_status("ats_pair_fwd");
}

int pair_bwd(const float* gS, const float* SY, const float* SV, const float* ST, const long long* SID,
             const long long* CS, const float* AX, const float* AT, const long long* AC, const long long* AID,
             const float* SC, long long Ns, long long M, long long ncell, long long S, long long GH, long long GW,
             double h, double tau, double cut, long long N, float* gv, void* ws, cudaStream_t s) {
  const PairWs w = carve(ws, M, ncell);
  cudaMemsetAsync(gv, 0, (size_t)N * 2 * sizeof(float), s);
  const RefEntries E{(const float2*)SY, (const float2*)SV, ST, SID};
  const PairConsts C = make_pair_consts(h, tau, cut);
  TileGrid T;
  if (M > 0 && ncell > 0 && tiled_grid(Ns, ncell, S, GH, GW, &T)) {
    cudaMemsetAsync(w.counts, 0, (size_t)ncell * sizeof(int), s);
    launch(k_anchor_count, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, AID, M, (const long long*)nullptr,
           0LL, S, GH, GW, ncell, w.counts, (int*)nullptr);
    exclusive_scan<int>(w.counts, ncell, w.partials, w.start, s);
    launch(k_anchor_records_bwd, clamp_grid(blocks_for(M, kThreads)), kThreads, 0, s, AC, (const float2*)AX, AT, AID,
           gS, SC, M, S, GH, GW, ncell, C.invh2, (const int*)w.start, w.counts, w.rec, w.gt, w.id);
    const int nrows = (int)(ncell / GW);
    const dim3 grid((unsigned)((GW + 7) / 8), (unsigned)(nrows < 65535 ? nrows : 65535));
    cudaEvent_t e0 = timing_begin(s);
    launch(k_pair_bwd_cells<false, true, RefEntries, long long>, grid, 256, 0, s, E, (const float4*)w.rec,
           (const float2*)w.gt, (const long long*)w.id, (const int*)w.start, CS, (int)GW, (int)GH, nrows, C, N, gv);
    timing_end("k_pair_bwd", s, e0);
    return launch_status("ats_pair_bwd");
  }
  const RefAnchors A = bucket_anchors(w, AC, AX, AT, AID, M, S, GH, GW, ncell, nullptr, s);
  const CellGrid G{GW, GH, S, ncell};
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
// Some callers cannot call cudaMalloc at the point where they need the pair sums: hosts that hand the
// library a fixed device-memory budget (a custom allocator, an embedded runtime), loops that forbid
// cudaMalloc after start-up because it can synchronise the device, and FFI layers with no device
// allocator of their own.  For them the forward's anchor buckets live in this file-scope device array
// instead of a caller workspace.  Every device that loads the library holds these bytes until the
// process exits.  In host code the array's name is a stand-in for the symbol, not a device address: its
// address on the current device comes from cudaGetSymbolAddress, looked up once per device on that
// device's first call and kept for the process (the primary context's module; cudaDeviceReset or another
// context on the device would invalidate it).
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

// Same kernels and result as pair_fwd; the workspace is g_pair_scratch.  The per-cell counters and the
// overflow word are zeroed on the stream by every call, and every other byte used is written before it is
// read, so what an earlier call left in the array does not matter.  Calls whose work overlaps on the GPU
// (two streams, or two host threads) share the array and race.  Not timed by atlb_timing_*, whose events
// would be created here.
int pair_fwd_noalloc(const float* SY, const float* SV, const float* ST, const long long* SID, const long long* CS,
                     const float* AX, const float* AT, const long long* AC, const long long* AID, const float* SC,
                     long long Ns, long long M, long long ncell, long long S, long long GH, long long GW, double h,
                     double tau, double cut, float* out, cudaStream_t s) {
  // the workspace size less its 256 bytes of alignment slack: the array itself is 256-byte aligned
  const size_t need = pair_workspace_bytes(M, ncell) - 256;
  if (need > kNoAllocScratchBytes) {
    set_error("atlb_ats_pair_fwd_noalloc: %lld anchors over %lld cells need %zu scratch bytes, above the fixed %zu",
              M, ncell, need, kNoAllocScratchBytes);
    return ATLB_ERR_WORKSPACE;
  }
  void* ws = nullptr;
  if (int st = pair_scratch_address(&ws)) return st;
  pair_fwd_ws(SY, SV, ST, SID, CS, AX, AT, AC, AID, SC, Ns, M, ncell, S, GH, GW, h, tau, cut, out, ws, false, s);
  return launch_status("ats_pair_fwd_noalloc");
}

}  // namespace atlb
