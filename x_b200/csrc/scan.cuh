// Exclusive prefix sum of per-cell int32 counts -> CSR offsets, in three launches:
//   partials (one sum per 4096-item chunk) -> scan of the partials (one CTA) -> chunk scan + offset.
// The counts are zeroed on the way so that the same array serves as the per-cell cursor of the
// scatter pass that follows (pos = offset[key] + atomicAdd(&counts[key], 1)).
#pragma once
#include "common.cuh"

namespace atlb {
namespace {  // per translation unit: every .cu that scans gets its own copy of the kernels

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr long long kScanChunk = (long long)kScanThreads * kScanItems;

inline long long scan_nchunks(long long n) { return (n + kScanChunk - 1) / kScanChunk; }
inline size_t scan_partials_bytes(long long n) { return (size_t)(scan_nchunks(n) + 1) * sizeof(long long); }

__device__ __forceinline__ long long block_exclusive_scan(long long v, long long* smem_warp, long long* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) smem_warp[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    long long w = lane < nw ? smem_warp[lane] : 0;
    long long wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    if (lane < nw) smem_warp[lane] = wi - w;
    if (lane == nw - 1) smem_warp[32] = wi;
  }
  __syncthreads();
  const long long out = smem_warp[wid] + incl - v;
  if (total) *total = smem_warp[32];
  __syncthreads();
  return out;
}

// The kScanItems counts of thread t of chunk c are counts[c * kScanChunk + t * kScanItems + q]: one 16-byte
// load when the chunk's counts are 16-byte aligned (every chunk of a 16-byte aligned array).
__device__ __forceinline__ void load_items(const int* __restrict__ counts, long long n, long long base, int (&v)[kScanItems]) {
  static_assert(kScanItems == 4, "vector load of 4 ints");
  if (base + kScanItems <= n && ((reinterpret_cast<uintptr_t>(counts) & 15) == 0)) {
    const int4 q = __ldg(reinterpret_cast<const int4*>(counts + base));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
#pragma unroll
    for (int q = 0; q < kScanItems; ++q) v[q] = base + q < n ? counts[base + q] : 0;
  }
}

__global__ void __launch_bounds__(kScanThreads) k_scan_partials(const int* __restrict__ counts, long long n,
                                                                long long* __restrict__ partials) {
  __shared__ long long sw[33];
  const long long base = blockIdx.x * kScanChunk + (long long)threadIdx.x * kScanItems;
  int v[kScanItems];
  load_items(counts, n, base, v);
  const long long s = (long long)v[0] + v[1] + v[2] + v[3];
  long long tot;
  block_exclusive_scan(s, sw, &tot);
  if (threadIdx.x == 0) partials[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kScanThreads) k_scan_partials_scan(long long* __restrict__ partials, long long nchunks) {
  __shared__ long long sw[33];
  long long carry = 0;
  for (long long base = 0; base < nchunks; base += kScanThreads) {
    const long long i = base + threadIdx.x;
    const long long v = i < nchunks ? partials[i] : 0;
    long long tot;
    const long long ex = block_exclusive_scan(v, sw, &tot);
    if (i < nchunks) partials[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) partials[nchunks] = carry;
}

// offsets[i] = exclusive prefix (OutT = long long or int); offsets[n] = total; counts[i] = 0, or (CURSORS)
// counts[i] = offsets[i], so that a scatter's atomicAdd on counts returns absolute slots.
template <typename OutT, bool CURSORS = false>
__global__ void __launch_bounds__(kScanThreads) k_scan_final(int* __restrict__ counts, long long n,
                                                             const long long* __restrict__ partials,
                                                             OutT* __restrict__ offsets) {
  __shared__ long long sw[33];
  const long long base = blockIdx.x * kScanChunk + (long long)threadIdx.x * kScanItems;
  int v[kScanItems];
  load_items(counts, n, base, v);
  const long long s = (long long)v[0] + v[1] + v[2] + v[3];
  long long ex = block_exclusive_scan(s, sw, nullptr) + partials[blockIdx.x];
  if (sizeof(OutT) == 4 && base + kScanItems <= n && ((reinterpret_cast<uintptr_t>(offsets) & 15) == 0) &&
      ((reinterpret_cast<uintptr_t>(counts) & 15) == 0)) {
    const int o0 = (int)ex, o1 = o0 + v[0], o2 = o1 + v[1], o3 = o2 + v[2];
    *reinterpret_cast<int4*>(offsets + base) = make_int4(o0, o1, o2, o3);
    *reinterpret_cast<int4*>(counts + base) = CURSORS ? make_int4(o0, o1, o2, o3) : make_int4(0, 0, 0, 0);
  } else {
#pragma unroll
    for (int q = 0; q < kScanItems; ++q) {
      const long long i = base + q;
      if (i < n) {
        offsets[i] = (OutT)ex;
        counts[i] = CURSORS ? (int)ex : 0;
      }
      ex += v[q];
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) offsets[n] = (OutT)partials[gridDim.x];
}

// counts[0..n) -> offsets[0..n] (exclusive, offsets[n] = total); counts zeroed, or (cursors) set to the
// offsets (int offsets only).
template <typename OutT>
inline void exclusive_scan(int* counts, long long n, long long* partials, OutT* offsets, cudaStream_t s,
                           bool cursors = false) {
  const long long nch = scan_nchunks(n);
  if (nch == 0) {
    cudaMemsetAsync(offsets, 0, sizeof(OutT), s);
    return;
  }
  launch(k_scan_partials, (unsigned)nch, kScanThreads, 0, s, counts, n, partials);
  launch(k_scan_partials_scan, 1, kScanThreads, 0, s, partials, nch);
  if (cursors)
    launch(k_scan_final<OutT, true>, (unsigned)nch, kScanThreads, 0, s, counts, n, partials, offsets);
  else
    launch(k_scan_final<OutT, false>, (unsigned)nch, kScanThreads, 0, s, counts, n, partials, offsets);
}

}  // namespace
}  // namespace atlb
