// Shared device helpers for the anchored-transport-score kernels (sm_100a).
//
// Exactness: every floating-point expression that decides an INTEGER result (slice ranges, cell
// keys, anchor cells, the pair cut-off test, "inside" masks) is written with explicitly rounded
// intrinsics (__fadd_rn, __fmul_rn, __fdiv_rn, ...).  nvcc never contracts those into FMAs, so they
// round exactly as torch's eager CPU ops and the reference's x86-64 OpenMP build do.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <climits>
#include <cstring>
#include <atomic>
#include <mutex>
#include <utility>

#include "atl_b200.h"

namespace atlb {

constexpr int kWarp = 32;

// ------------------------------------------------------------------------------------ exact fp32
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Ordered-int encoding of floats for atomicMin / atomicMax over signed values.
__device__ __forceinline__ int float_to_ordered(float f) {
  int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
__host__ __device__ __forceinline__ float ordered_to_float(int i) {
#ifdef __CUDA_ARCH__
  return __int_as_float(i >= 0 ? i : i ^ 0x7fffffff);
#else
  union { int i; float f; } u;
  u.i = i >= 0 ? i : i ^ 0x7fffffff;
  return u.f;
#endif
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Vectorised fire-and-forget float2 add into global memory (sm_90+ vector reduction).
__device__ __forceinline__ void red_add_f2(float* addr, float a, float b) {
  asm volatile("red.relaxed.gpu.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add_f4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}
__device__ __forceinline__ void red_add_f1(float* addr, float a) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(addr), "f"(a) : "memory");
}

inline int blocks_for(long long n, int threads) { return (int)((n + threads - 1) / threads); }
inline int clamp_grid(long long blocks) {
  const long long cap = 148LL * 64;  // grid-stride loops beyond 64 CTAs per SM
  return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// Process-wide count of kernels launched by this library (instrumentation: atlb_kernel_launches()).
extern std::atomic<unsigned long long> g_launches;

template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  kernel<<<grid, block, smem, s>>>(std::forward<Args>(args)...);
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// Opt-in event timing of a launch (timing.cu); both are no-ops unless atlb_timing_enable(1).
cudaEvent_t timing_begin(cudaStream_t s);
void timing_end(const char* name, cudaStream_t s, cudaEvent_t e0);

// True on the first call for the current device per flag set (one bit per device): kernel attributes, such
// as the opt-in to more than 48 KB of dynamic shared memory, are per device.
inline std::mutex g_attr_mu;
inline bool first_use_on_device(unsigned long long& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return true;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  const unsigned long long m = 1ULL << dev;
  if (done & m) return false;
  done |= m;
  return true;
}

// Host-side status plumbing (capi.cu owns the thread-local message).
void set_error(const char* fmt, ...);
int launch_status(const char* what);

}  // namespace atlb
