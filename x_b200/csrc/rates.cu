// Execution-unit rates of the device the kernels run on: the denominators of the compute roofline of the
// pair and splat kernels, whose bound is not HBM bandwidth but FP32 issue, the SFU (ex2), L2 reductions
// (red.global) or shared-memory atomics.
//
// Each rate comes from one kernel that runs a single kind of operation on every SM (8 CTAs of 256 threads
// per SM, the residency limit of 2048 threads) in 8 independent chains per thread, timed with CUDA events
// after an identical warm-up launch.  Loop overhead is kept below ~3% by unrolling 16 operations per chain.
// The L2 reduction kernels scatter to pseudo-random word addresses of a 32 MB buffer (resident in L2), the
// access pattern of the pair backward's per-entry gradient reductions; the v4 form writes 16-byte aligned
// quads, the pattern of the splat's tile flush.
#include "common.cuh"
#include "plan_math.cuh"

namespace atlb {
namespace {

constexpr int kRateThreads = 256;
constexpr int kRateCtasPerSm = 8;
constexpr int kChains = 8;
constexpr int kUnroll = 16;
constexpr size_t kRedWords = (size_t)8 << 20;  // 32 MB of floats
constexpr unsigned kSmemWords = 4096;

__device__ __forceinline__ unsigned lcg(unsigned h) { return h * 1664525u + 1013904223u; }

__global__ void __launch_bounds__(kRateThreads) k_rate_ffma(float m, float c, int iters, float* sink) {
  float a[kChains];
#pragma unroll
  for (int q = 0; q < kChains; ++q) a[q] = threadIdx.x * 1e-3f + q;
  for (int i = 0; i < iters; i += kUnroll) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int q = 0; q < kChains; ++q) a[q] = __fmaf_rn(a[q], m, c);
  }
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < kChains; ++q) s += a[q];
  if (s == -1.f) sink[0] = s;  // keeps the chains live; never true for the arguments used
}

__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__global__ void __launch_bounds__(kRateThreads) k_rate_ffma2(float m, float c, int iters, float* sink) {
  unsigned long long a[kChains];
  unsigned long long mm, cc;
  asm("mov.b64 %0, {%1, %1};" : "=l"(mm) : "f"(m));
  asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
#pragma unroll
  for (int q = 0; q < kChains; ++q) {
    const float x = threadIdx.x * 1e-3f + q;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a[q]) : "f"(x), "f"(x + 0.5f));
  }
  for (int i = 0; i < iters; i += kUnroll) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int q = 0; q < kChains; ++q) a[q] = ffma2(a[q], mm, cc);
  }
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < kChains; ++q) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a[q]));
    s += lo + hi;
  }
  if (s == -1.f) sink[0] = s;
}

__global__ void __launch_bounds__(kRateThreads) k_rate_ex2(int iters, float* sink) {
  float a[kChains];
#pragma unroll
  for (int q = 0; q < kChains; ++q) a[q] = 0.1f * q + threadIdx.x * 1e-4f;
  for (int i = 0; i < iters; i += kUnroll) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int q = 0; q < kChains; ++q) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(a[q]) : "f"(-a[q]));  // -> 0.64...
  }
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < kChains; ++q) s += a[q];
  if (s == -1.f) sink[0] = s;
}

__global__ void __launch_bounds__(kRateThreads) k_rate_red(float* __restrict__ buf, int iters) {
  unsigned h = (blockIdx.x * blockDim.x + threadIdx.x) * 2654435761u;
  for (int i = 0; i < iters; i += kChains) {
#pragma unroll
    for (int q = 0; q < kChains; ++q) {
      h = lcg(h);
      red_add_f1(buf + ((h >> 7) & (unsigned)(kRedWords - 1)), 1.f);
    }
  }
}

__global__ void __launch_bounds__(kRateThreads) k_rate_red_v4(float* __restrict__ buf, int iters) {
  unsigned h = (blockIdx.x * blockDim.x + threadIdx.x) * 2654435761u;
  for (int i = 0; i < iters; i += kChains) {
#pragma unroll
    for (int q = 0; q < kChains; ++q) {
      h = lcg(h);
      red_add_f4(buf + ((h >> 7) & (unsigned)(kRedWords - 4)), 1.f, 1.f, 1.f, 1.f);
    }
  }
}

__global__ void __launch_bounds__(kRateThreads) k_rate_smem_atomic(int iters, float* sink) {
  __shared__ float sh[kSmemWords];
  for (unsigned i = threadIdx.x; i < kSmemWords; i += blockDim.x) sh[i] = 0.f;
  __syncthreads();
  unsigned h = (blockIdx.x * blockDim.x + threadIdx.x) * 2654435761u;
  for (int i = 0; i < iters; i += kChains) {
#pragma unroll
    for (int q = 0; q < kChains; ++q) {
      h = lcg(h);
      atomicAdd(&sh[(h >> 7) & (kSmemWords - 1)], 1.f);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && sh[0] < 0.f) sink[0] = sh[0];
}

// Runs `launch_once` twice (warm-up, then timed between events) and returns ops / second of the timed run.
template <class F>
int timed_rate(cudaStream_t s, double ops, F launch_once, double* rate) {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    if (e0) cudaEventDestroy(e0);
    set_error("measure_unit_rates: cudaEventCreate failed");
    return ATLB_ERR_CUDA;
  }
  launch_once();
  cudaEventRecord(e0, s);
  launch_once();
  cudaEventRecord(e1, s);
  cudaError_t e = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) {
    set_error("measure_unit_rates: %s", cudaGetErrorString(e));
    return ATLB_ERR_CUDA;
  }
  if (int st = launch_status("measure_unit_rates")) return st;
  *rate = ms > 0.f ? ops / (ms * 1e-3) : 0.0;
  return ATLB_OK;
}

}  // namespace

size_t unit_rates_scratch_bytes() { return kRedWords * sizeof(float) + 512; }

int measure_unit_rates(atlb_unit_rates* out, void* scratch, cudaStream_t s) {
  int dev = 0, nsm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) !=
                                                 cudaSuccess || nsm <= 0) {
    set_error("measure_unit_rates: no CUDA device");
    return ATLB_ERR_CUDA;
  }
  float* buf = (float*)align_ptr(scratch);
  float* sink = buf + kRedWords;
  const int blocks = nsm * kRateCtasPerSm;
  const double threads = (double)blocks * kRateThreads;
  const float m = 0.999f, c = 1e-3f;
  int st;
  const int it_fma = 8192, it_ex2 = 1024, it_red = 256, it_smem = 1024;
  st = timed_rate(s, threads * it_fma * kChains, [&] {
    launch(k_rate_ffma, blocks, kRateThreads, 0, s, m, c, it_fma, sink);
  }, &out->fp32_lane_ops);
  if (st) return st;
  st = timed_rate(s, threads * it_fma * kChains * 2, [&] {
    launch(k_rate_ffma2, blocks, kRateThreads, 0, s, m, c, it_fma, sink);
  }, &out->fp32x2_lane_ops);
  if (st) return st;
  st = timed_rate(s, threads * it_ex2 * kChains, [&] {
    launch(k_rate_ex2, blocks, kRateThreads, 0, s, it_ex2, sink);
  }, &out->ex2);
  if (st) return st;
  cudaMemsetAsync(buf, 0, kRedWords * sizeof(float), s);
  st = timed_rate(s, threads * it_red, [&] { launch(k_rate_red, blocks, kRateThreads, 0, s, buf, it_red); },
                  &out->red_f32);
  if (st) return st;
  st = timed_rate(s, threads * it_red, [&] { launch(k_rate_red_v4, blocks, kRateThreads, 0, s, buf, it_red); },
                  &out->red_v4);
  if (st) return st;
  return timed_rate(s, threads * it_smem, [&] {
    launch(k_rate_smem_atomic, blocks, kRateThreads, 0, s, it_smem, sink);
  }, &out->smem_atomic);
}

}  // namespace atlb
