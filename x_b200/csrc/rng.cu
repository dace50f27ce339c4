// Opt-in device draws of the objective's noise (include/atl_b200.h, atlb_rng_*): see rng.cuh.
#include "common.cuh"
#include "rng.cuh"

namespace atlb {
namespace {

constexpr int kThreads = 256;

template <bool NORMAL>
__global__ void __launch_bounds__(kThreads) k_rng2(RngKey K, long long n, float2* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = NORMAL ? rng_normal2(K, (unsigned long long)i) : rng_uniform2(K, (unsigned long long)i);
}

}  // namespace

int rng_draw2(bool normal, unsigned long long seed, unsigned long long call, long long n, float* out,
              cudaStream_t s) {
  if (n <= 0) return ATLB_OK;
  const RngKey K = make_rng_key(seed, call);
  const int grid = clamp_grid(blocks_for(n, kThreads));
  if (normal)
    launch(k_rng2<true>, grid, kThreads, 0, s, K, n, (float2*)out);
  else
    launch(k_rng2<false>, grid, kThreads, 0, s, K, n, (float2*)out);
  return launch_status(normal ? "rng_normal2" : "rng_uniform2");
}

}  // namespace atlb
