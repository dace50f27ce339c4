// Parameters of the pixel-trajectory transport kernels (traj.cu), shared with the C ABI (capi.cu).
#pragma once

namespace atlb {

constexpr int kTrajKMax = 16;

struct TrajView {
  const float* C;                 // (B, Hq, Wq, 2K) tile coefficients, channels-last
  int B, Hq, Wq, K, n_fp, basis;  // basis: 0 polynomial t^k, 1 Bezier (Bernstein, first point pinned)
  float offset, tile;
  float rtile;                    // RN(1 / tile)
  int tile_pow2;                  // tile is a power of two: (p - offset) / tile == (p - offset) * rtile exactly
  float bc[kTrajKMax];            // Bezier binomial factors exp(logc_k), as the reference computes them in fp32
};

}  // namespace atlb
