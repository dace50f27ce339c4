"""Gradient parity criteria shared by the GPU tests.

Gradients are fp32 sums whose order differs from the reference's (fp32 atomics and warp reductions on the
GPU; omp atomics or sequential loops on the CPU), so they are compared with the accurate value (the
oracle's double-accumulated sum) in two ways:

* norm-wise: ||g - g_ref|| / ||g_ref|| <= GRAD_RTOL (1e-5, the north star's float tolerance);
* per element, where the oracle supplies the bound's ingredients: |g - g_ref| <= GRAD_RTOL |g_ref| +
  (n + PER_TERM) u A, with u = 2^-24, A = the sum of the magnitudes of the element's contributions and n
  their count.  (n - 1) u A bounds the rounding of an fp32 sum of n terms in ANY order (recursive
  summation, first order); PER_TERM u A covers the rounding of each contribution itself (products,
  the kernel value's ex2.approx at 2^-22, and the upstream dL/dS) on either side.
"""
from __future__ import annotations

import numpy as np

U = 2.0 ** -24
GRAD_RTOL = 1e-5
PER_TERM = 32


def grad_errors(g, ref) -> dict:
    """Norm-wise relative error, the largest element error relative to the largest reference element, and
    the largest per-element relative error among elements above 1e-3 of the largest."""
    g = np.asarray(g, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    d = np.abs(g - r)
    scale = max(np.abs(r).max(initial=0.0), 1e-300)
    big = np.abs(r) > 1e-3 * scale
    return {"norm": float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300)),
            "max_over_max": float(d.max(initial=0.0) / scale),
            "max_rel_big": float((d[big] / np.abs(r[big])).max(initial=0.0))}


def assert_grad_parity(g, ref, A=None, n=None, rtol: float = GRAD_RTOL, what: str = "gradient"):
    """Norm-wise relative error within ``rtol`` and, when the bound's ingredients ``A`` / ``n`` are given,
    every element within its fp32-ordering bound."""
    e = grad_errors(g, ref)
    assert e["norm"] <= rtol, f"{what}: norm-wise relative error {e['norm']:.3e} > {rtol:.0e} ({e})"
    if A is not None:
        g64 = np.asarray(g, np.float64)
        r64 = np.asarray(ref, np.float64)
        bound = rtol * np.abs(r64) + (np.asarray(n, np.float64) + PER_TERM) * U * np.asarray(A, np.float64)
        bad = np.abs(g64 - r64) > bound
        assert not bad.any(), (f"{what}: {int(bad.sum())} elements beyond the fp32 ordering bound, worst "
                               f"{float((np.abs(g64 - r64) / np.maximum(bound, 1e-300)).max()):.2f}x")
    return e
