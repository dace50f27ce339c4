"""Opt-in device draws of the anchored objectives' noise (libatlb200 ``atlb_rng_*``).

The reference draws the dequantisation jitter u ~ U[0,1)^2 and the anchor smoothing noise z ~ N(0, I) on
the host with the objective's torch CPU generator (atl/objectives/ats.py:84-88, 133-135), then copies them to
the device.  These draws come from a counter-based generator (Philox4x32-10) on the device instead: no host
work and no copy per step, but a different random stream, so the objectives use them only when constructed
with ``device_rng=True``.  Draw ``call`` of a generator with seed ``seed`` is reproducible: item i of call c
always gets the same numbers.
"""
from __future__ import annotations

import torch

from . import _lib as L


def uniform2(seed: int, call: int, n: int, device) -> torch.Tensor:
    """(n, 2) float32 uniforms in [0, 1): stream 0 of (seed, call)."""
    out = torch.empty(n, 2, dtype=torch.float32, device=device)
    L.check(L.lib().atlb_rng_uniform2(int(seed) & (2**64 - 1), int(call), n, L.ptr(out), L.stream()), "rng_uniform2")
    return out


def normal2(seed: int, call: int, n: int, device) -> torch.Tensor:
    """(n, 2) float32 standard normals: stream 1 of (seed, call)."""
    out = torch.empty(n, 2, dtype=torch.float32, device=device)
    L.check(L.lib().atlb_rng_normal2(int(seed) & (2**64 - 1), int(call), n, L.ptr(out), L.stream()), "rng_normal2")
    return out


class DeviceDraws:
    """Seed and call counter of an objective's device draws: every ``next_call()`` is a fresh draw."""

    def __init__(self, seed=None):
        self.seed = int(seed) if seed is not None else int(torch.randint(0, 2**62, (1,)).item())
        self.calls = 0

    def next_call(self) -> int:
        c = self.calls
        self.calls += 1
        return c
