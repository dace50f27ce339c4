"""Seeded synthetic event windows with the shapes of the benchmark configurations.

The reference's own simulator (atl/data/synthetic.py) is not part of its tree, and its datasets
(DSEC / EVIMO2) are not available; these generators produce windows with the sizes, value ranges
and distributions the benchmark configurations name:

* ``uniform_window``   integer pixel coordinates uniform over the sensor, times uniform and sorted
                       (configuration 1, 100k events on 240x180);
* ``textured_window``  event density proportional to the gradient magnitude of a smooth random texture
                       (configuration 2, 1M events on 640x480, and its scaled versions);
* ``lowpass_flow``     Gaussian low-pass white noise (sigma in pixels) scaled to a maximum speed
                       (the dense per-pixel flow of configuration 2, in px per window).

Times are generated in seconds over the window duration and normalised to [0, 1] the way
EventPacket.from_arrays does (float64 then float32).  Everything is drawn on the CPU from a seeded
generator (identical data on every machine and for every implementation) and then moved to
``device``.
"""
from __future__ import annotations

import math

import torch

from .events import EventPacket


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def _normalised_sorted_times(n: int, duration: float, g) -> torch.Tensor:
    t = torch.sort(torch.rand(n, generator=g, dtype=torch.float64, device=g.device) * duration).values
    if n > 0:
        t0, t1 = t.min(), t.max()
        t = (t - t0) / torch.clamp(t1 - t0, min=1e-12)
    return t.to(torch.float32)


def _polarity(n, g):
    return torch.where(torch.rand(n, generator=g, device=g.device) > 0.5, 1.0, -1.0).to(torch.float32)


def uniform_window(n: int, H: int, W: int, duration: float = 0.05, seed: int = 0, device="cpu") -> EventPacket:
    g = _gen(seed)
    x = torch.randint(0, W, (n,), generator=g).float()
    y = torch.randint(0, H, (n,), generator=g).float()
    t = _normalised_sorted_times(n, duration, g)
    p = _polarity(n, g)
    b = torch.zeros(n, dtype=torch.long)
    return EventPacket(torch.stack([x, y], 1), t, p, b, 1, H, W).to(device)


def _gauss_blur(img: torch.Tensor, sigma: float) -> torch.Tensor:
    """Separable Gaussian low-pass of a (C, H, W) tensor (reflect padding)."""
    r = max(int(math.ceil(3 * sigma)), 1)
    x = torch.arange(-r, r + 1, device=img.device, dtype=img.dtype)
    k = torch.exp(-x * x / (2 * sigma * sigma))
    k = k / k.sum()
    C = img.shape[0]
    z = img[None]
    pad_x, pad_y = min(r, img.shape[-1] - 1), min(r, img.shape[-2] - 1)
    z = torch.nn.functional.pad(z, (pad_x, pad_x, 0, 0), mode="reflect")
    z = torch.nn.functional.conv2d(z, k[r - pad_x:r + pad_x + 1].view(1, 1, 1, -1).expand(C, 1, 1, -1), groups=C)
    z = torch.nn.functional.pad(z, (0, 0, pad_y, pad_y), mode="reflect")
    z = torch.nn.functional.conv2d(z, k[r - pad_y:r + pad_y + 1].view(1, 1, -1, 1).expand(C, 1, -1, 1), groups=C)
    return z[0]


def textured_window(n: int, H: int, W: int, duration: float = 0.1, seed: int = 0, texture_sigma: float = 2.0,
                    batch: int = 1, device="cpu", draw_on_device: bool = False) -> EventPacket:
    """``batch`` windows of ``n`` events each, density proportional to |grad texture| (integer pixels).
    ``draw_on_device``: draw with a seeded generator of ``device`` instead of the CPU one (other numbers,
    same distributions; for windows of tens of millions of events)."""
    if draw_on_device:
        g = torch.Generator(device=device).manual_seed(int(seed))
        dev = torch.device(device)
    else:
        g, dev = _gen(seed), torch.device("cpu")
    xs, ts, ps, bs = [], [], [], []
    for k in range(batch):
        tex = _gauss_blur(torch.randn(1, H, W, generator=g, device=dev), texture_sigma)[0]
        gx = torch.zeros_like(tex); gy = torch.zeros_like(tex)
        gx[:, 1:-1] = 0.5 * (tex[:, 2:] - tex[:, :-2])
        gy[1:-1, :] = 0.5 * (tex[2:, :] - tex[:-2, :])
        w = torch.sqrt(gx * gx + gy * gy).reshape(-1) + 1e-6
        idx = torch.multinomial(w / w.sum(), n, replacement=True, generator=g)
        xs.append(torch.stack([(idx % W).float(), (idx // W).float()], 1).to(dev))
        ts.append(_normalised_sorted_times(n, duration, g))
        ps.append(_polarity(n, g))
        bs.append(torch.full((n,), k, dtype=torch.long, device=dev))
    return EventPacket(torch.cat(xs), torch.cat(ts), torch.cat(ps), torch.cat(bs), batch, H, W).to(device)


def lowpass_flow(B: int, H: int, W: int, sigma: float = 32.0, vmax: float = 20.0, seed: int = 0,
                 device="cpu") -> torch.Tensor:
    """(B, 2, H, W) float32 flow: Gaussian low-pass white noise scaled so that max |v| = vmax."""
    g = _gen(seed)
    out = []
    for _ in range(B):
        f = _gauss_blur(torch.randn(2, H, W, generator=g), sigma)
        mag = torch.sqrt(f[0] ** 2 + f[1] ** 2).max().clamp(min=1e-12)
        out.append(f * (vmax / mag))
    return torch.stack(out).float().contiguous().to(device)


CONFIGS = {
    # name: (events per window, H, W, duration s, windows)
    "config1": (100_000, 180, 240, 0.05, 1),
    "config2": (1_000_000, 480, 640, 0.1, 1),
    "config5_window": (64_000_000, 720, 1280, 0.2, 1),
}
