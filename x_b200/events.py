"""The event input of the anchored-score path.

The objectives and ops of this package read seven attributes of the events they are given, which is the
layout of the reference's ``atl.core.events.EventPacket`` (atl/core/events.py:23-34):

    xy          (N, 2) float32, pixel coordinates [x, y], pixel centres at integers
    t           (N,)   float32, time normalised to the window, [0, 1]
    p           (N,)   float32 polarity (+1 / -1; not used by the score)
    b           (N,)   int64 batch index in [0, batch_size)
    batch_size, height, width

with the events of all windows packed and sorted by (b, t).  Any object with these attributes works, the
reference's own EventPacket included; :class:`Events` below is this package's container for them, with the
few helpers the path needs (the device move, the in-image test used for anchor margins, and a check of the
sort invariant, which the fused kernels also verify on the device).
"""
from __future__ import annotations

from typing import Optional

import torch


class Events:
    """Packed, (b, t)-sorted events of ``batch_size`` windows of ``height`` x ``width`` pixels."""

    __slots__ = ("xy", "t", "p", "b", "batch_size", "height", "width", "duration", "meta")

    def __init__(self, xy: torch.Tensor, t: torch.Tensor, p: torch.Tensor, b: torch.Tensor, batch_size: int,
                 height: int, width: int, duration: Optional[torch.Tensor] = None, meta: Optional[dict] = None):
        if xy.dim() != 2 or xy.shape[-1] != 2 or not (t.shape[0] == p.shape[0] == b.shape[0] == xy.shape[0]):
            raise ValueError("Events: xy must be (N, 2) and t, p, b (N,)")
        self.xy, self.t, self.p, self.b = xy, t, p, b
        self.batch_size, self.height, self.width = int(batch_size), int(height), int(width)
        self.duration = duration  # per-window length in seconds (optional metadata)
        self.meta = {} if meta is None else meta

    @property
    def n(self) -> int:
        return int(self.t.shape[0])

    @property
    def device(self) -> torch.device:
        return self.t.device

    def to(self, device, non_blocking: bool = False) -> "Events":
        mv = lambda x: None if x is None else x.to(device, non_blocking=non_blocking)  # noqa: E731
        return Events(mv(self.xy), mv(self.t), mv(self.p), mv(self.b), self.batch_size, self.height, self.width,
                      mv(self.duration), dict(self.meta))

    def inside(self, xy: Optional[torch.Tensor] = None, margin: float = 0.0) -> torch.Tensor:
        """Boolean mask of the positions (default: the events') within the image extended by ``margin`` px
        (a negative margin shrinks it), pixel centres 0..W-1 and 0..H-1."""
        q = self.xy if xy is None else xy
        lo = -float(margin)
        return ((q[:, 0] >= lo) & (q[:, 0] <= self.width - 1 - lo) & (q[:, 1] >= lo) & (q[:, 1] <= self.height - 1 - lo))

    def is_sorted(self) -> bool:
        """True when the events are ordered by (b, t), the invariant the window counts rely on (keys b*4 + t
        compared in float64, as the reference's window search does)."""
        if self.n < 2:
            return True
        key = self.b.to(torch.float64) * 4.0 + self.t.to(torch.float64)
        return bool((key[1:] >= key[:-1]).all())

    def __repr__(self) -> str:
        return f"Events(n={self.n}, batch_size={self.batch_size}, {self.height}x{self.width}, device={self.device})"


# The reference's name for the container: code written against atl.core.events keeps working.
EventPacket = Events
