"""Frame sources for the live path.

The reference captures from V4L2 devices (`src/frameshow/*.cpp`); this
environment has no capture device, so the shipped source is synthetic: moving,
bouncing coloured rectangles over a noisy background, as 8-bit BGR frames
(the capture format), deterministic for a seed.  Any iterable of [H, W, 3]
uint8 arrays (BGR) works as a source.
"""
from __future__ import annotations

from typing import Iterator, Optional

import torch

__all__ = ["SyntheticFrameSource"]


class SyntheticFrameSource:
    def __init__(self, width: int = 640, height: int = 480, objects: int = 4, frames: Optional[int] = None,
                 seed: int = 0):
        self.w, self.h, self.frames = width, height, frames
        g = torch.Generator().manual_seed(seed)
        self.pos = torch.rand(objects, 2, generator=g) * torch.tensor([width * 0.7, height * 0.7])
        self.vel = (torch.rand(objects, 2, generator=g) - 0.5) * 12
        self.size = torch.rand(objects, 2, generator=g) * torch.tensor([width * 0.25, height * 0.25]) + 24
        self.color = (torch.rand(objects, 3, generator=g) * 200 + 40).to(torch.uint8)
        self.bg = (torch.rand(height, width, 3, generator=g) * 60 + 30).to(torch.uint8)
        self.t = 0

    def __iter__(self) -> Iterator[torch.Tensor]:
        while self.frames is None or self.t < self.frames:
            yield self.next_frame()

    def next_frame(self) -> torch.Tensor:
        f = self.bg.clone()
        lim = torch.tensor([self.w, self.h]) - self.size
        self.pos += self.vel
        bounce = (self.pos < 0) | (self.pos > lim)
        self.vel[bounce] *= -1
        self.pos = torch.minimum(self.pos.clamp(min=0), lim)
        for i in range(self.pos.shape[0]):
            x0, y0 = int(self.pos[i, 0]), int(self.pos[i, 1])
            x1, y1 = x0 + int(self.size[i, 0]), y0 + int(self.size[i, 1])
            f[y0:y1, x0:x1] = self.color[i]
        self.t += 1
        return f
