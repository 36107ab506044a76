"""Helpers for the channel-group planar activation layout (KP8 / KP4) used by
the tensor-core kernels: plane p holds channels [per*p, per*p+per) of every row
as one 16-byte record, with zeroed guard rows before and after (test helper)."""
from __future__ import annotations

import torch

G_PRE = 256
G_POST = 512


class Planar:
    def __init__(self, rows: int, channels: int, dtype=torch.bfloat16, device="cuda"):
        self.per = 16 // torch.tensor([], dtype=dtype).element_size()
        assert channels % self.per == 0
        self.rows, self.channels, self.dtype = rows, channels, dtype
        self.planes = channels // self.per
        total = G_PRE + rows + G_POST
        total = (total + 15) // 16 * 16
        self.t = torch.zeros((self.planes, total, self.per), dtype=dtype, device=device)
        self.plane_stride = total * 16

    @property
    def base(self) -> int:
        return self.t.data_ptr() + G_PRE * 16

    def set(self, x: torch.Tensor) -> "Planar":
        """x: [rows, channels] -> planar."""
        assert x.shape == (self.rows, self.channels)
        v = x.to(self.dtype).reshape(self.rows, self.planes, self.per).permute(1, 0, 2)
        self.t[:, G_PRE:G_PRE + self.rows] = v
        return self

    def get(self) -> torch.Tensor:
        """planar -> [rows, channels]."""
        v = self.t[:, G_PRE:G_PRE + self.rows]
        return v.permute(1, 0, 2).reshape(self.rows, self.channels)
