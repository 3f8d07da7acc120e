"""Mirror of src/kernels/rmsnorm.zig."""
from __future__ import annotations

from .. import ops


class RMSNorm:
    """RMSNorm (rmsnorm.zig:6-43); rows = x.count / dim as in rmsnorm.zig:33."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "RMSNorm":
        return cls(device)

    def forward(self, x, weight, out, dim, eps):
        ops.rmsnorm(self.device, x, weight, out, x.count // int(dim), dim, eps)
