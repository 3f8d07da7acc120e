"""Mirror of src/kernels/quantized.zig."""
from __future__ import annotations

from .. import ops


class QMatMulInt4:
    """QMatMulInt4 (quantized.zig:6-51): INT4 fused-dequant matvec.

    forward(x f32, w_packed u8, scales f16, zeros u8, out f32, m, k, n, group_size) binds
    the same five buffers and four scalars as the reference (quantized.zig:30-39) and is
    synchronous like it (quantized.zig:47-49).  Unlike the reference kernel, which
    computes row 0 only and requires k <= 4096 (shaders.zig:457-460), all m rows of x
    are computed and k is only required to be a multiple of group_size.
    """

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "QMatMulInt4":
        return cls(device)

    def forward(self, x, w_packed, scales, zeros, out, m, k, n, group_size):
        ops.qmatmul_int4(self.device, x, w_packed, scales, zeros, out, m, k, n, group_size)
