"""Mirror of src/kernels/fused.zig (the kernels on the INT4 FFN path)."""
from __future__ import annotations

from .. import ops


class FusedRMSNormRoPE:
    """FusedRMSNormRoPE (fused.zig:6-51); batch = x.count / dim (fused.zig:41)."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "FusedRMSNormRoPE":
        return cls(device)

    def forward(self, x, weight, cos_cache, sin_cache, out, dim, head_dim, pos, eps):
        ops.fused_rmsnorm_rope(self.device, x, weight, cos_cache, sin_cache, out,
                               x.count // int(dim), dim, head_dim, pos, eps)


class Matvec:
    """Matvec (fused.zig:53-89): out = W x, W f32 [N][K]; K of any size here."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "Matvec":
        return cls(device)

    def forward(self, x, W, out, K, N):
        ops.matvec(self.device, x, W, out, K, N)


class MatvecDual:
    """MatvecDual (fused.zig:91-133): out1 = W1 x, out2 = W2 x in one pass over x."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "MatvecDual":
        return cls(device)

    def forward(self, x, W1, W2, out1, out2, K, N):
        ops.matvec_dual(self.device, x, W1, W2, out1, out2, K, N)


class FusedSiluMul:
    """FusedSiluMul (fused.zig:178-213): out = silu(gate) * up, n = gate.count."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "FusedSiluMul":
        return cls(device)

    def forward(self, gate, up, out):
        ops.silu_mul(self.device, gate, up, out, gate.count)


class FusedInt4FFN:
    """INT4 Llama FFN, the composition of src/bench.zig:266-341 plus the down projection
    (src/model/llama.zig:220-231): out = down(silu(gate(n)) * up(n)), n = rmsnorm(x),
    optionally + x.  One persistent kernel; synchronous like the reference's forwards.
    gate/up/down are (w_packed, scales, zeros) buffer triples."""

    def __init__(self, device):
        self.device = device

    @classmethod
    def init(cls, device) -> "FusedInt4FFN":
        return cls(device)

    def forward(self, x, norm_weight, gate, up, down, out, m, hidden, inter, group_size,
                eps=1e-5, residual=False, h_out=None):
        ops.int4_ffn(self.device, x, norm_weight, gate, up, down, out, m, hidden, inter,
                     group_size, eps=eps, h_out=h_out, residual=residual)
