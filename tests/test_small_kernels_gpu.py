"""GPU parity of the small ops on the FFN path: RMSNorm (shaders.zig:16-56),
FusedRMSNormRoPE (shaders.zig:124-182) and FusedSiluMul (shaders.zig:344-357)."""
import numpy as np
import pytest

import oracle
from helpers import dev, host
from tiny_kernel import data, ops

pytestmark = pytest.mark.gpu

TOL = 1e-5  # f32 elementwise/reduction kernels vs f64, normwise


@pytest.mark.parametrize("rows,dim", [(1, 4096), (32, 4096), (3, 100)])
def test_rmsnorm(torch_cuda, tkdev, rows, dim):
    torch = torch_cuda
    x = data.make_x(1, "rn", rows, dim)
    w = data.make_norm_weight(1, "rnw", dim)
    out = torch.empty((rows, dim), dtype=torch.float32, device="cuda")
    ops.rmsnorm(tkdev, dev(torch, x), dev(torch, w), out, rows, dim, 1e-6)
    assert oracle.normwise_err(host(out), oracle.rmsnorm_f64(x, w, 1e-6)) <= TOL


@pytest.mark.parametrize("identity", [True, False])
def test_fused_rmsnorm_rope(torch_cuda, tkdev, identity):
    torch = torch_cuda
    rows, dim, head_dim, max_seq, pos = 2, 4096, 128, 64, 5
    x = data.make_x(2, "rr", rows, dim)
    w = data.make_norm_weight(2, "rrw", dim)
    half = head_dim // 2
    if identity:  # what src/bench.zig:310-311 passes
        c = np.ones(max_seq * half, np.float32)
        s = np.zeros(max_seq * half, np.float32)
    else:
        ang = np.outer(np.arange(max_seq), 1.0 / (10000 ** (np.arange(half) / half)))
        c = np.cos(ang).astype(np.float32).reshape(-1)
        s = np.sin(ang).astype(np.float32).reshape(-1)
    out = torch.empty((rows, dim), dtype=torch.float32, device="cuda")
    ops.fused_rmsnorm_rope(tkdev, dev(torch, x), dev(torch, w), dev(torch, c), dev(torch, s),
                           out, rows, dim, head_dim, pos, 1e-6)
    ref = oracle.fused_rmsnorm_rope_f64(x, w, c, s, head_dim, pos, 1e-6)
    assert oracle.normwise_err(host(out), ref) <= TOL
    if identity:
        plain = torch.empty_like(out)
        ops.rmsnorm(tkdev, dev(torch, x), dev(torch, w), plain, rows, dim, 1e-6)
        assert np.array_equal(host(plain), host(out))


def test_silu_mul(torch_cuda, tkdev):
    torch = torch_cuda
    n = 14336
    g = (data.make_x(3, "g", 1, n) * 4).reshape(-1)
    u = data.make_x(3, "u", 1, n).reshape(-1)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ops.silu_mul(tkdev, dev(torch, g), dev(torch, u), out, n)
    assert oracle.normwise_err(host(out), oracle.silu_mul_f64(g, u)) <= TOL


def test_mirror_api_fused(tkdev):
    import tiny_kernel as tk
    n = 1000
    g = data.make_x(4, "mg", 1, n).reshape(-1)
    u = data.make_x(4, "mu", 1, n).reshape(-1)
    bg = tkdev.create_buffer_with_data("f32", g)
    bu = tkdev.create_buffer_with_data("f32", u)
    bo = tkdev.create_buffer("f32", n)
    tk.kernels.fused.FusedSiluMul.init(tkdev).forward(bg, bu, bo)
    assert oracle.normwise_err(bo.slice(), oracle.silu_mul_f64(g, u)) <= TOL
