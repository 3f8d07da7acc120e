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


@pytest.mark.parametrize("nbytes", [0, 4, 4096 + 12, 1 << 20])
def test_async_buffer_copies_round_trip(torch_cuda, tkdev, nbytes):
    """tk_buffer_upload_async / tk_buffer_download_async: bytes queued on the device's stream
    (NULL) and on a caller's stream come back unchanged after one wait."""
    import ctypes as C

    import tiny_kernel as tk
    from tiny_kernel import _lib
    L = _lib.lib()
    torch = torch_cuda
    src = np.random.default_rng(nbytes).integers(0, 256, size=max(nbytes, 1), dtype=np.uint8)
    hin = tk.Buffer(tkdev, "u8", max(nbytes, 1), kind=_lib.TK_MEM_HOST)
    hout = tk.Buffer(tkdev, "u8", max(nbytes, 1), kind=_lib.TK_MEM_HOST)
    view_in = np.frombuffer((C.c_char * hin.nbytes).from_address(hin.ptr), np.uint8)
    view_out = np.frombuffer((C.c_char * hout.nbytes).from_address(hout.ptr), np.uint8)
    view_in[:] = src
    d = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    side = torch.cuda.Stream()
    try:
        for stream in (None, side.cuda_stream):
            view_out[:] = 0
            _lib.check(L.tk_buffer_upload_async(tkdev.handle, d.data_ptr(), hin.ptr, nbytes, stream))
            _lib.check(L.tk_buffer_download_async(tkdev.handle, hout.ptr, d.data_ptr(), nbytes,
                                                  stream))
            if stream is None:
                _lib.check(L.tk_device_synchronize(tkdev.handle))
            else:
                side.synchronize()
            assert np.array_equal(view_out[:nbytes], src[:nbytes])
    finally:
        hin.deinit()
        hout.deinit()
