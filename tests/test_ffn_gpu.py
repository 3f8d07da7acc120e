"""GPU parity of the INT4 Llama FFN (rmsnorm -> gate/up -> silu*up -> down [+ x]).

The reference composes norm, gate, up and silu*up in src/bench.zig:266-341; the down
projection and residual follow src/model/llama.zig:220-231.  Tolerance: normwise max
error 1e-3 against the f64 oracle (TOL), plus the precision the engine actually holds.
"""
import numpy as np
import pytest

import oracle
from helpers import dev, host, mat_dev
from tiny_kernel import data, ops

pytestmark = pytest.mark.gpu

TOL = 1e-3
# The engine's activation quantisation (x and h): int16 per group at 1-2 rows (2^-15 of each
# group's max |x|), int8 hi + lo/256 parts at 3-4 rows (2^-13).
PRECISION = 7e-4
GEMM_PRECISION = 8e-4  # the tcgen05 GEMM path (5+ rows)
EPS = 1e-5


def run_ffn(torch, tkdev, x, W, residual=False, inplace=False, want_h=True):
    xd = dev(torch, x)
    nw = dev(torch, W.norm_w)
    gate, up, down = (mat_dev(torch, M) for M in (W.gate, W.up, W.down))
    m = x.shape[0]
    out = xd if inplace else torch.empty((m, W.hidden), dtype=torch.float32, device="cuda")
    h = torch.empty((m, W.inter), dtype=torch.float32, device="cuda") if want_h else None
    ops.int4_ffn(tkdev, xd, nw, gate, up, down, out, m, W.hidden, W.inter, W.gs, eps=EPS,
                 h_out=h, residual=residual)
    return host(out), (host(h) if want_h else None)


@pytest.mark.parametrize("m,hidden,inter,gs", [
    (1, 4096, 14336, 64),     # config 1 (Llama-3-8B FFN, batch 1)
    (1, 256, 384, 64),
    (2, 512, 1024, 32),
    (3, 384, 256, 128),
    (4, 128, 128, 16),
    (6, 256, 512, 64),        # > 4 rows: the tcgen05 GEMM
])
def test_ffn_vs_oracle(torch_cuda, tkdev, m, hidden, inter, gs):
    W = data.make_ffn(21, hidden, inter, gs)
    x = data.make_x(22, f"ffnx{m}", m, hidden)
    y, h = run_ffn(torch_cuda, tkdev, x, W)
    ref, ref_h = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, return_h=True)
    eh, ey = oracle.normwise_err(h, ref_h), oracle.normwise_err(y, ref)
    assert eh <= TOL and ey <= TOL, (eh, ey)
    bar = GEMM_PRECISION if ops.ffn_path(m, hidden, inter, gs) == 2 else PRECISION
    assert eh <= bar and ey <= bar, (eh, ey)


def test_ffn_residual_and_inplace(torch_cuda, tkdev):
    W = data.make_ffn(31, 512, 768, 64)
    x = data.make_x(32, "resx", 2, 512)
    ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, residual=True)
    y, _ = run_ffn(torch_cuda, tkdev, x, W, residual=True)
    assert oracle.normwise_err(y, ref) <= PRECISION
    y2, _ = run_ffn(torch_cuda, tkdev, x, W, residual=True, inplace=True, want_h=False)
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))


def test_ffn_bench_zero_point(torch_cuda, tkdev):
    W = data.make_ffn(41, 1024, 2048, 64, zeros="eight")
    x = data.make_x(42, "z8x", 1, 1024)
    y, _ = run_ffn(torch_cuda, tkdev, x, W)
    ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS)
    assert oracle.normwise_err(y, ref) <= PRECISION


def test_ffn_fallback_shape(torch_cuda, tkdev):
    """hidden/inter not multiples of 128: the CUDA-core composition."""
    W = data.make_ffn(51, 192, 320, 32)
    x = data.make_x(52, "fbx", 2, 192)
    y, h = run_ffn(torch_cuda, tkdev, x, W)
    ref, ref_h = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, return_h=True)
    assert oracle.normwise_err(y, ref) <= PRECISION
    assert oracle.normwise_err(h, ref_h) <= PRECISION


def test_ffn_deterministic(torch_cuda, tkdev):
    W = data.make_ffn(61, 4096, 14336, 64)
    x = data.make_x(62, "detx", 1, 4096)
    a, _ = run_ffn(torch_cuda, tkdev, x, W, want_h=False)
    b, _ = run_ffn(torch_cuda, tkdev, x, W, want_h=False)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("m,hidden,inter,gs,residual", [
    (1, 4096, 14336, 64, False),   # config 1: the decode kernel reads / writes host memory itself
    (2, 4096, 14336, 64, True),    # residual from the kernel's own copy of x
    (1, 512, 1024, 64, True),
    (2, 256, 512, 32, True),
    (3, 384, 256, 128, False),     # the decode kernel at three rows (four-row instantiation)
    (16, 512, 1024, 64, True),     # the tcgen05 GEMM: staged
])
def test_ffn_host_io_matches_device_buffers(torch_cuda, tkdev, m, hidden, inter, gs, residual):
    """TK_FFN_HOST_IO: x and out in pinned host memory give the same bits as device buffers, on
    the first call (run directly, then recorded as a graph) and on three repeats with new
    contents in the same buffers (replays of the recorded graph)."""
    import tiny_kernel as tk
    torch = torch_cuda
    W = data.make_ffn(91, hidden, inter, gs)
    xb = tk.Buffer(tkdev, "f32", m * hidden, kind=2)
    ob = tk.Buffer(tkdev, "f32", m * hidden, kind=2)
    gate, up, down = (mat_dev(torch, M) for M in (W.gate, W.up, W.down))
    nw = dev(torch, W.norm_w)
    for call in range(4):
        x = data.make_x(92 + call, f"hio{m}", m, hidden)
        y_dev, _ = run_ffn(torch, tkdev, x, W, residual=residual, want_h=False)
        xb.slice()[:] = x.reshape(-1)
        ob.slice()[:] = np.nan
        ops.int4_ffn(tkdev, xb, nw, gate, up, down, ob, m, hidden, inter, gs, eps=EPS,
                     residual=residual, host_io=True)
        y_host = ob.slice().reshape(m, hidden).copy()
        assert np.array_equal(y_host.view(np.uint32), y_dev.view(np.uint32)), call
        ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, residual=residual)
        assert oracle.normwise_err(y_host, ref) <= TOL
    xb.deinit()
    ob.deinit()
