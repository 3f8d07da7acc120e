"""GPU parity of the batch >= 5 path: the tcgen05 INT4 GEMM (qmatmul_int4 and the FFN).

From 5 rows on, qmatmul_int4 (src/kernels/shaders.zig:442-501) and the INT4 FFN
(src/bench.zig:266-341 + the down projection and residual of src/model/llama.zig:220-231)
run as GEMMs on the 5th-generation tensor cores: weights dequantised to f16 in shared memory,
activations (and the FFN's h) in f16, f32 accumulation.  Bar: the path's normwise max error
1e-3 against the f64 oracle; the f16 rounding of x, of the dequantised weights and of h holds
well inside it (GEMM_PRECISION).  Results are bit-identical run to run (fixed reduction
order, including the split-K reduction).
"""
import numpy as np
import pytest

import oracle
from helpers import dev, host, mat_dev
from tiny_kernel import data, ops

pytestmark = pytest.mark.gpu

TOL = 1e-3
GEMM_PRECISION = 8e-4
EPS = 1e-5


def run_qmatmul(torch, tkdev, x, M):
    xd = dev(torch, x)
    w, s, z = mat_dev(torch, M)
    out = torch.empty((x.shape[0], M.N), dtype=torch.float32, device="cuda")
    ops.qmatmul_int4(tkdev, xd, w, s, z, out, x.shape[0], M.K, M.N, M.gs)
    return host(out)


@pytest.mark.parametrize("m,K,N,gs", [
    (16, 512, 256, 64),
    (16, 4096, 14336, 64),    # config 0 shape at batch 16 (config 2)
    (40, 1024, 512, 32),      # a ragged token tile
    (128, 256, 768, 128),
    (300, 512, 512, 16),      # two token tiles of 256
    (24, 1024, 512, 32),      # a ragged token tile of 32
])
def test_gemm_qmatmul_vs_oracle(torch_cuda, tkdev, m, K, N, gs):
    assert ops.path(m, K, N, gs) == 2
    M = data.make_int4_matrix(51, f"gm{K}x{N}", K, N, gs)
    x = data.make_x(52, f"gmx{m}", m, K)
    y = run_qmatmul(torch_cuda, tkdev, x, M)
    ref = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
    e = oracle.normwise_err(y, ref)
    assert e <= TOL and e <= GEMM_PRECISION, e


def run_ffn(torch, tkdev, x, W, residual=False):
    xd = dev(torch, x)
    m = x.shape[0]
    out = torch.empty((m, W.hidden), dtype=torch.float32, device="cuda")
    h = torch.empty((m, W.inter), dtype=torch.float32, device="cuda")
    ops.int4_ffn(tkdev, xd, dev(torch, W.norm_w), mat_dev(torch, W.gate), mat_dev(torch, W.up),
                 mat_dev(torch, W.down), out, m, W.hidden, W.inter, W.gs, eps=EPS, h_out=h,
                 residual=residual)
    return host(out), host(h)


@pytest.mark.parametrize("m,hidden,inter,gs,residual", [
    (16, 512, 1024, 64, False),
    (16, 4096, 14336, 64, False),   # config 2 at batch 16
    (64, 1024, 2048, 32, True),
    (256, 512, 768, 64, False),
])
def test_gemm_ffn_vs_oracle(torch_cuda, tkdev, m, hidden, inter, gs, residual):
    assert ops.ffn_path(m, hidden, inter, gs) == 2
    W = data.make_ffn(61, hidden, inter, gs)
    x = data.make_x(62, f"gfx{m}", m, hidden)
    y, h = run_ffn(torch_cuda, tkdev, x, W, residual)
    ref, ref_h = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, residual=residual,
                                return_h=True)
    eh, ey = oracle.normwise_err(h, ref_h), oracle.normwise_err(y, ref)
    assert eh <= TOL and ey <= TOL, (eh, ey)
    assert eh <= GEMM_PRECISION and ey <= GEMM_PRECISION, (eh, ey)


def test_gemm_deterministic(torch_cuda, tkdev):
    W = data.make_ffn(71, 1024, 2048, 64)
    x = data.make_x(72, "gdet", 32, 1024)
    a, _ = run_ffn(torch_cuda, tkdev, x, W)
    b, _ = run_ffn(torch_cuda, tkdev, x, W)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
