"""GPU parity of the fp32 Matvec / MatvecDual (src/kernels/fused.zig:53-133, shaders.zig:184-266).

W is f32 row-major [N][K] (out_dim, in_dim).  The kernel sums in a different f32 order than the
shader's sequential loop; both are compared with the f64 oracle at normwise 2e-5 (f32 sums of
K terms), and small cases also with the shader's own sequential f32 order.  Shapes include the
reference model's projections (Q/O: dim x dim, K/V: kv_dim x dim, llama.zig:191-214), K above the
shader's 4096 limit, and ragged K (scalar path).
"""
import numpy as np
import pytest

import oracle
from helpers import host
from tiny_kernel import ops
from tiny_kernel.kernels.fused import Matvec, MatvecDual

pytestmark = pytest.mark.gpu

TOL = 2e-5


def _data(seed, K, N):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(K).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    return x, W


@pytest.mark.parametrize("K,N", [
    (4096, 4096),   # Q / O projections (dim x dim)
    (4096, 1024),   # K / V with grouped heads (kv_dim x dim)
    (14336, 4096),  # K above the shader's 4096-float staging limit
    (4097, 37),     # ragged K: scalar path
    (1, 1),
    (64, 3),
])
def test_matvec_vs_oracle(torch_cuda, tkdev, K, N):
    torch = torch_cuda
    x, W = _data(K * 7 + N, K, N)
    xd, Wd = torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda()
    out = torch.empty(N, dtype=torch.float32, device="cuda")
    Matvec.init(tkdev).forward(xd, Wd, out, K, N)
    y = host(out)
    assert oracle.normwise_err(y, oracle.matvec_f64(x, W, K, N)) <= TOL
    if K * N <= 4096:
        assert oracle.normwise_err(y, oracle.matvec_f32_sequential(x, W, K, N)) <= TOL


@pytest.mark.parametrize("K,N", [(4096, 4096), (2048, 4096), (130, 9)])
def test_matvec_dual_vs_oracle(torch_cuda, tkdev, K, N):
    torch = torch_cuda
    x, W1 = _data(K + N, K, N)
    _, W2 = _data(K + N + 1, K, N)
    xd = torch.from_numpy(x).cuda()
    W1d, W2d = torch.from_numpy(W1).cuda(), torch.from_numpy(W2).cuda()
    o1 = torch.empty(N, dtype=torch.float32, device="cuda")
    o2 = torch.empty(N, dtype=torch.float32, device="cuda")
    MatvecDual.init(tkdev).forward(xd, W1d, W2d, o1, o2, K, N)
    assert oracle.normwise_err(host(o1), oracle.matvec_f64(x, W1, K, N)) <= TOL
    assert oracle.normwise_err(host(o2), oracle.matvec_f64(x, W2, K, N)) <= TOL


def test_matvec_rejects_bad_arguments(torch_cuda, tkdev):
    from tiny_kernel import _lib
    L = _lib.lib()
    assert L.tk_matvec(tkdev.handle, None, None, None, 4, 4) == _lib.TK_ERR_ARG
    x = torch_cuda.zeros(4, device="cuda")
    assert L.tk_matvec(tkdev.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 4) == _lib.TK_ERR_ARG
    with pytest.raises(Exception):
        ops.matvec_dual(tkdev, x, x, None, x, None, 4, 1)
