"""GPU parity of the GGUF Q4_0 -> qmatmul_int4 repacker (tk_repack_q4_0).

The reference loads Q4_0 tensors by decoding them to f32 (src/model/llama.zig:341-353); the
repacker instead writes the INT4 layout of src/kernels/shaders.zig:442-501 (group 32, zero point
8, scale = the block's d), which dequantises to the same values exactly.  Checked: the repacked
arrays bit-exact against the oracle's restatement, both nibble orders, ragged column counts;
qmatmul_int4 on the repacked weights against the f64 product with the loader's f32 weights.
"""
import numpy as np
import pytest

import oracle
from helpers import host
from test_oracle_cpu import _q4_0_blocks
from tiny_kernel import _lib, data, ops

pytestmark = pytest.mark.gpu


def _repack(torch, tkdev, blocks, n_rows, k, order):
    b = torch.from_numpy(blocks).cuda()
    w = torch.empty((k // 2, n_rows), dtype=torch.uint8, device="cuda")
    s = torch.empty((k // 32, n_rows), dtype=torch.int16, device="cuda")
    z = torch.empty((k // 32, n_rows // 2), dtype=torch.uint8, device="cuda")
    ops.repack_q4_0(tkdev, b, w, s, z, n_rows, k, order)
    return w, s, z


@pytest.mark.parametrize("n_rows,k,order", [(4096, 4096, 0), (14336, 4096, 1), (130, 96, 0),
                                            (2, 32, 1)])
def test_repack_bit_exact(torch_cuda, tkdev, n_rows, k, order):
    blocks = _q4_0_blocks(n_rows + k + order, n_rows, k)
    w, s, z = _repack(torch_cuda, tkdev, blocks, n_rows, k, order)
    rw, rs, rz = oracle.q4_0_repack(blocks, n_rows, k, order)
    assert np.array_equal(host(w), rw)
    assert np.array_equal(host(s).view(np.uint16), rs)
    assert np.array_equal(host(z), rz)


@pytest.mark.parametrize("order", [0, 1])
def test_qmatmul_on_repacked_weights(torch_cuda, tkdev, order):
    torch = torch_cuda
    n_rows, k = 4096, 4096
    blocks = _q4_0_blocks(77 + order, n_rows, k)
    w, s, z = _repack(torch, tkdev, blocks, n_rows, k, order)
    x = data.make_x(78, "q40x", 1, k)
    out = torch.empty((1, n_rows), dtype=torch.float32, device="cuda")
    ops.qmatmul_int4(tkdev, torch.from_numpy(x).cuda(), w, s, z, out, 1, k, n_rows, 32)
    dense = oracle.q4_0_decode_f32(blocks, n_rows, k, order)
    ref = oracle.matvec_f64(x.reshape(-1), dense, k, n_rows)
    assert oracle.normwise_err(host(out).reshape(-1), ref) <= 1e-3


def test_repack_rejects_bad_shapes(torch_cuda, tkdev):
    L = _lib.lib()
    t = torch_cuda.zeros(64, dtype=torch_cuda.uint8, device="cuda")
    p = t.data_ptr()
    assert L.tk_repack_q4_0(tkdev.handle, p, p, p, p, 2, 48, 0) == _lib.TK_ERR_ARG   # k % 32
    assert L.tk_repack_q4_0(tkdev.handle, p, p, p, p, 3, 32, 0) == _lib.TK_ERR_ARG   # odd rows
    assert L.tk_repack_q4_0(tkdev.handle, p, p, p, p, 2, 32, 2) == _lib.TK_ERR_ARG   # order
    assert L.tk_repack_q4_0(tkdev.handle, None, p, p, p, 2, 32, 0) == _lib.TK_ERR_ARG
