"""GPU check of tk_qmatmul_int4_noalloc, the allocation-free qmatmul_int4 entry point.

That entry point exists for callers that cannot call cudaMalloc (a process whose device
memory is pre-reserved by its own allocator, a loop that must not take cudaMalloc's
device-wide synchronisation, a binding that cannot own a tk_device): its scratch is one
static device array per GPU instead of buffers a device context allocates.  This test
calls it through the C ABI on several inputs in a row and checks each result against the
regular entry point tk_qmatmul_int4 on the same inputs, within the path's tolerance: config 0,
a smaller shape on the same scratch, row counts above 4 (several 4-row engine chunks sharing
one error word), and shapes the engine does not take (n not a multiple of 128, an x that is
not 16-byte aligned: the CUDA-core kernel, no scratch).  It also checks the size limit is
reported as an error.

The file name sorts last so that a run stopping at the first failure has already run every
other test; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from helpers import dev, host, mat_dev
from tiny_kernel import _lib, data, ops

pytestmark = pytest.mark.gpu

TOL = 1e-3  # normwise max relative error, the path's tolerance


def _noalloc(torch, x, w, s, z, out, m, k, n, gs):
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    return L.tk_qmatmul_int4_noalloc(x.data_ptr(), w.data_ptr(), s.data_ptr(), z.data_ptr(),
                                     out.data_ptr(), m, k, n, gs, C.c_void_p(stream))


def test_noalloc_matches_regular_entry_two_calls(torch_cuda, tkdev):
    torch = torch_cuda
    torch.cuda.synchronize()
    cases = [
        # m, K, N, gs, seed, x offset (floats): config 0 first, then a smaller shape on the
        # same scratch, then 2 and 3 engine chunks of <= 4 rows, then the CUDA-core kernel
        (1, 4096, 14336, 64, 31, 0),
        (2, 1024, 2048, 32, 32, 0),
        (5, 512, 1024, 64, 33, 0),
        (9, 256, 1024, 32, 34, 0),
        (3, 256, 200, 32, 35, 0),    # n % 128 != 0
        (2, 512, 256, 64, 36, 1),    # x not 16-byte aligned
    ]
    for m, K, N, gs, seed, off in cases:
        M = data.make_int4_matrix(seed, f"na{K}x{N}", K, N, gs)
        x = data.make_x(seed, f"nax{m}", m, K)
        xbuf = torch.zeros(m * K + off, dtype=torch.float32, device="cuda")
        xbuf[off:] = dev(torch, x).reshape(-1)
        xd = xbuf[off:]
        w, s, z = mat_dev(torch, M)
        ref_out = torch.empty((m, N), dtype=torch.float32, device="cuda")
        ops.qmatmul_int4(tkdev, xd, w, s, z, ref_out, m, K, N, gs)
        out = torch.full((m, N), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        st = _noalloc(torch, xd, w, s, z, out, m, K, N, gs)
        assert st == _lib.TK_OK, _lib.lib().tk_last_error_string()
        got, want = host(out), host(ref_out)
        assert np.isfinite(got).all()
        assert oracle.normwise_err(got, want) <= TOL
        ref64 = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
        assert oracle.normwise_err(got, ref64) <= TOL


def test_noalloc_rejects_shapes_beyond_its_scratch(torch_cuda):
    torch = torch_cuda
    m, K, N, gs = 4, 14336, 28672, 16  # records + partials far above 4 MiB
    x = torch.zeros((m, K), dtype=torch.float32, device="cuda")
    w = torch.zeros((K // 2, N), dtype=torch.uint8, device="cuda")
    s = torch.zeros((K // gs, N), dtype=torch.int16, device="cuda")
    z = torch.zeros((K // gs, N // 2), dtype=torch.uint8, device="cuda")
    out = torch.zeros((m, N), dtype=torch.float32, device="cuda")
    st = _noalloc(torch, x, w, s, z, out, m, K, N, gs)
    assert st == _lib.TK_ERR_ARG
    assert b"scratch" in _lib.lib().tk_last_error_string()
