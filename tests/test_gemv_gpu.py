"""GPU parity of qmatmul_int4 (src/kernels/shaders.zig:442-501) through the C ABI.

Bars: dequantisation bit-exact in f32; the CUDA-core fallback bit-exact against the
reference's f32 accumulation order; the tensor-core engine within the path's tolerance
(normwise max error 1e-3 against the f64 oracle, written below as TOL).
"""
import numpy as np
import pytest

import oracle
from helpers import dev, host, mat_dev
from tiny_kernel import data, ops
from tiny_kernel._lib import TK_ERR_ARG, TKError

pytestmark = pytest.mark.gpu

TOL = 1e-3          # normwise max relative error vs f64 (the path's contract)
# What the streaming engine's activation quantisation holds: int16 per group (one power-of-two
# scale, dp2a, exact int32 sums) at 1-2 rows, about 2e-5; int8 hi + lo/256 parts (int8 tensor-core
# MMAs, exact int32 sums) at 3-4 rows, about 1e-4.
PRECISION = 5e-4
GEMM_PRECISION = 8e-4  # the tcgen05 GEMM path (5+ rows): f16 activations and dequantised weights


def f32_reference_order(x, M):
    """The reference shader's arithmetic (shaders.zig:481-497) in numpy f32:
    acc += (x[k] * scale) * (q - zero), k ascending, no FMA."""
    K, N, gs = M.K, M.N, M.gs
    x = np.asarray(x, dtype=np.float32).reshape(-1, K)
    q = oracle.unpack_codes(M.w, K, N).astype(np.float32)
    zz = oracle.unpack_zeros(M.z, K // gs, N).astype(np.float32)
    sc = M.s.view(np.float16).astype(np.float32)
    out = np.zeros((x.shape[0], N), dtype=np.float32)
    for r in range(x.shape[0]):
        acc = np.zeros(N, dtype=np.float32)
        for k in range(K):
            g = k // gs
            t = (np.float32(x[r, k]) * sc[g]).astype(np.float32)
            acc = (acc + t * (q[k] - zz[g])).astype(np.float32)
        out[r] = acc
    return out


def run_qmatmul(torch, tkdev, x, M):
    xd = dev(torch, x)
    w, s, z = mat_dev(torch, M)
    out = torch.empty((x.shape[0], M.N), dtype=torch.float32, device="cuda")
    ops.qmatmul_int4(tkdev, xd, w, s, z, out, x.shape[0], M.K, M.N, M.gs)
    return host(out)


@pytest.mark.parametrize("K,N,gs", [(256, 384, 64), (512, 256, 32), (128, 512, 128), (64, 130, 8)])
def test_dequant_bit_exact(torch_cuda, tkdev, K, N, gs):
    torch = torch_cuda
    M = data.make_int4_matrix(11, f"dq{K}x{N}", K, N, gs)
    w, s, z = mat_dev(torch, M)
    out = torch.empty((K, N), dtype=torch.float32, device="cuda")
    ops.dequant_int4(tkdev, w, s, z, out, K, N, gs)
    ref = oracle.dequant_f32(M.w, M.s, M.z, K, N, gs)
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))


ENGINE_CASES = [
    # m, K, N, gs
    (1, 256, 128, 64),
    (1, 4096, 14336, 64),     # config 0: y[1,14336] = x[1,4096] . W^T
    (1, 14336, 4096, 64),     # the FFN down-projection shape
    (2, 512, 256, 32),
    (3, 1024, 384, 128),
    (4, 768, 640, 16),
    (5, 512, 256, 64),        # > 4 rows: processed in chunks of 4
    (8, 256, 1024, 64),
    (1, 128, 128, 16),
]


@pytest.mark.parametrize("m,K,N,gs", ENGINE_CASES)
def test_qmatmul_engine_vs_oracle(torch_cuda, tkdev, m, K, N, gs):
    path = ops.path(m, K, N, gs)
    assert path in (1, 3) if m <= 4 else path in (1, 2), path
    M = data.make_int4_matrix(1000 + m, f"q{K}x{N}", K, N, gs)
    x = data.make_x(7, f"x{m}x{K}", m, K)
    y = run_qmatmul(torch_cuda, tkdev, x, M)
    ref = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
    err = oracle.normwise_err(y, ref)
    assert err <= TOL, err
    assert err <= (GEMM_PRECISION if path == 2 else PRECISION), err


@pytest.mark.parametrize("m,K,N,gs", [(1, 40, 10, 8), (2, 192, 94, 24), (1, 96, 256, 48),
                                      (3, 256, 200, 64)])
def test_qmatmul_fallback_bit_exact(torch_cuda, tkdev, m, K, N, gs):
    assert ops.path(m, K, N, gs) == 0
    M = data.make_int4_matrix(77, f"f{K}x{N}", K, N, gs)
    x = data.make_x(8, f"fx{m}", m, K)
    y = run_qmatmul(torch_cuda, tkdev, x, M)
    ref = f32_reference_order(x, M)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("K,N", [(4096, 14336), (4096, 256)])
def test_known_answer_bench_constants(torch_cuda, tkdev, K, N):
    """src/bench.zig:242-245: x=0.1, bytes 0x77, scale f16(0.01), zero bytes 0x88."""
    gs = 64
    M = data.Int4Matrix(np.full((K // 2, N), 0x77, np.uint8),
                        np.full((K // gs, N), np.float16(0.01).view(np.uint16), np.uint16),
                        np.full((K // gs, N // 2), 0x88, np.uint8), K, N, gs)
    x = np.full((1, K), 0.1, np.float32)
    y = run_qmatmul(torch_cuda, tkdev, x, M)
    kat = oracle.kat_bench_constants()
    assert abs(kat - (-4.096875)) < 1e-6
    # one row: the engine quantises x to int16 per group (0.1 -> 26214 * 2^-18), about 1.5e-5
    # relative
    assert np.all(np.abs(y - kat) <= 1e-4 * abs(kat)), (y.min(), y.max(), kat)


def test_engine_deterministic(torch_cuda, tkdev):
    torch = torch_cuda
    M = data.make_int4_matrix(5, "det", 4096, 14336, 64)
    x = data.make_x(5, "detx", 1, 4096)
    xd = dev(torch, x)
    w, s, z = mat_dev(torch, M)
    outs = []
    for _ in range(3):
        out = torch.empty((1, 14336), dtype=torch.float32, device="cuda")
        ops.qmatmul_int4(tkdev, xd, w, s, z, out, 1, 4096, 14336, 64)
        outs.append(host(out).view(np.uint32).copy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_zero_point_eight_and_extreme_inputs(torch_cuda, tkdev):
    """Bench-style zero point 8; x with a 1e4 spike and exact zeros (per-group scaling)."""
    K, N, gs = 1024, 512, 64
    M = data.make_int4_matrix(9, "z8", K, N, gs, zeros="eight")
    x = data.make_x(9, "z8x", 2, K)
    x[0, 5] = 1.0e4
    x[1, :128] = 0.0
    y = run_qmatmul(torch_cuda, tkdev, x, M)
    ref = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
    assert oracle.normwise_err(y, ref) <= PRECISION


def test_mirror_api_buffers(tkdev):
    """QMatMulInt4.init/forward with managed Buffers, as quantized.zig is used."""
    import tiny_kernel as tk
    K, N, gs = 512, 256, 64
    M = data.make_int4_matrix(3, "mirror", K, N, gs)
    x = data.make_x(3, "mirrorx", 1, K)
    bx = tkdev.create_buffer_with_data("f32", x)
    bw = tkdev.create_buffer_with_data("u8", M.w)
    bs = tkdev.create_buffer_with_data("u16", M.s)
    bz = tkdev.create_buffer_with_data("u8", M.z)
    bo = tkdev.create_buffer("f32", N)
    q = tk.kernels.quantized.QMatMulInt4.init(tkdev)
    q.forward(bx, bw, bs, bz, bo, 1, K, N, gs)
    ref = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
    assert oracle.normwise_err(bo.slice(), ref) <= PRECISION
    for b in (bx, bw, bs, bz, bo):
        b.deinit()


@pytest.mark.parametrize("m,k,n,gs", [(1, 64, 31, 8), (1, 60, 32, 8), (1, 64, 32, 12),
                                      (0, 64, 32, 8)])
def test_invalid_shapes_rejected(torch_cuda, tkdev, m, k, n, gs):
    torch = torch_cuda
    buf = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    with pytest.raises(TKError) as ei:
        ops.qmatmul_int4(tkdev, buf, buf, buf, buf, buf, m, k, n, gs)
    assert ei.value.status == TK_ERR_ARG
