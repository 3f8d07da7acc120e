"""Within-group dynamic range: qmatmul_int4 (src/kernels/shaders.zig:442-501) on activations whose
groups mix values near 1e3 with values near 1e-3, on every path (decode kernel at 1, 2 and 4 rows,
the streaming engine at 4 rows (TK_DECODE=0), tcgen05 GEMM at 16).

The reference computes in f32 (shaders.zig:481-497), so each of its output columns carries f32
relative precision whatever the spread inside a group.  The paths here quantise activations per
weight group:
  decode    int16 with one power-of-two scale per group (max |x| * 2^e in [2^14, 2^15)):
            |x - x^| <= 2^-14 max|x_g|
  engine    int8 hi + lo/256 parts at a scale with max |x| * 2^e in [32, 64):
            |x - x^| <= 2^-13 max|x_g|
  GEMM      f16 activations and f16 dequantised weights, f32 accumulation: per product
            <= 2^-10 relative
followed by exact int32 sums (decode, engine) and f32 scaling.  So an output column carried only
by a group's small values is exact to the group's fixed point on the decode kernel and the engine
-- its error is bounded by the group maximum, not by the column's own size -- and to f16
precision on the GEMM.  The test
builds exactly that case and asserts, column by column:
  * every path: the componentwise bound of its arithmetic above;
  * every path: columns carried by the large values within 1e-3 relative;
  * the GEMM path: columns carried only by the small values within 2e-3 relative;
  * every path: the normwise contract (1e-3).
The relative error of the small-value columns of the fixed-point paths is printed (it is the loss the
fixed-point groups make on this adversarial case).
"""
import numpy as np
import pytest

import oracle
from helpers import dev, host, mat_dev
from tiny_kernel import data, ops

pytestmark = pytest.mark.gpu

TOL = 1e-3
K, N, GS = 2048, 2048, 64
BOUND_C = {3: 2.0 ** -14, 1: 2.0 ** -13}  # fixed-point paths: error per unit of group max
GEMM_REL = 2.0 ** -9                      # the GEMM's componentwise relative bound


def _pack(q):
    """codes q [K][N] (0..15) -> packed u8 [K/2][N], even k in the low nibble."""
    return (q[0::2] | (q[1::2] << 4)).astype(np.uint8)


def _case(seed, m):
    """x [m][K] with a fixed half of every group's positions small (1e-3) and the rest large
    (1e3), all positive; columns of three kinds: small-only (codes equal the zero point on the
    large positions, above it on the small ones), large-only (the reverse) and mixed."""
    rng = np.random.default_rng(seed)
    G = K // GS
    small = np.zeros(K, dtype=bool)
    for g in range(G):
        small[g * GS + rng.choice(GS, GS // 2, replace=False)] = True
    x = np.where(small, 1e-3 * rng.uniform(0.5, 1.5, (m, K)),
                 1e3 * rng.uniform(0.5, 1.0, (m, K))).astype(np.float32)
    kind = np.arange(N) % 3  # 0 small-only, 1 large-only, 2 mixed
    z = np.full((G, N), 8, dtype=np.uint8)
    z[:, kind == 2] = rng.integers(0, 16, (G, int((kind == 2).sum())))
    q = rng.integers(0, 16, (K, N)).astype(np.uint8)
    zk = np.repeat(z, GS, axis=0)  # zero point of every k
    above = rng.integers(9, 16, (K, N)).astype(np.uint8)
    q = np.where((kind == 0)[None, :] & small[:, None], above, q)
    q = np.where((kind == 0)[None, :] & ~small[:, None], zk, q)
    q = np.where((kind == 1)[None, :] & ~small[:, None], above, q)
    q = np.where((kind == 1)[None, :] & small[:, None], zk, q)
    s = data.f16_uniform(seed + 7, G * N, 0.005, 0.02).reshape(G, N)
    zp = (z[:, 0::2] | (z[:, 1::2] << 4)).astype(np.uint8)
    M = data.Int4Matrix(_pack(q), s, zp, K, N, GS)
    return x, M, kind


@pytest.mark.parametrize("m,engine", [(1, False), (2, False), (4, False), (4, True), (16, False)])
def test_within_group_dynamic_range(torch_cuda, tkdev, tkdev_engine, m, engine):
    torch = torch_cuda
    x, M, kind = _case(41 + m, m)
    if engine:
        tkdev, path = tkdev_engine, 1
    else:
        path = ops.path(m, K, N, GS)
        assert path == {1: 3, 2: 3, 4: 3, 16: 2}[m], path
    w, s, z = mat_dev(torch, M)
    out = torch.empty((m, N), dtype=torch.float32, device="cuda")
    ops.qmatmul_int4(tkdev, dev(torch, x), w, s, z, out, m, K, N, GS)
    y = host(out).astype(np.float64)
    ref = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, GS)
    W = oracle.dequant_f32(M.w, M.s, M.z, K, N, GS).astype(np.float64)  # exact f16 products
    ax = np.abs(x.astype(np.float64))
    err = np.abs(y - ref)
    absdot = ax @ np.abs(W)  # sum_k |x_k| |w_kj|
    if path == 2:
        bound = GEMM_REL * absdot
    else:
        gmax = ax.reshape(m, K // GS, GS).max(axis=2)                 # [m][G]
        wsum = np.abs(W).reshape(K // GS, GS, N).sum(axis=1)          # [G][N]
        sc = M.s.view(np.float16).astype(np.float64)                 # [G][N]
        # group fixed point, plus the f32 conversion of each group's exact integer sum and the
        # scale products
        bound = BOUND_C[path] * (gmax @ wsum) + 2.0 ** -18 * (gmax @ (GS * sc))
    assert np.all(err <= bound), (m, float((err / bound).max()))
    rel = err / np.abs(ref)
    print(f"m={m} path {path}: rel err small-only cols max {rel[:, kind == 0].max():.2e}, "
          f"large-only max {rel[:, kind == 1].max():.2e}, "
          f"normwise {oracle.normwise_err(y, ref):.2e}, worst err/bound {(err / bound).max():.2f}")
    assert rel[:, kind == 1].max() <= TOL
    if path == 2:
        assert rel[:, kind == 0].max() <= 2e-3
    assert oracle.normwise_err(y, ref) <= TOL
