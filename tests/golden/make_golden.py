"""Regenerates the golden fixtures of this directory (run from anywhere):

    python tests/golden/make_golden.py

The reference (Zig + Metal) holds no golden vectors and cannot run on Linux, so these
fixtures are produced by the f64 oracle (oracle/oracle.py) on seeded inputs from
tiny_kernel.data.  They pin the oracle and the generators against silent change, and give
the GPU tests small fixed cases.  One fixture, `kat_bench.npz`, is the known answer the
reference's own bench constants imply (src/bench.zig:242-245).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "tiny-kernel_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402
from tiny_kernel import data  # noqa: E402

SEED = 4242


def qmatmul_case(name, m, K, N, gs, zeros="random"):
    M = data.make_int4_matrix(SEED, name, K, N, gs, zeros)
    x = data.make_x(SEED, name + "/x", m, K)
    y = oracle.qmatmul_f64(x, M.w, M.s, M.z, K, N, gs)
    extra = {}
    if K * N <= 1 << 16:  # the f32 dequantised matrix only for the small cases
        extra["dequant"] = oracle.dequant_f32(M.w, M.s, M.z, K, N, gs)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), x=x, w=M.w, s=M.s, z=M.z, y=y,
                        shape=np.array([m, K, N, gs]), **extra)


def ffn_case(name, m, hidden, inter, gs, residual):
    W = data.make_ffn(SEED, hidden, inter, gs, layer=0)
    x = data.make_x(SEED, name + "/x", m, hidden)
    y, h = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, 1e-5, residual=residual,
                          return_h=True)
    arrs = {"x": x, "norm_w": W.norm_w, "y": y, "h": h,
            "shape": np.array([m, hidden, inter, gs, int(residual)])}
    for nm, M in (("gate", W.gate), ("up", W.up), ("down", W.down)):
        arrs[nm + "_w"], arrs[nm + "_s"], arrs[nm + "_z"] = M.w, M.s, M.z
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)


def small_ops_case():
    x = data.make_x(SEED, "ops/x", 3, 256)
    w = data.make_norm_weight(SEED, "ops/w", 256)
    head_dim, pos, max_seq = 64, 3, 8
    ang = (np.arange(max_seq)[:, None] * 10000.0 ** (-np.arange(head_dim // 2) * 2.0 / head_dim))
    cosc = np.cos(ang).astype(np.float32).reshape(-1)
    sinc = np.sin(ang).astype(np.float32).reshape(-1)
    g = data.make_x(SEED, "ops/g", 1, 1000).reshape(-1) * 4.0
    u = data.make_x(SEED, "ops/u", 1, 1000).reshape(-1)
    np.savez_compressed(
        os.path.join(HERE, "small_ops.npz"), x=x, w=w, cos=cosc, sin=sinc, g=g, u=u,
        rmsnorm=oracle.rmsnorm_f64(x, w, 1e-5),
        rope=oracle.fused_rmsnorm_rope_f64(x, w, cosc, sinc, head_dim, pos, 1e-5),
        silu_mul=oracle.silu_mul_f64(g, u), meta=np.array([head_dim, pos, max_seq]))


def kat_case():
    # src/bench.zig:242-245: x = 0.1, packed bytes 0x77 (q = 7), scales f16(0.01), zeros 0x88
    K, N, gs = 4096, 256, 64
    x = np.full((1, K), 0.1, dtype=np.float32)
    w = np.full((K // 2, N), 0x77, dtype=np.uint8)
    s = np.full((K // gs, N), np.float16(0.01).view(np.uint16), dtype=np.uint16)
    z = np.full((K // gs, N // 2), 0x88, dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "kat_bench.npz"), x=x, w=w, s=s, z=z,
                        y=np.full((1, N), oracle.kat_bench_constants()),
                        shape=np.array([1, K, N, gs]))


def main():
    qmatmul_case("qmatmul_m2_k256_n128_g64", 2, 256, 128, 64)
    qmatmul_case("qmatmul_m1_k512_n256_g32", 1, 512, 256, 32)
    qmatmul_case("qmatmul_m3_k128_n130_g16", 3, 128, 130, 16)       # n not a multiple of 128
    qmatmul_case("qmatmul_m1_k256_n128_g64_z8", 1, 256, 128, 64, zeros="eight")
    ffn_case("ffn_m1_h256_i512_g64", 1, 256, 512, 64, residual=False)
    ffn_case("ffn_m2_h256_i384_g32_res", 2, 256, 384, 32, residual=True)
    small_ops_case()
    kat_case()


if __name__ == "__main__":
    main()
