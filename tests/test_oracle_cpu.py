"""CPU checks of the checker itself (no GPU): the f64 oracle against the known answer of
the reference's bench constants and against the committed golden fixtures, the C++
std::thread transcription of the shaders against the oracle, and the seeded generators.

The reference (Zig + Metal, no numerical tests) cannot run here, so the oracle is pinned
only by the bench-constant known answer (src/bench.zig:242-245); the fixtures guard the
oracle and the generators against silent change.
"""
import glob
import os

import numpy as np
import pytest

import cpu
import oracle
from tiny_kernel import data
from tiny_kernel.data import Int4Matrix

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def test_kat_bench_constants_f64():
    # 4096 * 0.1 * f16(0.01) * (7 - 8), with x stored as f32 as the reference does
    assert oracle.kat_bench_constants() == pytest.approx(-4.096875, abs=1e-6)
    f = _load("kat_bench")
    m, K, N, gs = f["shape"]
    y = oracle.qmatmul_f64(f["x"], f["w"], f["s"], f["z"], K, N, gs)
    assert np.allclose(y, oracle.kat_bench_constants(), rtol=0, atol=1e-12)


def test_kat_bench_constants_shader_order_f32():
    # The shader accumulates x*scale*(q-z) over k in f32 (shaders.zig:488-495):
    # the C++ transcription reproduces that order; the survey derived -4.096759.
    f = _load("kat_bench")
    m, K, N, gs = (int(v) for v in f["shape"])
    M = Int4Matrix(f["w"], f["s"], f["z"], K, N, gs)
    y = cpu.qmatmul_int4(f["x"], M, threads=2)
    assert np.all(y == y[0, 0])
    assert float(y[0, 0]) == pytest.approx(-4.096759, abs=2e-6)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "qmatmul_*.npz"))))
def test_golden_qmatmul(path):
    f = np.load(path)
    m, K, N, gs = (int(v) for v in f["shape"])
    y = oracle.qmatmul_f64(f["x"], f["w"], f["s"], f["z"], K, N, gs)
    assert np.array_equal(y, f["y"])
    if "dequant" in f:
        deq = oracle.dequant_f32(f["w"], f["s"], f["z"], K, N, gs)
        assert np.array_equal(deq.view(np.uint32), f["dequant"].view(np.uint32))
    # the C++ transcription (f32, shader order) stays within the path tolerance
    yc = cpu.qmatmul_int4(f["x"], Int4Matrix(f["w"], f["s"], f["z"], K, N, gs), threads=2)
    assert oracle.normwise_err(yc, f["y"]) <= 1e-5


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "ffn_*.npz"))))
def test_golden_ffn(path):
    f = np.load(path)
    m, hidden, inter, gs, residual = (int(v) for v in f["shape"])
    mats = [Int4Matrix(f[n + "_w"], f[n + "_s"], f[n + "_z"], K, N, gs)
            for n, K, N in (("gate", hidden, inter), ("up", hidden, inter), ("down", inter, hidden))]
    y, h = oracle.ffn_f64(f["x"], f["norm_w"], *mats, 1e-5, residual=bool(residual), return_h=True)
    assert np.array_equal(y, f["y"]) and np.array_equal(h, f["h"])
    W = data.FFNWeights(f["norm_w"], *mats, hidden, inter, gs)
    yc = cpu.FFNRunner(W, m, 1e-5, residual=bool(residual), threads=2)(f["x"])
    assert oracle.normwise_err(yc, f["y"]) <= 1e-5


def test_golden_small_ops():
    f = _load("small_ops")
    head_dim, pos, _ = (int(v) for v in f["meta"])
    assert np.array_equal(oracle.rmsnorm_f64(f["x"], f["w"], 1e-5), f["rmsnorm"])
    assert np.array_equal(
        oracle.fused_rmsnorm_rope_f64(f["x"], f["w"], f["cos"], f["sin"], head_dim, pos, 1e-5),
        f["rope"])
    assert np.array_equal(oracle.silu_mul_f64(f["g"], f["u"]), f["silu_mul"])


def test_generators_are_reproducible_and_distributed():
    M = data.make_int4_matrix(7, "t", 256, 128, 64)
    M2 = data.make_int4_matrix(7, "t", 256, 128, 64)
    assert np.array_equal(M.w, M2.w) and np.array_equal(M.s, M2.s) and np.array_equal(M.z, M2.z)
    s = M.s.view(np.float16).astype(np.float64)
    assert s.min() >= 0.005 - 1e-5 and s.max() <= 0.02 + 1e-5
    q = oracle.unpack_codes(M.w, 256, 128)
    assert q.min() == 0 and q.max() == 15
    x = data.make_x(7, "x", 1, 1 << 16)
    assert abs(float(x.mean())) < 0.02 and abs(float(x.std()) - 1.0) < 0.02
    z8 = data.make_int4_matrix(7, "t8", 128, 64, 64, zeros="eight")
    assert np.all(oracle.unpack_zeros(z8.z, 2, 64) == 8)


def test_unpack_layout_matches_reference_indexing():
    # byte (k/2)*N + n, even k = low nibble (shaders.zig:479-495); zeros byte g*(N/2)+n/2,
    # even n = low nibble (shaders.zig:467-468)
    K, N = 4, 4
    w = np.array([[0x21, 0x43, 0x65, 0x87], [0xA9, 0xCB, 0xED, 0x0F]], dtype=np.uint8)
    q = oracle.unpack_codes(w, K, N)
    assert q[0].tolist() == [1, 3, 5, 7] and q[1].tolist() == [2, 4, 6, 8]
    assert q[2].tolist() == [9, 11, 13, 15] and q[3].tolist() == [10, 12, 14, 0]
    z = oracle.unpack_zeros(np.array([[0x21, 0x43]], dtype=np.uint8), 1, 4)
    assert z[0].tolist() == [1, 2, 3, 4]


def test_oracle_catches_a_planted_layout_mistake():
    # a checker that swapped the nibble order would be blind; make sure it is not
    M = data.make_int4_matrix(3, "plant", 128, 64, 32)
    x = data.make_x(3, "plantx", 1, 128)
    good = oracle.qmatmul_f64(x, M.w, M.s, M.z, 128, 64, 32)
    swapped = ((M.w >> 4) | (M.w << 4)).astype(np.uint8)
    bad = oracle.qmatmul_f64(x, swapped, M.s, M.z, 128, 64, 32)
    assert oracle.normwise_err(bad, good) > 1e-2


def test_matvec_oracle_matches_shader_order():
    """The f64 Matvec oracle against the shader's own sequential f32 loop (shaders.zig:211-215)
    on a small case: the two differ only by f32 rounding."""
    rng = np.random.default_rng(5)
    K, N = 33, 7
    x = rng.standard_normal(K).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32)
    y64 = oracle.matvec_f64(x, W, K, N)
    y32 = oracle.matvec_f32_sequential(x, W, K, N)
    assert np.allclose(y64, W.astype(np.float64) @ x.astype(np.float64))
    assert oracle.normwise_err(y32, y64) < 1e-6


def _q4_0_blocks(seed, n_rows, k):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n_rows, k // 32, 18), dtype=np.uint8)
    d = (rng.uniform(0.005, 0.02, size=(n_rows, k // 32))).astype(np.float16)
    b[:, :, 0:2] = d.view(np.uint8).reshape(n_rows, k // 32, 2)
    return b.reshape(-1)


def test_q4_0_known_answer():
    """One block, d = 0.5, qs[i] = (2i+1) << 4 | 2i mod 16: the reference loader's order
    (src/model/llama.zig:347-350) gives weight j = (j mod 16 - 8) * 0.5 for j < 32 (2i -> low
    nibble 2i, 2i+1 -> high nibble 2i+1); ggml's order puts the low nibbles first."""
    blk = np.zeros(18, dtype=np.uint8)
    blk[0:2] = np.array([0.5], dtype=np.float16).view(np.uint8)
    for i in range(16):
        blk[2 + i] = ((2 * i) % 16) | (((2 * i + 1) % 16) << 4)
    ref = oracle.q4_0_decode_f32(blk, 1, 32, order=0)[0]
    assert np.array_equal(ref, (np.arange(32) % 16 - 8).astype(np.float32) * 0.5)
    ggml = oracle.q4_0_decode_f32(blk, 1, 32, order=1)[0]
    assert np.array_equal(ggml[:16], ((2 * np.arange(16)) % 16 - 8).astype(np.float32) * 0.5)
    assert np.array_equal(ggml[16:], ((2 * np.arange(16) + 1) % 16 - 8).astype(np.float32) * 0.5)


@pytest.mark.parametrize("order", [0, 1])
def test_q4_0_repack_oracle_exact(order):
    """The layout restatement dequantises (shaders.zig:474-495 semantics, group 32) to exactly
    the loader's f32 weights, transposed to [k][n]."""
    n_rows, k = 6, 96
    blocks = _q4_0_blocks(11 + order, n_rows, k)
    w, s, z = oracle.q4_0_repack(blocks, n_rows, k, order)
    dense = oracle.dequant_f32(w, s, z, k, n_rows, 32)
    assert np.array_equal(dense, oracle.q4_0_decode_f32(blocks, n_rows, k, order).T)


def test_sampler_oracle():
    """softmax_f64 sums to 1 and sample_index follows the shader's first-exceeding search
    (shaders.zig:875-886), falling back to the last index."""
    logits = np.array([1.0, 2.0, 3.0], dtype=np.float32)
    p = oracle.softmax_f64(logits, 1.0)
    assert abs(p.sum() - 1.0) < 1e-12 and np.argmax(p) == 2
    assert oracle.sample_index(p, 0.0) == 0
    assert oracle.sample_index(p, p[0] + 1e-9) == 1
    assert oracle.sample_index(p, 1.5) == 2
    assert oracle.argmax_ref([3.0, 5.0, 5.0, 1.0]) == 1


def test_paged_attention_oracle_small():
    """The f64 restatement against a direct loop over tokens on a tiny case."""
    rng = np.random.default_rng(9)
    H, D, MB = 2, 4, 3
    q = rng.standard_normal((1, H, D))
    kc = rng.standard_normal((MB, H, 16, D))
    vc = rng.standard_normal((MB, H, 16, D))
    bt = np.array([[2, 0, 1]], dtype=np.int32)
    n = 20
    got = oracle.paged_attention_f64(q, kc, vc, bt, [n], 1, H, D, MB)
    for h in range(H):
        ks = np.array([kc[bt[0, t // 16], h, t % 16] for t in range(n)])
        vs = np.array([vc[bt[0, t // 16], h, t % 16] for t in range(n)])
        s = ks @ q[0, h] / np.sqrt(D)
        w = np.exp(s - s.max())
        assert np.allclose(got[0, h], (w / w.sum()) @ vs)
