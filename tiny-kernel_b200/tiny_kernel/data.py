"""Seeded synthetic inputs for the INT4 GEMV / FFN path.

All randomness comes from SplitMix64 (Steele, Lea, Flood 2014) used as a counter-based
generator: value i of stream s is mix64(s + (i + 1) * 0x9E3779B97F4A7C15).  Streams are
derived from (seed, tag) so every tensor of a configuration is reproducible on its own.

Distributions (the reference names no dataset; these follow its bench conventions,
src/bench.zig:242-245, with random values instead of constants):
  x            f32  ~ N(0, 1)                (Box-Muller in f64, rounded to f32)
  codes        u8   uniform bytes = two uniform 4-bit codes per byte
  scales       f16  ~ U[0.005, 0.02]         (rounded to nearest f16)
  zeros        u8   uniform nibbles 0..15    (or 0x88 = zero point 8, the bench value)
  norm weight  f32  ~ N(1, 0.05)
Layout is the reference qmatmul_int4 layout (src/kernels/shaders.zig:442-501):
  w_packed [K/2][N], scales [K/gs][N], zeros [K/gs][N/2].
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def derive_seed(seed: int, tag: str) -> int:
    """64-bit stream seed for (seed, tag)."""
    h = hashlib.blake2b(tag.encode(), digest_size=8).digest()
    v = np.uint64((int(seed) ^ int.from_bytes(h, "little")) & 0xFFFFFFFFFFFFFFFF)
    return int(_mix64(np.array([v], dtype=np.uint64))[0])


def u64(stream_seed: int, n: int, offset: int = 0) -> np.ndarray:
    idx = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix64(np.uint64(stream_seed) + idx * GOLDEN)


def uniform_bytes(stream_seed: int, nbytes: int) -> np.ndarray:
    n64 = (nbytes + 7) // 8
    return u64(stream_seed, n64).view(np.uint8)[:nbytes].copy()


def uniform01(stream_seed: int, n: int) -> np.ndarray:
    return (u64(stream_seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(stream_seed: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    u = uniform01(stream_seed, 2 * n)
    u1, u2 = u[0::2], u[1::2]
    z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
    return mean + std * z


@dataclasses.dataclass
class Int4Matrix:
    """One INT4 matrix in the reference layout; y = x @ W with W [K, N]."""
    w: np.ndarray   # u8  [K/2, N]
    s: np.ndarray   # u16 [K/gs, N]  (f16 bit patterns)
    z: np.ndarray   # u8  [K/gs, N/2]
    K: int
    N: int
    gs: int

    @property
    def nbytes(self) -> int:
        return self.w.nbytes + self.s.nbytes + self.z.nbytes


def f16_uniform(stream_seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    v = lo + (hi - lo) * uniform01(stream_seed, n)
    return v.astype(np.float16).view(np.uint16)


def make_int4_matrix(seed: int, tag: str, K: int, N: int, gs: int,
                     zeros: str = "random") -> Int4Matrix:
    if K % gs or gs % 2 or N % 2:
        raise ValueError("K % gs, gs and N must be even-compatible")
    G = K // gs
    w = uniform_bytes(derive_seed(seed, tag + "/codes"), (K // 2) * N).reshape(K // 2, N)
    s = f16_uniform(derive_seed(seed, tag + "/scales"), G * N, 0.005, 0.02).reshape(G, N)
    if zeros == "random":
        z = uniform_bytes(derive_seed(seed, tag + "/zeros"), G * (N // 2)).reshape(G, N // 2)
    elif zeros == "eight":
        z = np.full((G, N // 2), 0x88, dtype=np.uint8)
    else:
        raise ValueError(zeros)
    return Int4Matrix(w, s, z, K, N, gs)


def make_x(seed: int, tag: str, m: int, k: int) -> np.ndarray:
    return normal(derive_seed(seed, tag), m * k).astype(np.float32).reshape(m, k)


def make_norm_weight(seed: int, tag: str, dim: int) -> np.ndarray:
    return normal(derive_seed(seed, tag), dim, 1.0, 0.05).astype(np.float32)


@dataclasses.dataclass
class FFNWeights:
    norm_w: np.ndarray
    gate: Int4Matrix
    up: Int4Matrix
    down: Int4Matrix
    hidden: int
    inter: int
    gs: int

    @property
    def nbytes(self) -> int:
        return self.norm_w.nbytes + self.gate.nbytes + self.up.nbytes + self.down.nbytes


def make_ffn(seed: int, hidden: int, inter: int, gs: int, layer: int = 0,
             zeros: str = "random") -> FFNWeights:
    p = f"ffn{layer}"
    return FFNWeights(
        norm_w=make_norm_weight(seed, p + "/norm", hidden),
        gate=make_int4_matrix(seed, p + "/gate", hidden, inter, gs, zeros),
        up=make_int4_matrix(seed, p + "/up", hidden, inter, gs, zeros),
        down=make_int4_matrix(seed, p + "/down", inter, hidden, gs, zeros),
        hidden=hidden, inter=inter, gs=gs)


def int4_matrix_bytes(K: int, N: int, gs: int) -> int:
    """Algorithmic bytes of one matrix: K*N/2 codes + (K/gs)*N*2 scales + (K/gs)*N/2 zeros."""
    return K * N // 2 + (K // gs) * N * 2 + (K // gs) * (N // 2)
