"""f64 oracle of the reference INT4 GEMV / FFN path (test infrastructure only).

A CPU restatement, in numpy float64, of the reference's Metal shaders:
  qmatmul_int4        src/kernels/shaders.zig:442-501 (layout :479-495, zeros :467-476)
  rmsnorm             src/kernels/shaders.zig:16-56   (out = x * rsqrt(mean(x^2)+eps) * w)
  fused_rmsnorm_rope  src/kernels/shaders.zig:124-182
  fused_silu_mul      src/kernels/shaders.zig:344-357 + fast_silu :7-9
  INT4 FFN            src/bench.zig:266-341 (norm -> gate, up -> silu*up) + the down
                      projection and residual of src/model/llama.zig:220-231
The dequantised weight is float(scale) * (float(q) - float(zero)), which is exact in f32;
`dequant_f32` returns it bit for bit.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg use this module, and only as the checker.
"""
from __future__ import annotations

import numpy as np


def unpack_codes(w: np.ndarray, K: int, N: int) -> np.ndarray:
    """q[k][n] (u8 [K, N]) from the packed [K/2][N] bytes; even k = low nibble."""
    w = np.asarray(w, dtype=np.uint8).reshape(K // 2, N)
    q = np.empty((K, N), dtype=np.uint8)
    q[0::2] = w & 0x0F
    q[1::2] = w >> 4
    return q


def unpack_zeros(z: np.ndarray, G: int, N: int) -> np.ndarray:
    """zero[g][n] (u8 [G, N]) from the packed [G][N/2] bytes; even n = low nibble."""
    z = np.asarray(z, dtype=np.uint8).reshape(G, N // 2)
    out = np.empty((G, N), dtype=np.uint8)
    out[:, 0::2] = z & 0x0F
    out[:, 1::2] = z >> 4
    return out


def scales_f64(s: np.ndarray) -> np.ndarray:
    return np.asarray(s, dtype=np.uint16).view(np.float16).astype(np.float64)


def dequant_f32(w, s, z, K: int, N: int, gs: int) -> np.ndarray:
    """f32 [K, N] = float(scale[g][n]) * (float(q[k][n]) - float(zero[g][n]))."""
    G = K // gs
    q = unpack_codes(w, K, N).astype(np.float32)
    zz = np.repeat(unpack_zeros(z, G, N).astype(np.float32), gs, axis=0)
    sc = np.repeat(np.asarray(s, dtype=np.uint16).view(np.float16).astype(np.float32).reshape(G, N),
                   gs, axis=0)
    return (sc * (q - zz)).astype(np.float32)


def qmatmul_f64(x, w, s, z, K: int, N: int, gs: int) -> np.ndarray:
    """y[m][n] = sum_k x[m][k] * scale * (q - zero), in float64; x is [M, K] (or [K])."""
    x = np.asarray(x, dtype=np.float64).reshape(-1, K)
    G = K // gs
    w = np.asarray(w, dtype=np.uint8).reshape(K // 2, N)
    sc = scales_f64(s).reshape(G, N)
    zz = unpack_zeros(z, G, N).astype(np.float64)
    y = np.zeros((x.shape[0], N), dtype=np.float64)
    rows = gs // 2
    for g in range(G):
        blk = w[g * rows:(g + 1) * rows]
        q = np.empty((gs, N), dtype=np.float64)
        q[0::2] = blk & 0x0F
        q[1::2] = blk >> 4
        xg = x[:, g * gs:(g + 1) * gs]
        y += sc[g] * (xg @ q - np.outer(xg.sum(axis=1), zz[g]))
    return y


def rmsnorm_f64(x, w, eps: float) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    dim = x.shape[-1]
    rms = 1.0 / np.sqrt((x * x).sum(axis=-1, keepdims=True) / dim + eps)
    return x * rms * np.asarray(w, dtype=np.float64)


def fused_rmsnorm_rope_f64(x, w, cos_cache, sin_cache, head_dim: int, pos: int,
                           eps: float) -> np.ndarray:
    n = rmsnorm_f64(x, w, eps)
    half = head_dim // 2
    dim = n.shape[-1]
    c = np.asarray(cos_cache, dtype=np.float64)[pos * half:(pos + 1) * half]
    s = np.asarray(sin_cache, dtype=np.float64)[pos * half:(pos + 1) * half]
    out = np.empty_like(n)
    for h0 in range(0, dim, head_dim):
        a = n[..., h0:h0 + half]
        b = n[..., h0 + half:h0 + head_dim]
        out[..., h0:h0 + half] = a * c - b * s
        out[..., h0 + half:h0 + head_dim] = b * c + a * s
    return out


def silu_mul_f64(g, u) -> np.ndarray:
    g = np.asarray(g, dtype=np.float64)
    return g / (1.0 + np.exp(-g)) * np.asarray(u, dtype=np.float64)


def ffn_f64(x, norm_w, gate, up, down, eps: float, residual: bool = False,
            return_h: bool = False):
    """gate/up/down: objects with w, s, z, K, N, gs (tiny_kernel.data.Int4Matrix)."""
    x = np.asarray(x, dtype=np.float64)
    n = rmsnorm_f64(x, norm_w, eps)
    g = qmatmul_f64(n, gate.w, gate.s, gate.z, gate.K, gate.N, gate.gs)
    u = qmatmul_f64(n, up.w, up.s, up.z, up.K, up.N, up.gs)
    h = silu_mul_f64(g, u)
    y = qmatmul_f64(h, down.w, down.s, down.z, down.K, down.N, down.gs)
    if residual:
        y = y + x
    return (y, h) if return_h else y


def matvec_f64(x, W, K: int, N: int) -> np.ndarray:
    """Matvec (src/kernels/shaders.zig:184-226): out[n] = sum_k W[n*K + k] * x[k], W row-major
    [N][K]; computed in f64."""
    Wm = np.asarray(W, dtype=np.float64).reshape(N, K)
    return Wm @ np.asarray(x, dtype=np.float64).reshape(K)


def matvec_f32_sequential(x, W, K: int, N: int) -> np.ndarray:
    """The shader's own f32 order (shaders.zig:211-215): acc += x[k] * W[n*K + k] for k = 0..K-1.
    Pure-Python loop: small cases only."""
    Wm = np.asarray(W, dtype=np.float32).reshape(N, K)
    xs = np.asarray(x, dtype=np.float32).reshape(K)
    out = np.zeros(N, dtype=np.float32)
    for n in range(N):
        acc = np.float32(0.0)
        for k in range(K):
            acc = np.float32(acc + np.float32(xs[k] * Wm[n, k]))
        out[n] = acc
    return out


def q4_0_decode_f32(blocks, n_rows: int, k: int, order: int = 0) -> np.ndarray:
    """GGUF Q4_0 -> dense f32 [n_rows][k] (weight = (q - 8) * d).  order 0 follows the reference
    loader (src/model/llama.zig:341-353: weight 2i = low nibble of qs[i], 2i+1 = high nibble);
    order 1 the ggml layout (weight i = low nibble, i + 16 = high nibble)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(n_rows, k // 32, 18)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)  # [n][k/32][1]
    qs = b[:, :, 2:]
    lo, hi = (qs & 0xF).astype(np.float32), (qs >> 4).astype(np.float32)
    q = np.empty((n_rows, k // 32, 32), dtype=np.float32)
    if order == 0:
        q[:, :, 0::2], q[:, :, 1::2] = lo, hi
    else:
        q[:, :, :16], q[:, :, 16:] = lo, hi
    return ((q - 8.0) * d).reshape(n_rows, k).astype(np.float32)


def q4_0_repack(blocks, n_rows: int, k: int, order: int = 0):
    """The qmatmul_int4 layout (group size 32) of GGUF Q4_0 blocks: (w_packed [k/2][n],
    scales f16 bits [k/32][n], zeros [k/32][n/2] = 0x88), codes and d unchanged."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(n_rows, k // 32, 18)
    d = b[:, :, 0:2].copy().view(np.uint16)[:, :, 0]  # [n][k/32]
    qs = b[:, :, 2:]
    lo, hi = qs & 0xF, qs >> 4
    q = np.empty((n_rows, k // 32, 32), dtype=np.uint8)
    if order == 0:
        q[:, :, 0::2], q[:, :, 1::2] = lo, hi
    else:
        q[:, :, :16], q[:, :, 16:] = lo, hi
    qk = q.reshape(n_rows, k).T  # [k][n]
    w = (qk[0::2] | (qk[1::2] << 4)).astype(np.uint8)
    return (np.ascontiguousarray(w), np.ascontiguousarray(d.T.astype(np.uint16)),
            np.full((k // 32, n_rows // 2), 0x88, dtype=np.uint8))


def paged_attention_f64(q, k_cache, v_cache, block_tables, context_lens, batch: int,
                        num_heads: int, head_dim: int, max_blocks: int) -> np.ndarray:
    """paged_attention (src/kernels/shaders.zig:503-587) in f64: for sequence b, head h,
    softmax(q . k_t * head_dim^-1/2) over tokens t < context_lens[b], weighting v_t; token t is
    row t % 16 of physical block block_tables[b][t / 16] in caches [block][heads][16][head_dim].
    An empty sequence gives zeros."""
    B = 16
    q = np.asarray(q, dtype=np.float64).reshape(batch, num_heads, head_dim)
    kc = np.asarray(k_cache, dtype=np.float64).reshape(-1, num_heads, B, head_dim)
    vc = np.asarray(v_cache, dtype=np.float64).reshape(-1, num_heads, B, head_dim)
    bt = np.asarray(block_tables).reshape(batch, max_blocks)
    out = np.zeros((batch, num_heads, head_dim))
    scale = 1.0 / np.sqrt(head_dim)
    for b in range(batch):
        n = int(context_lens[b])
        if n <= 0:
            continue
        t = np.arange(n)
        phys = bt[b, t // B]
        for h in range(num_heads):
            K = kc[phys, h, t % B]
            V = vc[phys, h, t % B]
            s = K @ q[b, h] * scale
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ V
    return out


def argmax_ref(x) -> int:
    """Index of the largest value, the smallest index on ties (numpy's argmax)."""
    return int(np.argmax(np.asarray(x, dtype=np.float64)))


def softmax_f64(logits, temperature: float) -> np.ndarray:
    """softmax(logits / temperature) in f64 (shaders.zig:826-873)."""
    z = np.asarray(logits, dtype=np.float64) / float(temperature)
    e = np.exp(z - z.max())
    return e / e.sum()


def sample_index(probs, random_val: float) -> int:
    """The first i with random_val < cumsum(probs)[i], len - 1 if none (shaders.zig:875-886)."""
    c = np.cumsum(np.asarray(probs, dtype=np.float64))
    hit = np.nonzero(random_val < c)[0]
    return int(hit[0]) if len(hit) else len(c) - 1


def normwise_err(y, ref) -> float:
    """max_i |y_i - ref_i| / max_i |ref_i| (the path's error metric)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(y - ref).max() / (den if den > 0 else 1.0))


def kat_bench_constants() -> float:
    """Known answer from the reference bench constants (src/bench.zig:242-245):
    x = 0.1, every byte 0x77 (q = 7), scale = f16(0.01), zero byte 0x88 (z = 8), K = 4096:
    y[n] = 4096 * 0.1 * f16(0.01) * (7 - 8) for every n (computed in float64 with x
    rounded to f32 as the reference stores it)."""
    return 4096 * float(np.float32(0.1)) * float(np.float16(0.01)) * (7 - 8)
