"""Pointer-level calls into libtkcuda (device pointers as ints, e.g. tensor.data_ptr()).

``stream`` is a CUDA stream handle (int) or None for the device's own stream.  With
``sync=True`` the call is the synchronous entry point (results ready on return, as the
reference's forward() is); otherwise it only enqueues on ``stream``.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import Int4MatrixC, check


def _ptr(v) -> int:
    if v is None:
        return None
    if hasattr(v, "ptr"):
        return v.ptr
    if hasattr(v, "data_ptr"):
        return v.data_ptr()
    return int(v)


def _dev(device) -> int:
    return device.handle if hasattr(device, "handle") else int(device)


def qmatmul_int4(device, x, w_packed, scales, zeros, out, m, k, n, group_size,
                 stream=None, sync=True):
    L = _lib.lib()
    args = (_dev(device), _ptr(x), _ptr(w_packed), _ptr(scales), _ptr(zeros), _ptr(out),
            int(m), int(k), int(n), int(group_size))
    if sync and stream is None:
        check(L.tk_qmatmul_int4(*args))
    else:
        check(L.tk_qmatmul_int4_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def matrix(w_packed, scales, zeros) -> Int4MatrixC:
    return Int4MatrixC(_ptr(w_packed), _ptr(scales), _ptr(zeros))


def int4_ffn(device, x, norm_weight, gate, up, down, out, m, hidden, inter, group_size,
             eps=1e-5, h_out=None, residual=False, stream=None, sync=True, host_io=False):
    """gate/up/down: (w_packed, scales, zeros) triples or Int4MatrixC.  host_io: x and out are
    pinned host buffers (TK_FFN_HOST_IO)."""
    L = _lib.lib()
    mats = [g if isinstance(g, Int4MatrixC) else matrix(*g) for g in (gate, up, down)]
    flags = (_lib.TK_FFN_RESIDUAL if residual else 0) | (_lib.TK_FFN_HOST_IO if host_io else 0)
    args = (_dev(device), _ptr(x), _ptr(norm_weight), C.byref(mats[0]), C.byref(mats[1]),
            C.byref(mats[2]), _ptr(out), _ptr(h_out), int(m), int(hidden), int(inter),
            int(group_size), float(eps), flags)
    if sync and stream is None:
        check(L.tk_int4_ffn(*args))
    else:
        check(L.tk_int4_ffn_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def rmsnorm(device, x, weight, out, rows, dim, eps, stream=None, sync=True):
    L = _lib.lib()
    args = (_dev(device), _ptr(x), _ptr(weight), _ptr(out), int(rows), int(dim), float(eps))
    if sync and stream is None:
        check(L.tk_rmsnorm(*args))
    else:
        check(L.tk_rmsnorm_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def fused_rmsnorm_rope(device, x, weight, cos_cache, sin_cache, out, rows, dim, head_dim, pos,
                       eps, stream=None, sync=True):
    L = _lib.lib()
    args = (_dev(device), _ptr(x), _ptr(weight), _ptr(cos_cache), _ptr(sin_cache), _ptr(out),
            int(rows), int(dim), int(head_dim), int(pos), float(eps))
    if sync and stream is None:
        check(L.tk_fused_rmsnorm_rope(*args))
    else:
        check(L.tk_fused_rmsnorm_rope_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def silu_mul(device, gate, up, out, n, stream=None, sync=True):
    L = _lib.lib()
    args = (_dev(device), _ptr(gate), _ptr(up), _ptr(out), int(n))
    if sync and stream is None:
        check(L.tk_silu_mul(*args))
    else:
        check(L.tk_silu_mul_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def matvec(device, x, W, out, K, N, stream=None, sync=True):
    """out[n] = sum_k W[n][k] x[k], W f32 [N][K] (Matvec, fused.zig:53-89)."""
    L = _lib.lib()
    args = (_dev(device), _ptr(x), _ptr(W), _ptr(out), int(K), int(N))
    if sync and stream is None:
        check(L.tk_matvec(*args))
    else:
        check(L.tk_matvec_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def matvec_dual(device, x, W1, W2, out1, out2, K, N, stream=None, sync=True):
    """Two matvecs sharing x (MatvecDual, fused.zig:91-133)."""
    L = _lib.lib()
    args = (_dev(device), _ptr(x), _ptr(W1), _ptr(W2), _ptr(out1), _ptr(out2), int(K), int(N))
    if sync and stream is None:
        check(L.tk_matvec_dual(*args))
    else:
        check(L.tk_matvec_dual_async(*args, stream))
        if sync:
            check(L.tk_device_synchronize(_dev(device)))


def repack_q4_0(device, blocks, w_packed, scales, zeros, n_rows, k, order=0):
    """GGUF Q4_0 blocks [n_rows][k/32] x 18 B -> qmatmul_int4 layout, group size 32
    (order 0: the reference loader's nibble order, 1: ggml's)."""
    check(_lib.lib().tk_repack_q4_0(_dev(device), _ptr(blocks), _ptr(w_packed), _ptr(scales),
                                    _ptr(zeros), int(n_rows), int(k), int(order)))


def paged_attention(device, q, k_cache, v_cache, block_tables, context_lens, o, batch,
                    num_heads, head_dim, max_blocks):
    """PagedAttention.forward (attention.zig:51-100): decode attention over block-tabled caches."""
    check(_lib.lib().tk_paged_attention(_dev(device), _ptr(q), _ptr(k_cache), _ptr(v_cache),
                                        _ptr(block_tables), _ptr(context_lens), _ptr(o),
                                        int(batch), int(num_heads), int(head_dim),
                                        int(max_blocks)))


def argmax(device, x, n, out):
    """out[0] = index of the largest of x[0..n) (ties: the smallest index)."""
    check(_lib.lib().tk_argmax(_dev(device), _ptr(x), int(n), _ptr(out)))


def softmax_sample(device, logits, probs, sampled, vocab, temperature, random_val):
    """probs = softmax(logits / temperature); sampled[0] = first index whose cumulative
    probability exceeds random_val (shaders.zig:826-887)."""
    check(_lib.lib().tk_softmax_sample(_dev(device), _ptr(logits), _ptr(probs), _ptr(sampled),
                                       int(vocab), float(temperature), float(random_val)))


def dequant_int4(device, w_packed, scales, zeros, out, k, n, group_size):
    check(_lib.lib().tk_dequant_int4(_dev(device), _ptr(w_packed), _ptr(scales), _ptr(zeros),
                                     _ptr(out), int(k), int(n), int(group_size)))


def path(m, k, n, group_size) -> int:
    """qmatmul_int4's path: 3 = batch 1-2 decode kernel, 2 = tcgen05 GEMM, 1 = streaming engine,
    0 = CUDA-core fallback, -1 = invalid shape."""
    return _lib.lib().tk_qmatmul_int4_path(int(m), int(k), int(n), int(group_size))


def ffn_path(m, hidden, inter, group_size) -> int:
    """int4_ffn's path, with the same codes as path()."""
    return _lib.lib().tk_int4_ffn_path(int(m), int(hidden), int(inter), int(group_size))
