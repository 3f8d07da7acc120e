"""Tensor parallelism of the INT4 FFN across the GPUs of one node.

Sharding (one exchange per FFN):
  gate/up  column split: rank r owns output columns [r*I/tp, (r+1)*I/tp) -- a strided slice of
           every packed row ([K/2][N]), scale row ([K/gs][N]) and zero row ([K/gs][N/2]);
  down     row split: rank r owns K rows [r*I/tp, (r+1)*I/tp) -- contiguous in all three arrays.
Each rank normalises the replicated x itself, runs the FFN on its shard and produces a partial
[M, H] output; a sum all-reduce (NCCL over NVLink on GPUs, gloo on CPU) combines the partials.
The residual (x + FFN(x), src/model/llama.zig:220-231) is added once, after the reduction.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .data import FFNWeights, Int4Matrix


def shard_bounds(inter: int, gs: int, rank: int, world: int):
    """Column range [c0, c1) of the intermediate owned by `rank`; whole groups, even width."""
    if inter % world:
        raise ValueError(f"inter={inter} is not divisible by tp={world}")
    c0, c1 = rank * inter // world, (rank + 1) * inter // world
    if c0 % gs or c1 % gs:
        raise ValueError(f"shard [{c0},{c1}) does not align to group_size={gs}")
    return c0, c1


def shard_ffn(W: FFNWeights, rank: int, world: int) -> FFNWeights:
    """The rank's shard of an FFN (host copies, contiguous, reference layout)."""
    if world == 1:
        return W
    gs = W.gs
    c0, c1 = shard_bounds(W.inter, gs, rank, world)

    def cols(M: Int4Matrix) -> Int4Matrix:
        return Int4Matrix(np.ascontiguousarray(M.w[:, c0:c1]), np.ascontiguousarray(M.s[:, c0:c1]),
                          np.ascontiguousarray(M.z[:, c0 // 2:c1 // 2]), M.K, c1 - c0, gs)

    D = W.down
    down = Int4Matrix(np.ascontiguousarray(D.w[c0 // 2:c1 // 2]),
                      np.ascontiguousarray(D.s[c0 // gs:c1 // gs]),
                      np.ascontiguousarray(D.z[c0 // gs:c1 // gs]), c1 - c0, D.N, gs)
    return FFNWeights(W.norm_w, cols(W.gate), cols(W.up), down, W.hidden, c1 - c0, gs)


def unique_id() -> bytes:
    """A new group id (tk_tp_unique_id); rank 0 makes it and hands it to the other ranks."""
    buf = (C.c_uint8 * _lib.TK_TP_UNIQUE_ID_BYTES)()
    _lib.check(_lib.lib().tk_tp_unique_id(buf))
    return bytes(buf)


class Group:
    """A tensor-parallel group through the C ABI (tk_tp_*, NCCL inside libtkcuda): the native
    path a non-Python caller takes, with no torch.distributed involved."""

    def __init__(self, device, nranks: int, rank: int, uid: bytes):
        if len(uid) != _lib.TK_TP_UNIQUE_ID_BYTES:
            raise ValueError("group id must be 128 bytes")
        self.rank, self.nranks = rank, nranks
        self.device = device
        idbuf = (C.c_uint8 * _lib.TK_TP_UNIQUE_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        _lib.check(_lib.lib().tk_tp_create(device.handle, nranks, rank, idbuf, C.byref(h)))
        self.handle = h

    @property
    def uses_p2p(self) -> bool:
        """True when exchanges go over NVLink peer memory (the one-shot all-reduce)."""
        return bool(_lib.lib().tk_tp_uses_p2p(self.handle))

    def ffn_exchange(self, m, hidden, inter_shard, group_size) -> int:
        """How int4_ffn sums the ranks' outputs at this shape: 2 fused into the decode kernel,
        1 the peer-memory all-reduce kernel, 0 NCCL."""
        return int(_lib.lib().tk_int4_ffn_tp_exchange(self.handle, int(m), int(hidden),
                                                      int(inter_shard), int(group_size)))

    def close(self):
        if self.handle:
            _lib.lib().tk_tp_destroy(self.handle)
            self.handle = None

    def allreduce_sum(self, buf, count: int, stream=None):
        _lib.check(_lib.lib().tk_tp_allreduce_sum_f32(self.handle, _ptr(buf), int(count), stream))

    def int4_ffn(self, x, norm_weight, gate, up, down, out, m, hidden, inter_shard, group_size,
                 eps=1e-5, residual=False, stream=None, sync=True):
        """tk_int4_ffn_tp: this rank's shard, then the in-place sum over the group."""
        g, u, d = (_matrix(a) for a in (gate, up, down))
        flags = _lib.TK_FFN_RESIDUAL if residual else 0
        L = _lib.lib()
        if sync and stream is None:
            st = L.tk_int4_ffn_tp(self.handle, _ptr(x), _ptr(norm_weight), C.byref(g), C.byref(u),
                                  C.byref(d), _ptr(out), int(m), int(hidden), int(inter_shard),
                                  int(group_size), float(eps), flags)
        else:
            st = L.tk_int4_ffn_tp_async(self.handle, _ptr(x), _ptr(norm_weight), C.byref(g),
                                        C.byref(u), C.byref(d), _ptr(out), int(m), int(hidden),
                                        int(inter_shard), int(group_size), float(eps), flags,
                                        stream)
        _lib.check(st)
        if sync and stream is not None:
            self.device.synchronize()


def _ptr(v) -> int:
    return v if isinstance(v, int) else v.data_ptr()


def _matrix(a):
    if isinstance(a, _lib.Int4MatrixC):
        return a
    w, s, z = a
    return _lib.Int4MatrixC(_ptr(w), _ptr(s), _ptr(z))
