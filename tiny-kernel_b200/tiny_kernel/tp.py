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

import numpy as np

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
