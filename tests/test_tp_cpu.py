"""Tensor-parallel FFN on CPU ranks (gloo, world size 2 and 4): each rank runs the f64
oracle on its shard (tiny_kernel.tp.shard_ffn), the partial outputs are sum-all-reduced, and
the result must equal the unsharded FFN; the residual is added once, after the reduction.
Also checks the shard geometry (whole groups, strided gate/up columns, contiguous down rows)
and a rank that fails before the collective surfaces on the host without hanging."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tiny_kernel import data
from tiny_kernel.tp import shard_bounds, shard_ffn

HIDDEN, INTER, GS = 128, 512, 32


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, residual, q):
    import datetime

    import torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        W = data.make_ffn(5, HIDDEN, INTER, GS)
        x = data.make_x(5, "tpx", 2, HIDDEN)
        Ws = shard_ffn(W, rank, world)
        part = oracle.ffn_f64(x, Ws.norm_w, Ws.gate, Ws.up, Ws.down, 1e-5)
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        y = t.numpy()
        if residual:
            y = y + x
        if rank == 0:
            q.put(y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,residual", [(2, False), (4, True)])
def test_tp_shards_sum_to_full_ffn(world, residual):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, residual, q)) for r in range(world)]
    for p in procs:
        p.start()
    y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    W = data.make_ffn(5, HIDDEN, INTER, GS)
    x = data.make_x(5, "tpx", 2, HIDDEN)
    ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, 1e-5, residual=residual)
    assert oracle.normwise_err(y, ref) <= 1e-12


def test_shard_geometry():
    W = data.make_ffn(1, HIDDEN, INTER, GS)
    parts = [shard_ffn(W, r, 4) for r in range(4)]
    assert np.array_equal(np.concatenate([p.gate.w for p in parts], axis=1), W.gate.w)
    assert np.array_equal(np.concatenate([p.up.s for p in parts], axis=1), W.up.s)
    assert np.array_equal(np.concatenate([p.gate.z for p in parts], axis=1), W.gate.z)
    assert np.array_equal(np.concatenate([p.down.w for p in parts], axis=0), W.down.w)
    assert np.array_equal(np.concatenate([p.down.s for p in parts], axis=0), W.down.s)
    assert all(p.inter == INTER // 4 and p.down.K == INTER // 4 for p in parts)
    with pytest.raises(ValueError):
        shard_bounds(INTER, 256, 1, 4)  # 128-column shards cannot hold whole 256-groups


def _failing_rank(rank, world, port, q):
    import datetime

    import torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise SystemExit(3)  # leaves between steps, before the collective
        t = torch.zeros(4)
        try:
            dist.all_reduce(t)
            q.put("completed")
        except Exception as e:  # the survivor sees an error, not a hang
            q.put("error: " + type(e).__name__)
    finally:
        if rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert msg.startswith("error")
    assert procs[1].exitcode == 3
