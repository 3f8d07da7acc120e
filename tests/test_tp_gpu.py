"""GPU parity of the tensor-parallel INT4 FFN: one process per GPU, NCCL all-reduce, both through
torch.distributed and through the library's own C ABI group (tk_tp_*).

Rank r runs the engine on its shard (gate/up columns and down rows [r*I/tp, (r+1)*I/tp),
tiny_kernel.tp.shard_ffn); the f32 partial outputs are summed by an NCCL all-reduce over
NVLink; with the residual, rank 0's kernel adds x once before the reduction (the residual of
src/model/llama.zig:220-231).  Rank 0 compares the reduced output with the f64 oracle of the
unsharded FFN.  2 and 4 ranks; a case skips when the box has fewer GPUs than its ranks.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 7e-4  # the engine's FFN precision bar (the path tolerance is 1e-3)
EPS = 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, cases, result_path):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "tiny-kernel_b200"), os.path.join(root, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import oracle
    import tiny_kernel as tk
    from tiny_kernel import data, ops
    from tiny_kernel.tp import shard_ffn

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    dev = tk.init(rank)
    errs = []
    try:
        for (m, hidden, inter, gs, residual) in cases:
            W = data.make_ffn(41, hidden, inter, gs)
            x = data.make_x(42, f"tpx{m}", m, hidden)
            S = shard_ffn(W, rank, world)

            def d(a):
                a = np.ascontiguousarray(a)
                return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()

            out = torch.empty((m, hidden), dtype=torch.float32, device="cuda")
            ops.int4_ffn(dev, d(x), d(S.norm_w), [d(a) for a in (S.gate.w, S.gate.s, S.gate.z)],
                         [d(a) for a in (S.up.w, S.up.s, S.up.z)],
                         [d(a) for a in (S.down.w, S.down.s, S.down.z)], out, m, hidden, S.inter,
                         gs, eps=EPS, residual=residual and rank == 0)
            dist.all_reduce(out)
            torch.cuda.synchronize()
            if rank == 0:
                ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS, residual=residual)
                errs.append(float(oracle.normwise_err(out.cpu().numpy(), ref)))
    finally:
        dev.deinit()
        dist.destroy_process_group()
    if rank == 0:
        np.save(result_path, np.array(errs))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ffn_vs_oracle(torch_cuda, tmp_path, world):
    if torch_cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    cases = [(1, 4096, 14336, 64, False),   # config 1, TP2
             (1, 1024, 2048, 64, True),     # residual added once
             (4, 512, 1024, 32, False),
             (2, 256, 512, 64, True)]
    out = tmp_path / "errs.npy"
    mp.start_processes(_rank, args=(world, _free_port(), cases, str(out)), nprocs=world,
                       join=True, start_method="spawn")
    errs = np.load(out)
    assert len(errs) == len(cases)
    assert np.all(errs <= TOL), errs


def _rank_native(rank, world, uid, cases, result_path):
    """One rank of the C-ABI path: tk_tp_create + tk_int4_ffn_tp (NCCL inside libtkcuda)."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "tiny-kernel_b200"), os.path.join(root, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch

    import oracle
    import tiny_kernel as tk
    from tiny_kernel import data
    from tiny_kernel.tp import Group, shard_ffn

    torch.cuda.set_device(rank)
    dev = tk.init(rank)
    group = Group(dev, world, rank, uid)
    errs, exch, outs = [], [], []
    try:
        for (m, hidden, inter, gs, residual) in cases:
            W = data.make_ffn(43, hidden, inter, gs)
            S = shard_ffn(W, rank, world)

            def d(a):
                a = np.ascontiguousarray(a)
                return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()

            mats = [[d(a) for a in (M.w, M.s, M.z)] for M in (S.gate, S.up, S.down)]
            nw = d(S.norm_w)
            exch.append(group.ffn_exchange(m, hidden, S.inter, gs))
            # three calls with new inputs in the same buffers: the exchange areas' two halves
            # are used in turn
            xd = torch.empty((m, hidden), dtype=torch.float32, device="cuda")
            out = torch.empty((m, hidden), dtype=torch.float32, device="cuda")
            for call in range(3):
                x = data.make_x(44 + call, f"tpn{m}", m, hidden)
                xd.copy_(torch.from_numpy(x))
                group.int4_ffn(xd, nw, *mats, out, m, hidden, S.inter, gs, eps=EPS,
                               residual=residual)
                y = out.cpu().numpy()
                outs.append(y)
                if rank == 0:
                    ref = oracle.ffn_f64(x, W.norm_w, W.gate, W.up, W.down, EPS,
                                         residual=residual)
                    errs.append(float(oracle.normwise_err(y, ref)))
    finally:
        group.close()
        dev.deinit()
    np.save(f"{result_path}.out{rank}.npy", np.concatenate([o.reshape(-1) for o in outs]))
    if rank == 0:
        np.save(result_path, np.array(errs))
        np.save(f"{result_path}.exch.npy", np.array(exch))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ffn_native_group_vs_oracle(torch_cuda, tmp_path, world):
    if torch_cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from tiny_kernel.tp import unique_id
    cases = [(1, 4096, 14336, 64, False),   # config 1: the exchange fused into the decode kernel
             (1, 1024, 2048, 64, True),     # residual added once
             (2, 1024, 2048, 64, True),     # two rows, fused
             (4, 1024, 2048, 64, False),    # four rows: fused as well
             (16, 1024, 2048, 64, False)]   # batch 16: the tcgen05 GEMM on each shard
    out = tmp_path / "errs_native.npy"
    mp.start_processes(_rank_native, args=(world, unique_id(), cases, str(out)), nprocs=world,
                       join=True, start_method="spawn")
    errs = np.load(out)
    exch = np.load(f"{out}.exch.npy")
    print(f"TP{world}: exchanges {exch.tolist()}, errors {errs.tolist()}")
    assert len(errs) == 3 * len(cases)
    assert np.all(errs <= TOL), errs
    if exch[4] == 1:  # the group maps its peers: 1-4 rows take the fused exchange
        assert exch[0] == exch[1] == exch[2] == exch[3] == 2, exch
    # every rank holds the same sum, bit for bit
    ref = np.load(f"{out}.out0.npy")
    for r in range(1, world):
        assert np.array_equal(np.load(f"{out}.out{r}.npy").view(np.uint32), ref.view(np.uint32)), r
