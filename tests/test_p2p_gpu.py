"""GPU tests of the one-shot peer-memory all-reduce (tk_tp_allreduce_sum_f32), 2 and 4 GPUs.

Every rank generates every rank's input from the seed, so each can check the sum bit-exactly
against the f32 sum in rank order (the order the kernel uses); the size beyond the peer path's
limit goes to NCCL, checked bit-exactly at 2 ranks and within f32 rounding from 3 on.  Covered: ragged and vector sizes
up to the peer path's limit and one beyond it (NCCL), repeated calls (both buffer parities), a
CUDA graph replayed with new inputs (the epochs live on the device), and a wait that runs out:
rank 0 calls alone with a short bound and gets TK_ERR_TIMEOUT, no GPU fault.  A case skips
when the box has fewer GPUs than its ranks.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 4, 511, 512, 513, 4096, 65536 + 7, 262144, 262144 + 4]
PEER_MAX_FLOATS = 512 * 512  # the peer path's limit (512 chunks of 512 floats); NCCL beyond it


def _setup(rank):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "tiny-kernel_b200"), os.path.join(root, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")


def _inputs(n, world, it):
    return [np.random.default_rng(1000 * it + 17 * r + n).standard_normal(n).astype(np.float32)
            for r in range(world)]


def _expect(xs):
    v = xs[0].copy()
    for a in xs[1:]:
        v = (v + a).astype(np.float32)
    return v


def _matches(got, xs):
    """The peer path sums in rank order: bit-exact.  Beyond its limit NCCL reduces, whose order
    is its own from 3 ranks on (with 2, a + b is the same either way): within the f32 rounding
    of a sum in any order, (ranks - 1) * eps * sum |x_r| per element."""
    exp = _expect(xs)
    if len(xs) <= 2 or got.size <= PEER_MAX_FLOATS:
        return np.array_equal(got, exp)
    bound = (len(xs) - 1) * np.finfo(np.float32).eps * np.sum(np.abs(np.stack(xs)), axis=0)
    return bool(np.all(np.abs(got.astype(np.float64) - exp) <= bound))


def _rank_sum(rank, world, uid, result_path):
    _setup(rank)
    import torch

    import tiny_kernel as tk
    from tiny_kernel.tp import Group

    torch.cuda.set_device(rank)
    dev = tk.init(rank)
    g = Group(dev, world, rank, uid)
    bad = []
    try:
        assert g.uses_p2p
        for it in range(3):
            for n in SIZES:
                xs = _inputs(n, world, it)
                buf = torch.from_numpy(xs[rank]).cuda()
                g.allreduce_sum(buf, n)
                dev.synchronize()
                if not _matches(buf.cpu().numpy(), xs):
                    bad.append((it, n))
        # CUDA graph: the all-reduce captured once, replayed with new inputs
        n = 4096
        buf = torch.zeros(n, device="cuda")
        stream = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            g.allreduce_sum(buf, n, stream=stream.cuda_stream)
        for it in range(10, 14):
            xs = _inputs(n, world, it)
            buf.copy_(torch.from_numpy(xs[rank]))
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            if not np.array_equal(buf.cpu().numpy(), _expect(xs)):
                bad.append(("graph", it))
        del graph
    finally:
        g.close()
        dev.deinit()
    if rank == 0:
        np.save(result_path, np.array([len(bad)]))
        if bad:
            print("mismatches:", bad)


def _run(fn, world, *args):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(world,) + args, nprocs=world, join=True, start_method="spawn")


@pytest.mark.parametrize("world", [2, 4])
def test_p2p_allreduce_bit_exact(torch_cuda, tmp_path, world):
    if torch_cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from tiny_kernel.tp import unique_id
    out = tmp_path / "bad.npy"
    _run(_rank_sum, world, unique_id(), str(out))
    assert int(np.load(out)[0]) == 0


def _rank_timeout(rank, world, uid, result_path):
    import ctypes as C

    _setup(rank)
    os.environ["TK_WAIT_TIMEOUT_MS"] = "200"
    import torch

    import tiny_kernel as tk
    from tiny_kernel import _lib
    from tiny_kernel.tp import Group

    torch.cuda.set_device(rank)
    dev = tk.init(rank)
    g = Group(dev, world, rank, uid)
    status = 0
    try:
        if rank == 0:
            # rank 1 never joins this exchange: rank 0's flags are never set
            buf = torch.ones(1024, device="cuda")
            g.allreduce_sum(buf, 1024)
            torch.cuda.synchronize()
            status = _lib.lib().tk_device_check_error(dev.handle)
            # the group is now out of step with its peer: a further exchange is refused on
            # the host, before any launch
            again = _lib.lib().tk_tp_allreduce_sum_f32(g.handle, C.c_void_p(buf.data_ptr()), 1024,
                                                       None)
            status = status if again == _lib.TK_ERR_TIMEOUT else -100
    finally:
        g.close()  # a group that saw a timeout is not reused
        dev.deinit()
    if rank == 0:
        np.save(result_path, np.array([status]))


@pytest.mark.parametrize("world", [2])
def test_p2p_allreduce_wait_times_out(torch_cuda, tmp_path, world):
    if torch_cuda.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from tiny_kernel import _lib
    from tiny_kernel.tp import unique_id
    out = tmp_path / "status.npy"
    _run(_rank_timeout, world, unique_id(), str(out))
    assert int(np.load(out)[0]) == _lib.TK_ERR_TIMEOUT
