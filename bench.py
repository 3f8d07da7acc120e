#!/usr/bin/env python
"""INT4 FFN decode benchmark on B200: HBM GB/s (% of peak) and tokens/s.

Workload (default, one GPU): the Llama-3-8B-shaped INT4 FFN at batch 1 --
rmsnorm(eps 1e-5) -> gate/up INT4 GEMV (4096 -> 14336) -> silu(gate)*up -> down INT4 GEMV
(14336 -> 4096) in f32 -- on seeded synthetic inputs in the reference qmatmul_int4 layout
(group 64, f16 scales, 4-bit zero points).  One step = one FFN forward = one launch of the
persistent decode kernel at batch 1-2.  With --gpus N (torchrun, one rank per GPU) the FFN is
tensor-parallel: gate/up column-split, down row-split, the f32 partial outputs summed over the
ranks -- by the library's group (--collective lib, the default: at batch 1-2 inside the same
decode launch, over NVLink peer memory) or by a torch.distributed NCCL all-reduce (nccl).
--model 70b: the Llama-3-70B FFN shape (8192 -> 28672 -> 8192).  --layers L: one step is a
stack of L FFN blocks with their own weights, each x <- x + FFN(x) (the residual is added
once: after the fused sum, or by rank 0's kernel before an all-reduce).

value     whole-job algorithmic GB/s: FFN bytes (weights + x + norm weight + out) per step
          x steps / max-over-ranks device time; inputs resident in HBM; L2 defeated by
          rotating several weight copies whose total exceeds 3x the L2 size.
e2e       the same metric through the C ABI with host buffers, every step: one FFN block on one
          GPU is one synchronous tk_int4_ffn call with TK_FFN_HOST_IO (the kernel reads x from
          and writes y to pinned host memory over the host link); the matvec, stacks and
          tensor parallelism queue the activation's upload from pinned host memory, the step and
          the output's download on the device's stream and wait once (tk_device_synchronize).
--impl reference  times the CPU transcription of the reference shaders (oracle/), all host
          threads, on the same workload (the reference itself is Zig + Metal and cannot run
          on this Linux host).
--config 0  the bare INT4 matvec y[1,14336] = x[1,4096] . W^T (qmatmul_int4, the reference's own
          INT4 benchmark, src/bench.zig:219-264): one step = one launch; with --gpus N every rank
          runs its own replica (the matvec is not sharded).
parity    after the timed region one untimed step (host-generated weights: the default 8B FFN
          and config 0) is checked against the f64 oracle on rank 0; the line carries the
          normwise error and the process exits non-zero when it is above the 1e-3 contract.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "tiny-kernel_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

HIDDEN, INTER, GS, EPS = 4096, 14336, 64, 1e-5
SEED = 20261201
MODELS = {"8b": ("Llama-3-8B", 4096, 14336), "70b": ("Llama-3-70B", 8192, 28672)}


def ffn_bytes(m, hidden, inter, gs):
    from tiny_kernel.data import int4_matrix_bytes
    w = 2 * int4_matrix_bytes(hidden, inter, gs) + int4_matrix_bytes(inter, hidden, gs)
    return w + m * hidden * 4 + hidden * 4 + m * hidden * 4


def ffn_weight_bytes(hidden, inter, gs):
    """Packed weights + scales + zero points of the three matrices."""
    from tiny_kernel.data import int4_matrix_bytes
    return 2 * int4_matrix_bytes(hidden, inter, gs) + int4_matrix_bytes(inter, hidden, gs)


def ffn_flops(m, hidden, inter):
    """Multiply-adds of the three projections, 2 FLOPs each."""
    return 2 * m * 3 * hidden * inter


def arithmetic(path, m):
    """(short dtype, description) of the arithmetic the path computes in at m rows."""
    if path == 2:
        return ("int4->f16 x f16 -> f32",
                "INT4 weights dequantised to f16, f16 activations (and f16 h between the GEMMs), "
                "tcgen05 MMA with f32 accumulation, f32 output")
    if path == 3:
        return ("int4 x int16 -> int32 -> f32",
                "INT4 weights x activations quantised to int16 per group (one power-of-two "
                "scale), dp2a with exact int32 group sums, f32 scale and accumulation, f32 "
                "output" + (" (chunks of 4 rows)" if m > 4 else ""))
    if path == 1:
        return ("int4 x int8 hi/lo -> int32 -> f32",
                "INT4 weights x activations split into int8 hi + lo/256 parts per group, int8 "
                "tensor-core MMA with exact int32 group sums, f32 scale and accumulation, f32 "
                "output (chunks of 4 rows)")
    return ("f32", "f32 dequantisation and accumulation (CUDA cores)")


def load_peaks():
    """(HBM GB/s, dense f16/bf16 TFLOP/s burst, which)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def load_traffic(key):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "int4_ffn_decode_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(key)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (read-only) in a thread."""

    def __init__(self, index, period=0.005):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self._thr = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self._N = N
            self._h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self._h, N.NVML_CLOCK_SM)
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        except Exception as e:  # NVML missing: report no clocks rather than fail the bench
            self._err = str(e)
        return self

    def _run(self):
        N = self._N
        names = {
            "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
            "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        }
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self._h, N.NVML_CLOCK_SM))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for k, v in names.items():
                    if r & v and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def run_reference(args, world, rank):
    """CPU transcription of the reference shaders, all host threads (rank 0 only)."""
    if rank != 0:
        return
    import cpu
    from tiny_kernel import data
    m = args.batch
    name, hidden, inter = MODELS[args.model]
    x = data.make_x(SEED, "x", m, hidden)
    threads = cpu.default_threads()
    if args.config == 0:
        run_reference_matvec(args, world, m, hidden, inter, x, threads)
        return
    W = data.make_ffn(SEED, hidden, inter, GS)
    runner = cpu.FFNRunner(W, m, EPS, threads=threads)
    for _ in range(max(1, min(args.warmup, 3))):
        runner(x)
    t0 = time.perf_counter()
    runner(x)
    one = time.perf_counter() - t0
    steps = max(1, min(args.steps, int(60.0 / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        runner(x)
    dt = time.perf_counter() - t0
    nbytes = ffn_bytes(m, hidden, inter, GS)
    gbs = nbytes * steps / dt / 1e9
    L = args.layers
    line = {
        "impl": "reference", "metric": "INT4 FFN decode HBM GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(dt / steps * 1e3 * L, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tokens_per_s": round(m * steps / dt / L, 2),
        "ref_style_gibs": round(ffn_weight_bytes(hidden, inter, GS) * steps / dt / 2**30, 3),
        "config": {"workload": workload_name(name, m, L),
                   "hidden": hidden, "inter": inter, "group_size": GS, "batch": m, "layers": L,
                   "parallelism": "host CPU", "steps_requested": args.steps,
                   "sample": "one FFN block per timed step (every block of a stack is the same work)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} full FFN steps (the reference's Metal shaders cannot "
                                   f"run here: Zig + Metal; this is their C++ std::thread "
                                   f"transcription, oracle/cpu_baseline.cpp)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_matvec(args, world, m, hidden, inter, x, threads):
    """The reference arm of --config 0: qmatmul_int4 of the CPU transcription, all threads."""
    import cpu
    from tiny_kernel import data
    M = data.make_int4_matrix(SEED, "matvec", hidden, inter, GS)
    for _ in range(max(1, min(args.warmup, 3))):
        cpu.qmatmul_int4(x, M, threads)
    t0 = time.perf_counter()
    cpu.qmatmul_int4(x, M, threads)
    one = time.perf_counter() - t0
    steps = max(1, min(args.steps, int(60.0 / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu.qmatmul_int4(x, M, threads)
    dt = time.perf_counter() - t0
    nbytes = M.nbytes + m * hidden * 4 + m * inter * 4
    gbs = nbytes * steps / dt / 1e9
    line = {
        "impl": "reference", "metric": "INT4 matvec HBM GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(dt / steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tokens_per_s": round(m * steps / dt, 2),
        "ref_style_gibs": round(M.nbytes * steps / dt / 2**30, 3),
        "config": {"workload": f"INT4 matvec y[{m},{inter}] = x[{m},{hidden}] . W^T (qmatmul_int4)",
                   "hidden": hidden, "inter": inter, "group_size": GS, "batch": m, "layers": 1,
                   "parallelism": "host CPU", "steps_requested": args.steps,
                   "sample": "one matvec per timed step"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} full matvecs (the reference's Metal shader cannot run "
                                   f"here: Zig + Metal; this is its C++ std::thread "
                                   f"transcription, oracle/cpu_baseline.cpp)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_name(name, m, layers):
    base = f"{name} INT4 FFN decode (rmsnorm->gate/up->silu*up->down), batch {m}"
    return base if layers == 1 else f"{name} INT4 decode stack: {layers} FFN blocks with residual, batch {m}"


def device_ffn(seed, layer, hidden, inter, gs, device):
    """Synthetic INT4 FFN weights of the given (shard) shape generated on the GPU: uniform
    codes and zero points, f16 scales uniform [0.005, 0.02], norm weight ~ N(1, 0.05)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + layer)

    def mat(K, N):
        w = torch.randint(0, 256, (K // 2, N), dtype=torch.uint8, generator=g, device=device)
        sc = (torch.rand((K // gs, N), generator=g, device=device) * 0.015 + 0.005).half()
        z = torch.randint(0, 256, (K // gs, N // 2), dtype=torch.uint8, generator=g, device=device)
        return [w, sc.view(torch.int16), z]

    nw = (1.0 + 0.05 * torch.randn(hidden, generator=g, device=device)).float()
    return nw, mat(hidden, inter), mat(hidden, inter), mat(inter, hidden)


def cpu_baseline_sample(W, x, m, hidden, inter):
    import cpu
    threads = cpu.default_threads()
    runner = cpu.FFNRunner(W, m, EPS, threads=threads)
    runner(x)
    t0 = time.perf_counter()
    n = 0
    while True:
        runner(x)
        n += 1
        if time.perf_counter() - t0 > 10.0 or n >= 200:
            break
    dt = time.perf_counter() - t0
    return {"value": round(ffn_bytes(m, hidden, inter, GS) * n / dt / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{n} full FFN blocks on the host ({dt:.1f} s), C++ std::thread transcription "
                      f"of the reference shaders (oracle/cpu_baseline.cpp)"}


def align_ranks(pg, stream):
    """A one-element all-reduce enqueued on `stream`: the ranks' timed regions start on the
    device together (a host barrier alone leaves the ranks' graph replays skewed)."""
    if pg is None:
        return
    import torch
    t = torch.ones(1, device="cuda")
    with torch.cuda.stream(stream):
        pg.all_reduce(t)


def gather_ms(pg, ms):
    """(max over ranks, every rank's value) of a device time."""
    if pg is None:
        return ms, [ms]
    import torch
    t = torch.tensor([ms], device="cuda")
    outs = [torch.zeros_like(t) for _ in range(pg.get_world_size())]
    pg.all_gather(outs, t)
    vals = [float(o.item()) for o in outs]
    return max(vals), vals


def cpu_baseline_matvec(M, x, m, hidden, inter):
    """The CPU transcription's qmatmul_int4 on all host threads, about 10 s of matvecs."""
    import cpu
    threads = cpu.default_threads()
    cpu.qmatmul_int4(x, M, threads)
    t0 = time.perf_counter()
    n = 0
    while True:
        cpu.qmatmul_int4(x, M, threads)
        n += 1
        if time.perf_counter() - t0 > 10.0 or n >= 400:
            break
    dt = time.perf_counter() - t0
    nbytes = M.nbytes + m * hidden * 4 + m * inter * 4
    return {"value": round(nbytes * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{n} full matvecs on the host ({dt:.1f} s), C++ std::thread transcription "
                      f"of the reference qmatmul_int4 shader (oracle/cpu_baseline.cpp)"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--model", default="8b", choices=sorted(MODELS))
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--config", type=int, default=1, choices=[0, 1],
                    help="0: the bare INT4 matvec 1x4096x14336 (qmatmul_int4); 1: the INT4 FFN")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--collective", default="lib", choices=["lib", "p2p", "nccl"],
                    help="tensor-parallel exchange: the library's group (lib, or its old name "
                         "p2p: at batch 1-2 fused into the decode kernel over NVLink peer "
                         "memory, else a one-shot peer-memory all-reduce, NCCL beyond its size "
                         "limit) or torch.distributed NCCL after the library's shard FFN")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config == 0 and (args.layers != 1 or args.model != "8b"):
        raise SystemExit("--config 0 is the 4096 x 14336 matvec: no --layers / --model")
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import tiny_kernel as tk
    from tiny_kernel import data, ops
    from tiny_kernel.tp import shard_bounds, shard_ffn

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    dev = tk.init(local)
    matvec = args.config == 0
    group = None
    if pg is not None and args.collective in ("lib", "p2p") and not matvec:
        from tiny_kernel.tp import Group, unique_id
        box = [unique_id() if rank == 0 else None]
        pg.broadcast_object_list(box, src=0)
        group = Group(dev, world, rank, box[0])
    m = args.batch
    L = args.layers
    name, hidden, inter_full = MODELS[args.model]
    tp = 1 if matvec else world  # the matvec runs one replica per rank
    if not matvec:
        shard_bounds(inter_full, GS, rank, world)  # validates the split
    inter = inter_full // tp
    x_host = data.make_x(SEED, "x", m, hidden)

    def to_dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(a).cuda()

    # per-GPU weights: the seeded host generator (the oracle's) for the default one-block 8B
    # workload and the matvec, which the CPU baseline also runs; a GPU-side generator of the
    # shard's shapes for the larger workloads (gigabytes of host-side generation otherwise)
    host_gen = args.model == "8b" and L == 1
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    W_full = M0 = None
    if matvec:
        M0 = data.make_int4_matrix(SEED, "matvec", hidden, inter_full, GS)
        layer_bytes = data.int4_matrix_bytes(hidden, inter_full, GS) + m * hidden * 4 + m * inter_full * 4
        shard_w_bytes = data.int4_matrix_bytes(hidden, inter_full, GS)
        per_gpu_bytes = layer_bytes
        per_gpu_flops = 2 * m * hidden * inter_full
        step_bytes_total = layer_bytes * world  # every rank's replica
    else:
        layer_bytes = ffn_bytes(m, hidden, inter_full, GS)
        step_bytes_total = L * layer_bytes
        W_full = data.make_ffn(SEED, hidden, inter_full, GS) if host_gen else None
        shard_w_bytes = (2 * data.int4_matrix_bytes(hidden, inter, GS) +
                         data.int4_matrix_bytes(inter, hidden, GS))
        per_gpu_bytes = L * (shard_w_bytes + m * hidden * 4 * 2 + hidden * 4)
        per_gpu_flops = L * ffn_flops(m, hidden, inter)
    copies = max(4 if L == 1 else 1, math.ceil(3 * l2 / (L * shard_w_bytes)))
    layers = []  # [copy][layer] -> (norm weight, gate, up, down) device tensors, or the matrix
    if matvec:
        mat0 = [to_dev(a) for a in (M0.w, M0.s, M0.z)]
        layers.append(mat0)
        for _ in range(copies - 1):
            layers.append([t.clone() for t in mat0])
        mats = [ops.matrix(*c) for c in layers]
    else:
        if host_gen:
            W = shard_ffn(W_full, rank, world)
            mw = [[to_dev(a) for a in (M.w, M.s, M.z)] for M in (W.gate, W.up, W.down)]
            nw = to_dev(W.norm_w)
            layers.append([(nw, mw[0], mw[1], mw[2])])
            for _ in range(copies - 1):
                layers.append([(nw, [t.clone() for t in mw[0]], [t.clone() for t in mw[1]],
                                [t.clone() for t in mw[2]])])
        else:
            for c in range(copies):
                layers.append([device_ffn(SEED + 7919 * c + 104729 * rank, l, hidden, inter, GS,
                                          "cuda") for l in range(L)])
        mats = [[(nw, ops.matrix(*g), ops.matrix(*u), ops.matrix(*d)) for (nw, g, u, d) in cl]
                for cl in layers]
    x0 = to_dev(x_host)
    out_cols = inter_full if matvec else hidden
    xa = torch.empty((m, out_cols), dtype=torch.float32, device="cuda")
    xb = torch.empty((m, out_cols), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    # stacks carry the residual (added once, by rank 0's kernel, before the all-reduce)
    residual = L > 1 and (rank == 0 or group is not None)

    def run_step(i, x_in, bufs, sync, on=None):
        """One step: the matvec, or L FFN blocks; returns the buffer that holds the step's
        output.  Without sync the work is queued on `on` (a torch stream; default the bench's
        own stream)."""
        on = stream if on is None else on
        st = None if sync else on.cuda_stream
        if matvec:
            w = mats[i % copies]
            ops.qmatmul_int4(dev, x_in, w.w_packed, w.scales, w.zeros, bufs[0], m, hidden,
                             inter_full, GS, stream=st, sync=sync)
            return bufs[0]
        cur = x_in
        for l in range(L):
            nw, g, u, d = mats[i % copies][l]
            out = bufs[l % 2]
            if group is not None:
                # shard FFN + the exchange, both inside the library
                group.int4_ffn(cur, nw, g, u, d, out, m, hidden, inter, GS, eps=EPS,
                               residual=residual, stream=st, sync=sync)
                cur = out
                continue
            ops.int4_ffn(dev, cur, nw, g, u, d, out, m, hidden, inter, GS, eps=EPS,
                         residual=residual, stream=st, sync=sync)
            if pg is not None:
                if sync:
                    pg.all_reduce(out)
                    torch.cuda.current_stream().synchronize()
                else:
                    with torch.cuda.stream(on):
                        pg.all_reduce(out)
            cur = out
        return cur

    def step(i):
        run_step(i, x0, (xa, xb), False)

    # warm-up (also sizes the engine's scratch before any capture); the last warm-up step
    # counts the kernels one step enqueues
    for i in range(args.warmup):
        n0 = dev.launch_count()
        step(i)
        launches_per_step = dev.launch_count() - n0
    stream.synchronize()
    dev.synchronize()
    path = ops.path(m, hidden, inter_full, GS) if matvec else ops.ffn_path(m, hidden, inter, GS)

    graph = None
    per_graph = max(1, min(args.steps, 4000 // L))
    reps = math.ceil(args.steps / per_graph)
    steps_timed = args.steps
    if not args.no_graph:
        # one graph per rank; with several ranks it holds the NCCL all-reduces too (released
        # before the process group is destroyed)
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(per_graph):
                    step(i)
            graph.replay()
            stream.synchronize()
            steps_timed = reps * per_graph
        except Exception as e:  # capture unsupported: fall back to stream launches
            print(f"# graph capture failed ({e}); timing stream launches", file=sys.stderr)
            graph = None
            torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # one untimed step enqueued right before the first timed event keeps the GPU busy while
        # the host submits the timed graph, so the timed region holds the K steps and no launch
        # gap or idle-clock ramp
        if graph is not None:
            with torch.cuda.stream(stream):
                graph.replay()
        else:
            step(0)
        align_ranks(pg, stream)
        ev0.record(stream)
        if graph is not None:
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    graph.replay()
        else:
            for i in range(steps_timed):
                step(i)
        ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    ms, rank_ms = gather_ms(pg, ev0.elapsed_time(ev1))
    from tiny_kernel._lib import check, lib
    check(lib().tk_device_check_error(dev.handle))
    ms_per_step = ms / steps_timed
    value = step_bytes_total * steps_timed / (ms / 1e3) / 1e9
    peak, peak_tc, peak_kind = load_peaks()
    achieved = per_gpu_bytes / (ms_per_step / 1e3) / 1e9
    tflops = per_gpu_flops / (ms_per_step / 1e3) / 1e12
    # the bound of the step: whichever of HBM bytes and tensor FLOPs takes longer at peak
    tensor_bound = per_gpu_flops / (peak_tc * 1e12) > per_gpu_bytes / (peak * 1e9)

    # ---- end to end through the C ABI with host buffers -------------------------------
    # A user's step: the activation's upload, the kernel(s) and the output's download queued on
    # the device's stream, then one wait for the result (tk_device_synchronize), every step.
    import ctypes as C
    Lb = lib()
    xb_host = tk.Buffer(dev, "f32", m * hidden, kind=2)   # pinned host
    ob_host = tk.Buffer(dev, "f32", m * out_cols, kind=2)
    np.copyto(np.frombuffer((C.c_char * xb_host.nbytes).from_address(xb_host.ptr), np.float32),
              x_host.reshape(-1))
    xd = torch.empty((m, hidden), dtype=torch.float32, device="cuda")
    e2e_steps = max(1, min(steps_timed, 2000 // L))
    devstream = torch.cuda.ExternalStream(dev.stream())

    # One FFN block on one GPU: a single synchronous call with x and y in pinned host memory
    # (TK_FFN_HOST_IO: the kernel reads x and writes y over the host link).  Otherwise (matvec,
    # stacks, tensor parallel): queue the upload, the step and the download, then wait once.
    host_io = (not matvec) and L == 1 and pg is None and group is None
    if host_io:
        # the C-ABI call a host (the reference's Zig, any FFI) makes: tk_int4_ffn with its
        # arguments built once per weight copy, as a caller holding its buffers would
        from tiny_kernel._lib import TK_FFN_HOST_IO
        hio_args = []
        for c in range(copies):
            nw, g, u, d = mats[c][0]
            hio_args.append((dev.handle, C.c_void_p(xb_host.ptr), C.c_void_p(nw.data_ptr()),
                             C.byref(g), C.byref(u), C.byref(d), C.c_void_p(ob_host.ptr), None,
                             m, hidden, inter, GS, C.c_float(EPS), TK_FFN_HOST_IO))

    def e2e_step(i):
        if host_io:
            check(Lb.tk_int4_ffn(*hio_args[i % copies]))
            return
        check(Lb.tk_buffer_upload_async(dev.handle, xd.data_ptr(), xb_host.ptr, xb_host.nbytes,
                                        None))
        res = run_step(i, xd, (xa, xb), False, on=devstream)
        check(Lb.tk_buffer_download_async(dev.handle, ob_host.ptr, res.data_ptr(),
                                          ob_host.nbytes, None))
        check(Lb.tk_device_synchronize(dev.handle))

    # untimed: every weight copy once (a synchronous host-buffer call records its graph the first
    # time it meets a set of arguments)
    for i in range(max(3, copies)):
        e2e_step(i)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    align_ranks(pg, devstream)
    e0.record(devstream)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(devstream)
    e1.synchronize()
    e2e_ms, _ = gather_ms(pg, e0.elapsed_time(e1))
    e2e = step_bytes_total * e2e_steps / (e2e_ms / 1e3) / 1e9

    # ---- parity: one untimed step on host-generated weights against the f64 oracle -------
    parity = None
    if not args.no_parity and (matvec or host_gen):
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        res = run_step(0, x0, (xa, xb), True)
        torch.cuda.synchronize()
        y = res.cpu().numpy()
        if rank == 0:
            import oracle
            if matvec:
                ref = oracle.qmatmul_f64(x_host, M0.w, M0.s, M0.z, hidden, inter_full, GS)
                what = "qmatmul_int4 of the timed weights (copy 0)"
            else:
                ref = oracle.ffn_f64(x_host, W_full.norm_w, W_full.gate, W_full.up, W_full.down, EPS)
                what = ("the unsharded FFN" + (f", output summed over {world} ranks" if world > 1
                                               else ""))
            err = oracle.normwise_err(y, ref)
            parity = {"normwise_err": float(f"{err:.3e}"), "tol": 1e-3, "ok": bool(err <= 1e-3),
                      "checked": f"one step vs the f64 oracle of {what}"}
    elif not args.no_parity:
        parity = {"normwise_err": None, "tol": 1e-3, "ok": None,
                  "checked": "not checked: weights generated on the GPU (70B / stacks); the "
                             "-m gpu tests cover these shapes"}

    if rank == 0:
        cpu_base = None
        if world == 1 and not args.no_cpu_baseline and not matvec:
            try:
                Wc = W_full if W_full is not None else data.make_ffn(SEED, hidden, inter_full, GS)
                cpu_base = cpu_baseline_sample(Wc, x_host, m, hidden, inter_full)
            except Exception as e:
                cpu_base = {"value": None, "unit": "GB/s", "cores": None, "kind": "port",
                            "sample": f"unavailable: {e}"}
        elif world == 1 and not args.no_cpu_baseline and matvec:
            try:
                cpu_base = cpu_baseline_matvec(M0, x_host, m, hidden, inter_full)
            except Exception as e:
                cpu_base = {"value": None, "unit": "GB/s", "cores": None, "kind": "port",
                            "sample": f"unavailable: {e}"}
        traffic = (load_traffic(f"mv_m{m}") if matvec and world == 1 else
                   load_traffic(f"m{m}_tp{world}") if (args.model == "8b" and L == 1) else None)
        if path == 3:
            kern = ("tk::int4_decode_kernel (qmatmul_int4, one phase)" if matvec else
                    "tk::int4_decode_kernel (FFN: gate/up, h, down, y in one launch)")
        elif matvec:
            kern = "tk::int4_engine_kernel (qmatmul_int4, one phase)"
        elif path == 2:
            kern = ("tk::int4_gemm_kernel x2 (gate/up with silu*up, down split-K) + rmsnorm, "
                    "f16 cast, split-K reduction: the whole step")
        else:
            kern = "tk::int4_engine_kernel (FFN, gate/up then down)"
        if tensor_bound:
            roofline = {"bound": "tensor", "achieved": round(tflops, 2), "peak": peak_tc,
                        "unit": "TFLOP/s", "frac": round(tflops / peak_tc, 4),
                        "peak_kind": peak_kind + " bf16 dense (burst)", "traffic": traffic,
                        "kernel": kern, "hbm_gbs": round(achieved, 2)}
        else:
            roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                        "unit": "GB/s", "frac": round(achieved / peak, 4),
                        "peak_kind": peak_kind, "traffic": traffic, "kernel": kern,
                        "tflops": round(tflops, 2)}
        dtype, arith = arithmetic(path, m)
        if matvec:
            workload = f"INT4 matvec y[{m},{inter_full}] = x[{m},{hidden}] . W^T (qmatmul_int4)"
        else:
            workload = workload_name(name, m, L)
        line = {
            "metric": "INT4 matvec HBM GB/s" if matvec else "INT4 FFN decode HBM GB/s",
            "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": steps_timed, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
            "scaling": "weak" if matvec else "strong", "vs_baseline": None,
            "dtype": dtype, "data": "synthetic",
            "tokens_per_s": round(m * steps_timed / (ms / 1e3) * (world if matvec else 1), 1),
            # the reference bench's own figure (src/bench.zig:259-263): weight bytes only, in GiB/s
            "ref_style_gibs": round((shard_w_bytes * world if matvec else
                                     L * ffn_weight_bytes(hidden, inter_full, GS)) * steps_timed /
                                    (ms / 1e3) / 2**30, 2),
            "pct_of_peak": round(100.0 * achieved / peak, 2),
            "pct_of_8tbs": round(100.0 * achieved / 8000.0, 2),
            "config": {
                "workload": workload,
                "hidden": hidden, "inter": inter_full, "group_size": GS, "batch": m, "layers": L,
                "parallelism": (f"{world} replicas" if matvec else f"tp{world}"),
                "weight_copies": copies,
                "collective": (None if pg is None or matvec else
                               "torch.distributed NCCL all-reduce" if group is None else
                               {2: "fused into the decode kernel (peer stores over NVLink, "
                                   "rank-order sum)",
                                1: "peer-memory one-shot all-reduce kernel",
                                0: "NCCL all-reduce (library group)"}[
                                   group.ffn_exchange(m, hidden, inter, GS)]),
                "l2_guard": f"{copies} weight copies x {L} block(s) = "
                            f"{copies * L * shard_w_bytes / 1e6:.0f} MB per GPU (> 3x L2)",
                "launch": "cuda-graph" if graph is not None else "stream",
                "path": {3: "decode kernel (1-4 rows per launch)", 2: "tcgen05 GEMM",
                         1: "streaming engine"}.get(path, "CUDA-core"),
                "arithmetic": arith,
                "bytes_per_step": step_bytes_total,
                "rank_ms_per_step": [round(v / steps_timed, 6) for v in rank_ms],
            },
            "roofline": roofline,
            "cpu_baseline": cpu_base,
            "e2e": {"value": round(e2e, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": m * hidden * 4, "d2h_bytes_per_step": m * out_cols * 4,
                    "steps": e2e_steps, "ms_per_step": round(e2e_ms / e2e_steps, 5),
                    "how": ("tk_int4_ffn with TK_FFN_HOST_IO, synchronous: the kernel reads x from "
                            "and writes y to pinned host memory" if host_io else
                            "tk_buffer_upload_async + the step + tk_buffer_download_async, one "
                            "tk_device_synchronize")},
            "parity": parity,
            "gpu_launches": steps_timed * launches_per_step,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if group is not None:
        group.close()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    dev.deinit()
    if parity is not None and parity.get("ok") is False:
        sys.exit(f"parity check failed: normwise error {parity['normwise_err']} > 1e-3")


if __name__ == "__main__":
    main()
