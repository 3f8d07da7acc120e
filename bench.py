#!/usr/bin/env python
"""INT4 FFN decode benchmark on B200: HBM GB/s (% of peak) and tokens/s.

Workload (default, one GPU): the Llama-3-8B-shaped INT4 FFN at batch 1 --
rmsnorm(eps 1e-5) -> gate/up INT4 GEMV (4096 -> 14336) -> silu(gate)*up -> down INT4 GEMV
(14336 -> 4096) in f32 -- on seeded synthetic inputs in the reference qmatmul_int4 layout
(group 64, f16 scales, 4-bit zero points).  One step = one FFN forward = one launch of the
persistent engine.  With --gpus N (torchrun, one rank per GPU) the FFN is tensor-parallel:
gate/up column-split, down row-split, one NCCL all-reduce of the f32 partial outputs.

value     whole-job algorithmic GB/s: FFN bytes (weights + x + norm weight + out) per step
          x steps / max-over-ranks device time; inputs resident in HBM; L2 defeated by
          rotating several weight copies whose total exceeds 3x the L2 size.
e2e       the same metric through the synchronous C ABI (tk_int4_ffn) with the activation
          copied from pinned host memory and the output read back every step.
--impl reference  times the CPU transcription of the reference shaders (oracle/), all host
          threads, on the same workload (the reference itself is Zig + Metal and cannot run
          on this Linux host).
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


def ffn_bytes(m, hidden, inter, gs):
    from tiny_kernel.data import int4_matrix_bytes
    w = 2 * int4_matrix_bytes(hidden, inter, gs) + int4_matrix_bytes(inter, hidden, gs)
    return w + m * hidden * 4 + hidden * 4 + m * hidden * 4


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(m, n_gpus):
    """Per-launch DRAM bytes of the engine from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "int4_ffn_engine_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(f"m{m}_tp{n_gpus}")
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
    W = data.make_ffn(SEED, HIDDEN, INTER, GS)
    x = data.make_x(SEED, "x", m, HIDDEN)
    threads = cpu.default_threads()
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
    nbytes = ffn_bytes(m, HIDDEN, INTER, GS)
    gbs = nbytes * steps / dt / 1e9
    line = {
        "impl": "reference", "metric": "INT4 FFN decode HBM GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(dt / steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tokens_per_s": round(m * steps / dt, 2),
        "config": {"workload": f"Llama-3-8B INT4 FFN decode (rmsnorm->gate/up->silu*up->down), batch {m}",
                   "hidden": HIDDEN, "inter": INTER, "group_size": GS, "batch": m,
                   "parallelism": "host CPU", "steps_requested": args.steps},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} full FFN steps (the reference's Metal shaders cannot "
                                   f"run here: Zig + Metal; this is their C++ std::thread "
                                   f"transcription, oracle/cpu_baseline.cpp)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(W, x, m):
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
    return {"value": round(ffn_bytes(m, HIDDEN, INTER, GS) * n / dt / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{n} full FFN steps on the host ({dt:.1f} s), C++ std::thread transcription "
                      f"of the reference shaders (oracle/cpu_baseline.cpp)"}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import tiny_kernel as tk
    from tiny_kernel import data, ops
    from tiny_kernel.tp import shard_ffn

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    dev = tk.init(local)
    m = args.batch
    W_full = data.make_ffn(SEED, HIDDEN, INTER, GS)
    W = shard_ffn(W_full, rank, world)
    inter = W.inter
    x_host = data.make_x(SEED, "x", m, HIDDEN)

    def to_dev(a):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(a).cuda()

    step_bytes_total = ffn_bytes(m, HIDDEN, INTER, GS)
    shard_bytes = sum(M.nbytes for M in (W.gate, W.up, W.down))
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    copies = max(4, math.ceil(3 * l2 / shard_bytes))
    base = [to_dev(a) for M in (W.gate, W.up, W.down) for a in (M.w, M.s, M.z)]
    sets = [base] + [[t.clone() for t in base] for _ in range(copies - 1)]
    mats = [[ops.matrix(*s[3 * j:3 * j + 3]) for j in range(3)] for s in sets]
    nw = to_dev(W.norm_w)
    x = to_dev(x_host)
    out = torch.empty((m, HIDDEN), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step(i):
        g, u, d = mats[i % copies]
        ops.int4_ffn(dev, x, nw, g, u, d, out, m, HIDDEN, inter, GS, eps=EPS,
                     stream=stream.cuda_stream, sync=False)
        if pg is not None:
            with torch.cuda.stream(stream):
                pg.all_reduce(out)

    # warm-up (also sizes the engine's scratch before any capture)
    for i in range(args.warmup):
        step(i)
    stream.synchronize()
    dev.synchronize()

    graph = None
    if not args.no_graph and pg is None:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(args.steps):
                    step(i)
            graph.replay()
            stream.synchronize()
        except Exception as e:  # capture unsupported: fall back to stream launches
            print(f"# graph capture failed ({e}); timing stream launches", file=sys.stderr)
            graph = None
            torch.cuda.synchronize()
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        if graph is not None:
            with torch.cuda.stream(stream):
                graph.replay()
        else:
            for i in range(args.steps):
                step(i)
        ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if pg is not None:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    from tiny_kernel._lib import check, lib
    check(lib().tk_device_check_error(dev.handle))
    ms_per_step = ms / args.steps
    value = step_bytes_total * args.steps / (ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    per_gpu_bytes = shard_bytes + m * HIDDEN * 4 * 2 + HIDDEN * 4
    achieved = per_gpu_bytes / (ms_per_step / 1e3) / 1e9

    # ---- end to end through the synchronous C ABI with host buffers -------------------
    import ctypes as C
    L = lib()
    xb = tk.Buffer(dev, "f32", m * HIDDEN, kind=2)   # pinned host
    ob = tk.Buffer(dev, "f32", m * HIDDEN, kind=2)
    np.copyto(np.frombuffer((C.c_char * xb.nbytes).from_address(xb.ptr), np.float32), x_host.reshape(-1))
    xd = torch.empty((m, HIDDEN), dtype=torch.float32, device="cuda")
    e2e_steps = min(args.steps, 2000)
    for i in range(5):
        check(L.tk_buffer_upload(dev.handle, xd.data_ptr(), xb.ptr, xb.nbytes))
        g, u, d = mats[i % copies]
        ops.int4_ffn(dev, xd, nw, g, u, d, out, m, HIDDEN, inter, GS, eps=EPS)
        if pg is not None:
            pg.all_reduce(out)
        check(L.tk_buffer_download(dev.handle, ob.ptr, out.data_ptr(), ob.nbytes))
    if pg is not None:
        pg.barrier()
    devstream = torch.cuda.ExternalStream(dev.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(devstream)
    for i in range(e2e_steps):
        check(L.tk_buffer_upload(dev.handle, xd.data_ptr(), xb.ptr, xb.nbytes))
        g, u, d = mats[i % copies]
        ops.int4_ffn(dev, xd, nw, g, u, d, out, m, HIDDEN, inter, GS, eps=EPS)
        if pg is not None:
            pg.all_reduce(out)
            torch.cuda.current_stream().synchronize()
        check(L.tk_buffer_download(dev.handle, ob.ptr, out.data_ptr(), ob.nbytes))
    e1.record(devstream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if pg is not None:
        t = torch.tensor([e2e_ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = step_bytes_total * e2e_steps / (e2e_ms / 1e3) / 1e9

    if rank == 0:
        cpu_base = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                cpu_base = cpu_baseline_sample(W_full, x_host, m)
            except Exception as e:
                cpu_base = {"value": None, "unit": "GB/s", "cores": None, "kind": "port",
                            "sample": f"unavailable: {e}"}
        line = {
            "metric": "INT4 FFN decode HBM GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "tokens_per_s": round(m * args.steps / (ms / 1e3), 1),
            "pct_of_peak": round(100.0 * achieved / peak, 2),
            "pct_of_8tbs": round(100.0 * achieved / 8000.0, 2),
            "config": {
                "workload": f"Llama-3-8B INT4 FFN decode (rmsnorm->gate/up->silu*up->down), batch {m}",
                "hidden": HIDDEN, "inter": INTER, "group_size": GS, "batch": m,
                "parallelism": f"tp{world}", "weight_copies": copies,
                "l2_guard": f"{copies} rotating weight copies = {copies * shard_bytes / 1e6:.0f} MB per GPU (> 3x L2)",
                "launch": "cuda-graph" if graph is not None else "stream",
                "bytes_per_step": step_bytes_total,
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": peak_kind, "traffic": load_traffic(m, world),
                         "kernel": "tk::int4_engine_kernel (FFN, 2 phases)"},
            "cpu_baseline": cpu_base,
            "e2e": {"value": round(e2e, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": m * HIDDEN * 4, "d2h_bytes_per_step": m * HIDDEN * 4,
                    "steps": e2e_steps, "ms_per_step": round(e2e_ms / e2e_steps, 5)},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    dev.deinit()


if __name__ == "__main__":
    main()
