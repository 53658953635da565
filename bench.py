"""Benchmark of the B200 INT16 engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Workloads
  conv    BASELINE config 1 batched: 64 copies of the 1x64x88x160 int16 3x3
          conv (weights U[-256,256], int32 bias U[-2^16,2^16], pad 1, seed 0);
          one step = one launch over all copies.  Unit: int16 MAC/s.

Timing follows the driver contract: W untimed warm-up steps, then K steps
bracketed by a barrier and torch.cuda.synchronize(), device time from CUDA
events on the launching stream, max over ranks.  Inputs are larger than L2
(126 MB), so no flush is needed between steps.  `value` has inputs resident
in HBM; `e2e` goes through the public C ABI with host buffers: each step
copies its input from pinned host memory, runs ufb_conv2d (NCHW, as the
reference's uf_conv) and copies the result back.

--impl reference times the reference's own CPU INT16 path (oracle/_ref,
compiled from the reference sources) on the same workload, as a bounded
sample per step, using all host threads.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONV_BATCH = 64  # copies of the config-1 conv per step


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="conv", choices=["conv"])
    return p.parse_args()


class Clocks:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    f = [x.strip() for x in line.split(",")]
                    if len(f) >= 9 and int(f[0]) < self.gpus:
                        self.rows.append(f)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.rows[0][2]), "reasons": reasons,
                "samples": len(self.rows)}


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def conv_inputs(seed=0):
    rng = np.random.default_rng(seed)
    x = rng.integers(-4096, 4097, (CONV_BATCH, 64, 88, 160)).astype(np.int16)
    w = rng.integers(-256, 257, (64, 64, 3, 3)).astype(np.int16)
    b = rng.integers(-(1 << 16), (1 << 16) + 1, (64,)).astype(np.int32)
    return x, w, b


def load_traffic(key):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        return json.load(open(path)).get(key)
    return None


# ------------------------------------------------------------------ ours ----

def bench_conv_ours(args, rank, world, local):
    import torch
    import __graft_entry__ as entry
    ufb = entry.load_package()
    L = ufb.library()
    L.ufb_probe_i8_peak.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int64)]
    L.ufb_prepare_weights.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    L.ufb_weight_bytes.restype = C.c_int64
    L.ufb_weight_bytes.argtypes = [C.c_int] * 4
    L.ufb_to_split.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                               C.c_void_p]
    L.ufb_conv2d_split.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                   C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                   C.c_void_p]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    x, w, b = conv_inputs(seed=rank)
    n, ci, h, wd = x.shape
    co = w.shape[0]
    xd = torch.from_numpy(x).to(dev)
    wdv = torch.from_numpy(w).to(dev)
    bd = torch.from_numpy(b).to(dev)
    xs = torch.empty(n * h * wd * 2 * ci, dtype=torch.uint8, device=dev)
    os_ = torch.empty(n * h * wd * 2 * co, dtype=torch.uint8, device=dev)
    planes = torch.empty(L.ufb_weight_bytes(co, ci, 3, 3), dtype=torch.uint8, device=dev)
    assert L.ufb_prepare_weights(wdv.data_ptr(), co, ci, 3, 3, planes.data_ptr(), sp) == 0
    assert L.ufb_to_split(xd.data_ptr(), n, ci, h, wd, 1, xs.data_ptr(), ci, sp) == 0

    def step():
        rc = L.ufb_conv2d_split(xs.data_ptr(), n, ci, h, wd, ci, planes.data_ptr(), co, 3, 3, bd.data_ptr(), 32, 1,
                                1, os_.data_ptr(), co, sp)
        if rc:
            raise RuntimeError(L.ufb_last_error().decode())

    # int8 tensor-pipe peak, measured live with the dense kind::i8 probe
    ops = C.c_int64()
    for _ in range(2):
        L.ufb_probe_i8_peak(4000, 148, sp, C.byref(ops))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    L.ufb_probe_i8_peak(4000, 148, sp, C.byref(ops))
    e1.record(stream)
    torch.cuda.synchronize()
    peak_tops = ops.value / (e0.elapsed_time(e1) * 1e-3) / 1e12

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the sampler runs through warm-up and timed steps (a step lasts under 1 ms,
    # shorter than one nvidia-smi query), so its samples see the same load
    with Clocks(max(world, 1)) as clk:
        for _ in range(max(args.warmup, 3)):
            step()
        t_end = time.time() + 0.5
        while time.time() < t_end:
            step()
            torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    clocks = clk.summary()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, world, dev)
    if ufb.device_status(local) != 0:
        raise RuntimeError("kernel pipeline timeout")

    # end to end through the public NCHW C ABI with host buffers
    xh = torch.from_numpy(x).pin_memory()
    oh_ = torch.empty((n, co, h, wd), dtype=torch.int16).pin_memory()
    out_d = torch.empty((n, co, h, wd), dtype=torch.int16, device=dev)

    def e2e_step():
        xd.copy_(xh, non_blocking=True)
        rc = L.ufb_conv2d(xd.data_ptr(), n, ci, h, wd, wdv.data_ptr(), co, 3, 3, bd.data_ptr(), 32, 1, 1, 1, 1, 1,
                          out_d.data_ptr(), sp)
        if rc:
            raise RuntimeError(L.ufb_last_error().decode())
        oh_.copy_(out_d, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev)
    # parity spot check of the last e2e output against the CPU checker (one image)
    import oracle
    want = oracle.c_oracle().conv2d(x[:1], w, b, 1, 1)
    if not np.array_equal(oh_[:1].numpy(), want):
        raise RuntimeError("bench output differs from the CPU oracle")

    macs = n * co * h * wd * ci * 9
    value = world * macs / (ms_max * 1e-3)
    achieved_tops = 8 * macs / (ms * 1e-3) / 1e12
    res = {
        "metric": "INT16 3x3 conv int16-MAC/s (BASELINE config 1 shape, 64 copies per step)",
        "value": value, "unit": "MAC/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int16 (int8 planes, s32 accumulators, int64 recombination)", "data": "synthetic (seeded)",
        "config": {"workload": "config-1 conv 64x[1x64x88x160] 3x3 64->64 int32 bias, pad 1",
                   "batch": CONV_BATCH, "l2": "inputs larger than L2 (115 MB in + 115 MB out per step)",
                   "parallelism": f"replicas x{world}"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "roofline": {"bound": "tensor", "achieved": achieved_tops, "peak": peak_tops, "unit": "TOPS(int8)",
                     "frac": achieved_tops / peak_tops, "traffic": load_traffic("conv_config1_b64"),
                     "peak_source": "measured live: dense tcgen05 kind::i8 probe (ufb_probe_i8_peak)",
                     "algorithmic": "8 int8 ops per int16 MAC"},
        "e2e": {"value": world * macs / (e2e_ms * 1e-3), "unit": "MAC/s",
                "h2d_bytes_per_step": int(x.nbytes), "d2h_bytes_per_step": int(n * co * h * wd * 2)},
    }
    return res


def cpu_baseline_conv(threads):
    """Reference conv2d_reference (oracle/_ref) on a bounded sample: 8 of the 64 copies."""
    import oracle
    ref = oracle.ref_oracle()
    ref.set_threads(threads)
    x, w, b = conv_inputs(0)
    sample = 8
    ref.conv2d(x[:1], w, b, 1, 1)
    t0 = time.perf_counter()
    ref.conv2d(x[:sample], w, b, 1, 1)
    dt = time.perf_counter() - t0
    macs = sample * 64 * 88 * 160 * 64 * 9
    return {"value": macs / dt, "unit": "MAC/s", "cores": threads, "kind": "reference",
            "sample": f"{sample} of {CONV_BATCH} config-1 convs through the reference conv2d_reference "
                      f"({dt:.2f} s)"}


def main():
    args = parse()
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        base = cpu_baseline_conv(threads)
        steps = []
        for _ in range(args.steps):
            steps.append(cpu_baseline_conv(threads)["value"])
        value = statistics.median(steps)
        print(json.dumps({
            "impl": "reference", "metric": "INT16 3x3 conv int16-MAC/s (BASELINE config 1 shape, 64 copies per step)",
            "value": value, "unit": "MAC/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "int16", "data": "synthetic (seeded)",
            "config": {"workload": "config-1 conv 64x[1x64x88x160] 3x3 64->64 int32 bias, pad 1"},
            "cpu_baseline": dict(base, value=value),
            "e2e": {"value": value, "unit": "MAC/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    res = bench_conv_ours(args, rank, world, local)
    if rank == 0:
        res["cpu_baseline"] = cpu_baseline_conv(1)
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
