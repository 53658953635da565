"""Benchmark of the B200 INT16 engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Workloads
  decode  (default) BASELINE config 5: 64 independent seeded synthetic 1920x1088
          sequences of 32 frames (config-4 scene generator, seeds 100..163), each
          coded as 1 I packet (qp_i 0) + 4 P packets of 8 frames (qp_p 20,
          reset_interval 8 -> every P packet resets, skip 0.2), sharded
          64/N streams per GPU with no inter-GPU communication.  One step decodes
          every sequence of the rank completely (I packet, then the 4 P packets),
          host rANS included.  Unit: decoded frames/s (whole job).  At N=1 the
          line also carries `secondary`: the same decode at 626x352 (BASELINE
          configs 3-4; 64 sequences, seeds 3..66), the single-stream 120-frame
          config-4 GOP, the per-P-packet latency, and the reference CPU decode
          time of the config-3 packets when tests/golden/config3.json has it.
  conv    BASELINE config 1 batched: 64 copies of the 1x64x88x160 int16 3x3 conv.
  warp    BASELINE config 2: the fixed-point backward bilinear warp of int16
          features 1x64x176x320 by an int16 Q9 flow (N(0, 4^2) px per pixel plus a
          (3.25, -1.5) px translation, seed 1).  Unit: warps/s; roofline: HBM
          bytes (7.21 MB features + 0.225 MB flow + 7.21 MB output per call) over
          the measured copy bandwidth; L2 (126 MB) is flushed by a 256 MB write
          before every timed call.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize(), device time from CUDA events on the stream the
engine launches on, max over ranks.  The decoder's working set per step is
several GB (far above the 126 MB L2).  `value` leaves decoded frames in HBM;
`e2e` decodes through the same public C ABI and also converts every frame to
8-bit YUV420 (IntegerCodec::raw_frame) and copies it to pinned host memory.
Payloads always start in host memory (the entropy decoder runs on the host,
as in the reference).

--impl reference times the reference's own CPU INT16 decoder
(IntegerModel::decompress from oracle/_ref, compiled from the reference
sources) with all host threads on a bounded sample -- one P packet and one I
packet at 128x128 -- and extrapolates to the workload by pixel count.
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
from concurrent.futures import ThreadPoolExecutor
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONV_BATCH = 64
SEQS, FRAMES, W1080, H1080 = 64, 32, 1920, 1088
QP_I, QP_P, SKIP = 0, 20, 0.2
SAMPLE = 128  # reference sample resolution (pixels per side)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="decode", choices=["decode", "conv", "warp"])
    p.add_argument("--seqs", type=int, default=SEQS,
                   help="sequences in the job (default: BASELINE config 5's 64); smaller values are for profiling")
    p.add_argument("--shapes", action="store_true", help="print per launch shape convolution time to stderr")
    p.add_argument("--no-secondary", action="store_true", help="skip the 626x352 measurements (decode workload, N=1)")
    p.add_argument("--groups", type=int, default=2,
                   help="concurrent codec groups per rank (each with its own CUDA stream and host thread)")
    return p.parse_args()


class Clocks:
    """Samples nvidia-smi SM clocks and throttle reasons while the GPU is loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout
                for line in out.strip().splitlines():
                    f = [x.strip() for x in line.split(",")]
                    if len(f) >= 9:
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
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.rows[0][2]), "reasons": reasons,
                "samples": len(self.rows)}


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_over_ranks(value, world, device, op):
    """Max / sum of a host scalar over the ranks.  The ranks share no data: the
    group is gloo over host memory, so a multi-GPU run makes no NCCL call."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def merged_shapes(codecs):
    """The profiled launches of several codecs by shape and epilogue:
    {shape: [launches, int16 MACs, ms, algorithmic DRAM bytes]}."""
    table = {}
    for c in codecs:
        for k, v in c.shape_table().items():
            t = table.setdefault(k, [0, 0.0, 0.0, 0.0])
            for i in range(4):
                t[i] += v[i]
    return table


def print_shapes(table, frames):
    """Per launch shape convolution time of the profiled step, to stderr."""
    total = sum(t[2] for t in table.values())
    print(f"# shape  launches  ms  share  int8-TOPS  GB/s  ({frames} frames)", file=sys.stderr)
    for k, (n, macs, ms, hbm) in sorted(table.items(), key=lambda kv: -kv[1][2]):
        tops = 8 * macs / (ms * 1e-3) / 1e12 if ms else 0.0
        gbs = hbm / (ms * 1e-3) / 1e9 if ms else 0.0
        print(f"{k:52s} {n:6d} {ms:9.2f} {ms / total * 100:5.1f}% {tops:7.0f} {gbs:7.0f}", file=sys.stderr)


def launch_rooflines(table, peak_tops, hbm_gbs, step_ms):
    """Roofline of every profiled launch: the slower of its int8 MMA time at
    peak_tops and its algorithmic DRAM bytes at hbm_gbs.  Returns the
    tensor-core convolutions' summed floor against their summed event time
    and the depthwise launches' DRAM throughput."""
    floor = meas = hbm_ms = 0.0
    for k, (n, macs, ms, hbm) in table.items():
        if not k.startswith("conv") or not ms:
            continue
        t_tensor = 8 * macs / (peak_tops * 1e12) * 1e3
        t_hbm = hbm / (hbm_gbs * 1e9) * 1e3
        floor += max(t_tensor, t_hbm)
        meas += ms
        if t_hbm > t_tensor:
            hbm_ms += ms
    dw = [v for k, v in table.items() if k.startswith("depthwise")]
    dw_ms = sum(v[2] for v in dw)
    dw_bytes = sum(v[3] for v in dw)
    conv = {"frac": floor / meas if meas else None, "floor_ms": floor, "measured_ms": meas,
            "hbm_bound_time_share": hbm_ms / meas if meas else None,
            "peak_tops": peak_tops, "hbm_gbs": hbm_gbs,
            "rule": "per launch the slower of its int8 MMA time at the sustained probe peak and its algorithmic "
                    "DRAM bytes (input and residuals read once, output written once, weights) at the measured "
                    "copy bandwidth; summed over the step's tensor-core convolutions and divided by their "
                    "summed event time"}
    depth = None
    if dw_ms:
        depth = {"launches": int(sum(v[0] for v in dw)), "ms": dw_ms,
                 "share_of_serial_step": dw_ms / step_ms if step_ms else None,
                 "achieved_gbs": dw_bytes / (dw_ms * 1e-3) / 1e9,
                 "frac": dw_bytes / (dw_ms * 1e-3) / 1e9 / hbm_gbs, "bound": "hbm", "peak_gbs": hbm_gbs,
                 "algorithmic": "input read once, output written once (both byte planes), weights"}
    return conv, depth


def load_traffic(key):
    """DRAM bytes per launch recorded in a profile summary (a line `key: N` in
    profiles/*.md, written from an ncu capture of the same workload), or None."""
    import glob
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        for line in open(path):
            if line.startswith(key + ":"):
                return float(line.split(":", 1)[1].split()[0])
    return None


def i8_peak_tops(L, stream):
    """int8 tensor-pipe peak measured live with the dense kind::i8 probe."""
    import torch
    L.ufb_probe_i8_peak.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int64)]
    sp = C.c_void_p(stream.cuda_stream)
    ops = C.c_int64()
    for _ in range(2):
        L.ufb_probe_i8_peak(4000, 148, sp, C.byref(ops))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    L.ufb_probe_i8_peak(4000, 148, sp, C.byref(ops))
    e1.record(stream)
    torch.cuda.synchronize()
    return ops.value / (e0.elapsed_time(e1) * 1e-3) / 1e12


def i8_peak_sustained(L, stream, local, seconds=3.0):
    """int8 tensor-pipe peak under the power cap: the dense probe back to back
    for `seconds` (as the driver's sustained bf16 figure is taken), with the
    SM clocks sampled meanwhile.  Returns (TOPS, clock summary)."""
    import time
    import torch
    sp = C.c_void_p(stream.cuda_stream)
    ops = C.c_int64()
    total = 0
    with Clocks(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t0 = time.time()
        while time.time() - t0 < seconds:
            for _ in range(20):
                if L.ufb_probe_i8_peak(40000, 148, sp, C.byref(ops)):
                    raise RuntimeError(L.ufb_last_error().decode())
                total += ops.value
            torch.cuda.synchronize()
        e1.record(stream)
        torch.cuda.synchronize()
    return total / (e0.elapsed_time(e1) * 1e-3) / 1e12, clk.summary()


# --------------------------------------------------------------- decode ----

def shard(rank, world, seqs):
    per = max(seqs // world, 1)
    return list(range(rank * per, (rank + 1) * per))


def p_packets(frames):
    return (frames - 1 + 7) // 8


def encode_sequences(ufb, syn, mi, mv, seqs, batch, dev, width=W1080, height=H1080, frames=FRAMES, seed_base=100):
    """Seeded synthetic sequences coded by this engine's encoder (untimed
    setup).  Per group of streams: ids, I payloads, the I-frame reconstruction
    of the encoder, the lists of P payloads, their reset flags and the SHA-256
    of the encoder's decoded-picture-buffer states after the last P packet."""
    import torch
    groups = []
    for g0 in range(0, len(seqs), batch):
        ids = seqs[g0:g0 + batch]
        video = torch.stack([syn.synthetic_video_gpu(width, height, frames, seed_base + s, dev) for s in ids])
        ci = ufb.Codec(mi, len(ids))
        ci.set_skip_threshold(SKIP)
        cv = ufb.Codec(mv, len(ids))
        cv.set_skip_threshold(SKIP)
        i_pay, i_rec = ci.compress(video[:, 0].cpu().numpy(), QP_I, frames=True)
        cv.set_reference_from(ci)
        p_pays, resets = [], []
        count = 1
        for k in range(p_packets(frames)):
            chunk = video[:, 1 + 8 * k: 9 + 8 * k]
            if chunk.shape[1] < 8:  # pad by repeating the last frame (src/integer_codec.cpp:257-261)
                chunk = torch.cat([chunk] + [chunk[:, -1:]] * (8 - chunk.shape[1]), 1)
            reset = (count + 8) % 8 == 1  # reset_interval 8 (src/integer_codec.cpp:263-264)
            pay, _ = cv.compress(chunk.reshape(len(ids), 24, height, width).cpu().numpy(), QP_P, reset)
            p_pays.append(pay)
            resets.append(reset)
            count += 8
        states = {k: cv.state_hash(k) for k in ("reference", "memory", "context")}
        groups.append((ids, i_pay, i_rec if g0 == 0 else None, p_pays, resets, states))
        del video
    return groups


def bench_decode_ours(args, rank, world, local):
    import torch
    import __graft_entry__ as entry
    ufb = entry.load_package()
    syn = entry.load_synthetic()
    L = ufb.library()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    seqs = shard(rank, world, args.seqs)
    # at least two codec groups per rank (when it has two streams), so host rANS overlaps GPU work
    groups_wanted = max(2, args.groups)
    batch = max(1, (len(seqs) + groups_wanted - 1) // groups_wanted)
    mi = ufb.Model("image", syn.prepared("image", 1), device=local)
    mv = ufb.Model("htl", syn.prepared("htl", 2), device=local)
    groups = encode_sequences(ufb, syn, mi, mv, seqs, batch, dev)
    peak = i8_peak_tops(L, stream)

    decoders, sinks = [], []
    yuv_bytes = W1080 * H1080 * 3 // 2
    # one CUDA stream and one host thread per codec group: while one group waits
    # on its host rANS, the other group's kernels keep the GPU busy
    gstreams = [torch.cuda.Stream(dev) for _ in groups]
    pool = ThreadPoolExecutor(max_workers=len(groups))
    for (ids, *_), gs in zip(groups, gstreams):
        di, dv = ufb.Codec(mi, len(ids)), ufb.Codec(mv, len(ids))
        for c in (di, dv):
            c.set_skip_threshold(SKIP)
            c.set_stream(gs)
        decoders.append((di, dv))
        # page-locked YUV sinks, reused by every packet (a decoder's output ring)
        sinks.append(tuple(torch.empty((len(ids), f, yuv_bytes), dtype=torch.uint8, pin_memory=True).numpy()
                           for f in (1, 8)))

    host_s = [0.0] * len(groups)  # host entropy-coding seconds per codec group (Codec::host_seconds)

    def decode_group(g, yuv):
        """One codec group: I packet, then the 4 P packets of each of its streams."""
        (ids, i_pay, _, p_pays, resets, _), (di, dv), (si, sp) = groups[g], decoders[g], sinks[g]
        di.decompress(i_pay, W1080, H1080, QP_I, frames=False, yuv_out=si if yuv else None)
        host_s[g] += di.host_seconds()
        dv.set_reference_from(di)
        frames = len(ids)
        for k in range(4):
            dv.decompress(p_pays[k], W1080, H1080, QP_P, resets[k], frames=False, yuv_out=sp if yuv else None)
            host_s[g] += dv.host_seconds()
            frames += len(ids) * (8 if k < 3 else FRAMES - 1 - 24)
        return frames

    def step(yuv, concurrent=True):
        """Decode every sequence of this rank, the codec groups concurrently."""
        if not concurrent:
            return sum(decode_group(g, yuv) for g in range(len(groups)))
        return sum(pool.map(lambda g: decode_group(g, yuv), range(len(groups))))

    def timed(yuv, steps, profile=False):
        """Device time of `steps` steps.  profile=True brackets every tensor-core
        convolution with CUDA events and runs the groups one after the other, so
        that each event pair measures that convolution alone."""
        for pair in decoders:
            for c in pair:
                c.stats(reset=True)
                c.profile(profile)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed_e2e" if yuv else "timed")  # ncu --nvtx-include "timed/"
        e0.record(stream)
        for gs in gstreams:
            gs.wait_event(e0)
        frames = sum(step(yuv, concurrent=not profile) for _ in range(steps))
        for gs in gstreams:
            stream.wait_stream(gs)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        barrier(world)
        st = {"launches": 0, "conv_launches": 0, "conv_int16_macs": 0.0, "conv_ms": 0.0}
        if profile:
            st["shapes"] = merged_shapes([c for pair in decoders for c in pair])
            if args.shapes:
                print_shapes(st["shapes"], frames)
        for pair in decoders:
            for c in pair:
                s = c.stats()
                c.profile(False)
                for k in s:
                    st[k] += s[k]
        return frames, e0.elapsed_time(e1), st

    with Clocks(local) as clk:
        for _ in range(args.warmup):
            step(False)
        torch.cuda.synchronize()
        for g in range(len(groups)):
            host_s[g] = 0.0
        frames, ms, st = timed(False, args.steps)
        host_per_step = [x / args.steps for x in host_s]
    clocks = clk.summary()
    # roofline of the tensor-core convolutions: one more step, groups in turn,
    # every convolution bracketed by events (not part of the timed value)
    prof_frames, prof_ms, pst = timed(False, 1, profile=True)
    # the convolutions above run inside a long step under the power cap: their
    # denominator is the probe's sustained rate (the burst rate is kept beside it)
    peak_burst = peak
    peak, peak_clocks = i8_peak_sustained(L, stream, local)
    ms_max = reduce_over_ranks(ms, world, dev, "max")
    total_frames = reduce_over_ranks(frames, world, dev, "sum")

    # integrity checks: after the last decoded step every group's decoder holds
    # the encoder's decoded-picture-buffer states (which depend on every P
    # packet's reconstruction), and the I packet decodes to the encoder's frame
    for g, (_, dv) in enumerate(decoders):
        for k, want in groups[g][5].items():
            if dv.state_hash(k) != want:
                raise RuntimeError(f"group {g}: decoder {k} state after the P packets differs from the encoder's")
    _, i_pay, i_rec, _, _, _ = groups[0]
    got_i, _ = decoders[0][0].decompress(i_pay, W1080, H1080, QP_I, frames=True)
    if not np.array_equal(got_i, i_rec):
        raise RuntimeError("I-packet decode differs from the encoder reconstruction")

    e2e_frames, e2e_ms, _ = timed(True, 1)
    e2e_ms = reduce_over_ranks(e2e_ms, world, dev, "max")
    e2e_total = reduce_over_ranks(e2e_frames, world, dev, "sum")
    h2d = sum(len(p) for g in groups for p in list(g[1]) + [x for pp in g[3] for x in pp])
    d2h = len(seqs) * 33 * W1080 * H1080 * 3 // 2  # every decoded frame (incl. the padding frame) as YUV420

    per_step_ms = ms / args.steps
    achieved = 8 * pst["conv_int16_macs"] / (pst["conv_ms"] * 1e-3) / 1e12 if pst["conv_ms"] else None
    hbm, hbm_src = hbm_peak()
    per_launch, depthwise = launch_rooflines(pst["shapes"], peak, hbm, prof_ms)
    secondary = None
    if world == 1 and not args.no_secondary:
        del decoders, sinks
        secondary = bench_626(ufb, syn, mi, mv, dev, stream, peak)
    return {
        "metric": "INT16 HT-L decoded frames/s (1920x1088, BASELINE config 5)",
        "value": total_frames / (ms_max * 1e-3), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int16 (int8 tensor planes, s32 accumulators, exact 32-bit rna recombination)",
        "data": "synthetic (seeded scene generator, seeded random-init HT-L + image models)",
        "config": {"workload": f"config 5: {len(seqs) * world} seqs x 32 frames 1920x1088, I + 4 P packets each, "
                               "qp_i 0 qp_p 20, reset 8, skip 0.2", "streams_per_gpu": len(seqs), "codec_batch": batch,
                   "codec_groups": f"{len(groups)} concurrent (one CUDA stream and host thread each)",
                   "l2": "working set per step several GB, far above L2",
                   "parallelism": f"stream sharding x{world}, no inter-GPU communication"},
        "gpu_launches": int(st["launches"]),
        "clocks": clocks,
        "host": {"entropy_seconds_per_step_per_group": host_per_step,
                 "note": "host rANS (and its device<->host hand-offs) of each concurrent codec group per timed "
                         "step (Codec host_seconds), beside ms_per_step: where a rank's host work approaches "
                         "its step time, the host, not the GPU, bounds that rank"},
        "roofline": {"bound": "tensor", "kernel": "conv_i16_tc_kernel (all tensor-core convolution launches)",
                     "achieved": achieved, "peak": peak, "unit": "TOPS(int8)",
                     "frac": achieved / peak if achieved else None,
                     "peak_burst": peak_burst, "frac_of_burst": achieved / peak_burst if achieved else None,
                     "peak_clocks": peak_clocks,
                     # the probe holds its clock while the decode runs power-capped: the
                     # peak scaled by (step clock / probe clock), for reference only
                     "frac_at_step_clock": (achieved / (peak * clocks["sm_mhz"] / peak_clocks["sm_mhz"])
                                            if achieved and clocks.get("sm_mhz") and peak_clocks.get("sm_mhz")
                                            else None),
                     "traffic": load_traffic("htl_conv_res512_per_launch"),
                     "traffic_source": "from profile: ncu capture of an HT-L module run "
                                       "(profiles/conv_i16_tc_htl_blocks.md), not this run",
                     "traffic_launch": "DRAM read + write of one 512->512 residual-epilogue launch over 130560 "
                                       "pixels; algorithmic 401.1 MB (input, residual, output)",
                     "peak_source": "measured live: dense tcgen05 kind::i8 probe (ufb_probe_i8_peak) back to back "
                                    "for 3 s (sustained, the convolutions run inside a long step); peak_burst: "
                                    "one 1 ms probe",
                     "algorithmic": "8 int8 ops per int16 MAC",
                     "measured_on": "one extra step with the codec groups in turn, every convolution "
                                    "bracketed by CUDA events on its stream",
                     "conv_share_of_serial_step": pst["conv_ms"] / prof_ms if prof_ms else None,
                     "conv_launches_per_step": pst["conv_launches"],
                     "conv_int16_macs_per_step": pst["conv_int16_macs"],
                     # the same launches against each one's own bound (tensor or DRAM)
                     "per_launch_roofline": dict(per_launch, hbm_source=hbm_src)},
        "depthwise": depthwise,
        "e2e": {"value": e2e_total / (e2e_ms * 1e-3), "unit": "frames/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "secondary": secondary,
    }


def bench_626(ufb, syn, mi, mv, dev, stream, peak):
    """626x352: the config-5 multi-stream decode at the
    smaller frame size (64 sequences x 32 frames, seeds 3..66) and the
    single-stream 120-frame config-4 GOP (seed 3), with per-packet latency."""
    import torch
    W, H = 626, 352
    out = {"metric": "INT16 HT-L decoded frames/s (626x352, BASELINE configs 3-4)", "unit": "frames/s"}

    # multi-stream throughput: two concurrent codec groups, as the main workload
    groups = encode_sequences(ufb, syn, mi, mv, list(range(SEQS)), SEQS // 2, dev, W, H, FRAMES, seed_base=3)
    gstreams = [torch.cuda.Stream(dev) for _ in groups]
    decoders = []
    for (ids, *_), gs in zip(groups, gstreams):
        pair = ufb.Codec(mi, len(ids)), ufb.Codec(mv, len(ids))
        for c in pair:
            c.set_skip_threshold(SKIP)
            c.set_stream(gs)
        decoders.append(pair)
    pool = ThreadPoolExecutor(max_workers=len(groups))

    def decode_group(g):
        (ids, i_pay, _, p_pays, resets, _), (di, dv) = groups[g], decoders[g]
        di.decompress(i_pay, W, H, QP_I, frames=False)
        dv.set_reference_from(di)
        n = len(ids)
        for k, pay in enumerate(p_pays):
            dv.decompress(pay, W, H, QP_P, resets[k], frames=False)
            n += len(ids) * min(8, FRAMES - 1 - 8 * k)
        return n

    def run(steps, profile=False):
        for pair in decoders:
            for c in pair:
                c.stats(reset=True)
                c.profile(profile)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for gs in gstreams:
            gs.wait_event(e0)
        if profile:
            n = sum(decode_group(g) for _ in range(steps) for g in range(len(groups)))
        else:
            n = sum(sum(pool.map(decode_group, range(len(groups)))) for _ in range(steps))
        for gs in gstreams:
            stream.wait_stream(gs)
        e1.record(stream)
        torch.cuda.synchronize()
        st = {"conv_int16_macs": 0.0, "conv_ms": 0.0}
        if profile:
            st["shapes"] = merged_shapes([c for pair in decoders for c in pair])
        for pair in decoders:
            for c in pair:
                x = c.stats()
                c.profile(False)
                for k in ("conv_int16_macs", "conv_ms"):
                    st[k] += x[k]
        return n, e0.elapsed_time(e1), st

    run(2)
    frames, ms, _ = run(3)
    _, prof_ms, pst = run(1, profile=True)
    for g, (_, dv) in enumerate(decoders):
        for k, want in groups[g][5].items():
            if dv.state_hash(k) != want:
                raise RuntimeError(f"626x352 group {g}: decoder {k} state differs from the encoder's")
    achieved = 8 * pst["conv_int16_macs"] / (pst["conv_ms"] * 1e-3) / 1e12 if pst["conv_ms"] else None
    hbm, _ = hbm_peak()
    per_launch, depthwise = launch_rooflines(pst["shapes"], peak, hbm, prof_ms)
    out["multi_stream"] = {
        "value": frames / (ms * 1e-3), "unit": "frames/s", "ms_per_step": ms / 3, "steps": 3,
        "workload": f"{SEQS} seqs x {FRAMES} frames 626x352 (seeds 3..{2 + SEQS}), I + 4 P packets each, "
                    "qp_i 0 qp_p 20, reset 8, skip 0.2, two concurrent codec groups",
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS(int8)",
                     "frac": achieved / peak if achieved else None,
                     "per_launch_roofline_frac": per_launch["frac"],
                     "hbm_bound_time_share": per_launch["hbm_bound_time_share"],
                     "measured_on": "one extra step, groups in turn, every tensor-core convolution bracketed "
                                    "by CUDA events"},
        "depthwise": depthwise}
    del decoders, groups

    # single stream: the config-4 GOP (120 frames: I + 15 P packets), batch 1
    gop = encode_sequences(ufb, syn, mi, mv, [0], 1, dev, W, H, 120, seed_base=3)[0]
    gs = torch.cuda.Stream(dev)
    di, dv = ufb.Codec(mi, 1), ufb.Codec(mv, 1)
    for c in (di, dv):
        c.set_skip_threshold(SKIP)
        c.set_stream(gs)
    _, i_pay, _, p_pays, resets, states = gop

    def gop_decode(events=None):
        di.decompress(i_pay, W, H, QP_I, frames=False)
        dv.set_reference_from(di)
        for k, pay in enumerate(p_pays):
            if events is not None:
                events[k][0].record(gs)
            dv.decompress(pay, W, H, QP_P, resets[k], frames=False)
            if events is not None:
                events[k][1].record(gs)

    for _ in range(2):
        gop_decode()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in p_pays]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(gs)
    gop_decode(ev)
    e1.record(gs)
    torch.cuda.synchronize()
    for k, want in states.items():
        if dv.state_hash(k) != want:
            raise RuntimeError(f"config-4 GOP: decoder {k} state differs from the encoder's")
    gop_ms = e0.elapsed_time(e1)
    p_ms = [a.elapsed_time(b) for a, b in ev]
    out["config4_gop"] = {"value": 120 / (gop_ms * 1e-3), "unit": "frames/s", "ms": gop_ms,
                          "workload": "one 120-frame 626x352 stream (seed 3): I + 15 P packets, batch 1, host rANS "
                                      "included"}
    out["config3_p_packet"] = {"ms_mean": statistics.mean(p_ms), "ms_min": min(p_ms),
                               "workload": "decode of one 8-frame reset P packet of one 626x352 stream (the GOP's)"}
    try:
        with open(os.path.join(ROOT, "tests", "golden", "config3.json")) as f:
            g = json.load(f)
        p = [pk.get("decode_seconds") for pk in g["packets"] if pk["type"] == "P" and pk.get("reset")]
        i = g["packets"][0].get("decode_seconds")
        if p and p[0] and i:
            out["reference_cpu"] = {
                "p_packet_decode_s": p[0], "i_packet_decode_s": i, "cores": g["threads"],
                "frames_per_s": FRAMES / (i + 4 * p[0]),
                "source": "the reference's IntegerModel::decompress (oracle/_ref) on the same 626x352 config-3 "
                          "packets, timed on the build host by tests/golden/make_model_golden.py"}
    except (OSError, KeyError, ValueError):
        pass
    return out


def ref_decode_sample(threads):
    """Reference IntegerModel::decompress (oracle/_ref) on a 128x128 sample;
    returns (seconds per P packet, seconds per I packet)."""
    import oracle
    import __graft_entry__ as entry
    syn = entry.load_synthetic()
    ref = oracle.ref_oracle()
    ora = oracle.c_oracle()
    ref.set_threads(threads)
    img_t, vid_t = syn.prepared("image", 1), syn.prepared("htl", 2)
    video = syn.synthetic_video(SAMPLE, SAMPLE, 9, 100)
    ri = ref.model("image", img_t)
    ri.set_skip_threshold(SKIP)
    i_pay, rec = ri.compress(ora.from_bytes(syn.frames_to_chunk(video[:1])), QP_I)
    rv = ref.model("htl", vid_t)
    rv.set_skip_threshold(SKIP)
    rv.add_ref_feature_from_frame(rec[0])
    p_pay, _ = rv.compress(ora.from_bytes(syn.frames_to_chunk(video[1:9])), QP_P, True)
    di = ref.model("image", img_t)
    di.set_skip_threshold(SKIP)
    t0 = time.perf_counter()
    frames = di.decompress(i_pay, SAMPLE, SAMPLE, QP_I)
    t_i = time.perf_counter() - t0
    dv = ref.model("htl", vid_t)
    dv.set_skip_threshold(SKIP)
    dv.add_ref_feature_from_frame(frames[0])
    t0 = time.perf_counter()
    dv.decompress(p_pay, SAMPLE, SAMPLE, QP_P, True)
    t_p = time.perf_counter() - t0
    return t_p, t_i


def ref_fps_1080(t_p, t_i):
    """Extrapolate the 128x128 sample to a 1920x1088 32-frame sequence by pixel count."""
    seq_seconds = (t_i + 4 * t_p) * (W1080 * H1080) / (SAMPLE * SAMPLE)
    return FRAMES / seq_seconds


def ref_decode_note(t_p, t_i):
    return (f"reference IntegerModel::decompress at {SAMPLE}x{SAMPLE}: P packet {t_p:.2f} s, I packet {t_i:.2f} s, "
            f"extrapolated by pixel count to 1920x1088 sequences of 1 I + 4 P packets")


# ----------------------------------------------------------------- conv ----

def conv_inputs(seed=0):
    rng = np.random.default_rng(seed)
    x = rng.integers(-4096, 4097, (CONV_BATCH, 64, 88, 160)).astype(np.int16)
    w = rng.integers(-256, 257, (64, 64, 3, 3)).astype(np.int16)
    b = rng.integers(-(1 << 16), (1 << 16) + 1, (64,)).astype(np.int32)
    return x, w, b


def bench_conv_ours(args, rank, world, local):
    import torch
    import __graft_entry__ as entry
    ufb = entry.load_package()
    L = ufb.library()
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
    xd, wdv, bd = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
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

    peak = i8_peak_tops(L, stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the sampler runs through warm-up and timed steps (a step is shorter than one query)
    with Clocks(local) as clk:
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
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = reduce_over_ranks(ms, world, dev, "max")
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
    e2e_ms = reduce_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev, "max")
    import oracle
    if not np.array_equal(oh_[:1].numpy(), oracle.c_oracle().conv2d(x[:1], w, b, 1, 1)):
        raise RuntimeError("bench output differs from the CPU oracle")
    macs = n * co * h * wd * ci * 9
    achieved = 8 * macs / (ms * 1e-3) / 1e12
    return {
        "metric": "INT16 3x3 conv int16-MAC/s (BASELINE config 1 shape, 64 copies per step)",
        "value": world * macs / (ms_max * 1e-3), "unit": "MAC/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int16 (int8 planes, s32 accumulators, int64 recombination)",
        "data": "synthetic (seeded)",
        "config": {"workload": "config-1 conv 64x[1x64x88x160] 3x3 64->64 int32 bias, pad 1", "batch": CONV_BATCH,
                   "l2": "inputs larger than L2", "parallelism": f"replicas x{world}"},
        "gpu_launches": args.steps, "clocks": clk.summary(),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS(int8)",
                     "frac": achieved / peak, "traffic": load_traffic("conv_config1_b64"),
                     "traffic_source": "ncu capture in profiles/, not this run",
                     "peak_source": "measured live: dense tcgen05 kind::i8 probe (ufb_probe_i8_peak)"},
        "e2e": {"value": world * macs / (e2e_ms * 1e-3), "unit": "MAC/s", "h2d_bytes_per_step": int(x.nbytes),
                "d2h_bytes_per_step": int(n * co * h * wd * 2)},
    }


def ref_conv(threads):
    import oracle
    ref = oracle.ref_oracle()
    ref.set_threads(threads)
    x, w, b = conv_inputs(0)
    sample = 8
    t0 = time.perf_counter()
    ref.conv2d(x[:sample], w, b, 1, 1)
    dt = time.perf_counter() - t0
    return sample * 64 * 88 * 160 * 64 * 9 / dt, f"{sample} of {CONV_BATCH} config-1 convs ({dt:.2f} s)"


# ----------------------------------------------------------------- warp ----

WARP_SHAPE = (1, 64, 176, 320)


def warp_inputs(seed=1):
    rng = np.random.default_rng(seed)
    n, c, h, w = WARP_SHAPE
    f = rng.integers(-4096, 4097, WARP_SHAPE).astype(np.int16)
    flow = np.round(512 * (rng.normal(0, 4.0, (n, 2, h, w)) + np.array([3.25, -1.5])[None, :, None, None]))
    return f, np.clip(flow, -32768, 32767).astype(np.int16)


def warp_bytes():
    n, c, h, w = WARP_SHAPE
    return 2 * (2 * n * c * h * w) + 2 * n * 2 * h * w


def hbm_peak():
    """Measured copy bandwidth (MEASURED_PEAKS.json) or the pool's fallback figure."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback (6.65 TB/s)"


def bench_warp_ours(args, rank, world, local):
    import torch
    import __graft_entry__ as entry
    ufb = entry.load_package()
    L = ufb.library()
    L.ufb_warp.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    f, flow = warp_inputs(1 + rank)
    n, c, h, w = WARP_SHAPE
    fd, fld = torch.from_numpy(f).to(dev), torch.from_numpy(flow).to(dev)
    out = torch.empty_like(fd)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def launch(o=out, x=fd, fl=fld):
        rc = L.ufb_warp(x.data_ptr(), fl.data_ptr(), n, c, h, w, o.data_ptr(), sp)
        if rc:
            raise RuntimeError(L.ufb_last_error().decode())

    steps = max(args.steps, 20)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with Clocks(local) as clk:
        for _ in range(max(args.warmup, 3)):
            launch()
        t_end = time.time() + 0.5
        while time.time() < t_end:
            flush.fill_(1)
            launch()
            torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        for a, b in ev:
            flush.fill_(1)  # L2 holds nothing of the inputs when the call starts
            a.record(stream)
            launch()
            b.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    ms_max = reduce_over_ranks(ms, world, dev, "max")
    import oracle
    ora = oracle.c_oracle()
    want = ora.warp(f, flow)
    if not np.array_equal(out.cpu().numpy(), want):
        raise RuntimeError("warp output differs from the fixed-point oracle")
    # end to end through the public entry point: host (pinned) inputs in, host output back
    fh, flh = torch.from_numpy(f).pin_memory(), torch.from_numpy(flow).pin_memory()
    oh = torch.empty_like(fh).pin_memory()

    def e2e_step():
        fd.copy_(fh, non_blocking=True)
        fld.copy_(flh, non_blocking=True)
        launch()
        oh.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(steps):
        e2e_step()
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = reduce_over_ranks(e2.elapsed_time(e3) / steps, world, dev, "max")
    if not np.array_equal(oh.numpy(), want):
        raise RuntimeError("warp e2e output differs from the fixed-point oracle")
    peak, peak_src = hbm_peak()
    achieved = warp_bytes() / (ms * 1e-3) / 1e9
    return {
        "metric": "INT16 backward bilinear warp calls/s (BASELINE config 2, 1x64x176x320)",
        "value": world / (ms_max * 1e-3), "unit": "warps/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int16 (Q9 flow, 32-bit exact rna bilinear)", "data": "synthetic (seeded)",
        "config": {"workload": "config 2: features 1x64x176x320 U[-4096,4096], Q9 flow N(0,4^2)+(3.25,-1.5) px, "
                               "border clamp, seed 1", "l2": "flushed (256 MB write) before every timed call",
                   "parallelism": f"replicas x{world}"},
        "gpu_launches": steps, "clocks": clk.summary(),
        "roofline": {"bound": "hbm", "kernel": "warp_tile_kernel", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "traffic": load_traffic("warp_config2_per_launch"),
                     "traffic_source": "ncu capture (profiles/warp_tile_config2.md), not this run",
                     "algorithmic_bytes": warp_bytes(), "peak_source": peak_src,
                     "timing": "CUDA events around each launch on its stream, averaged"},
        "e2e": {"value": world / (e2e_ms * 1e-3), "unit": "warps/s", "h2d_bytes_per_step": int(f.nbytes + flow.nbytes),
                "d2h_bytes_per_step": int(f.nbytes)},
    }


def cpu_warp():
    """The fixed-point restatement (oracle/uf_oracle.c, one thread) on whole config-2 calls."""
    import oracle
    ora = oracle.c_oracle()
    f, flow = warp_inputs(1)
    calls, t0 = 0, time.perf_counter()
    while calls < 3 or time.perf_counter() - t0 < 2.0:
        ora.warp(f, flow)
        calls += 1
    dt = time.perf_counter() - t0
    return calls / dt, f"{calls} config-2 calls of the C restatement ufo_warp in {dt:.2f} s"


# ----------------------------------------------------------------- main ----

def main():
    args = parse()
    rank, world, local = dist_env()
    threads = os.cpu_count() or 1
    if args.impl == "reference":
        if rank != 0:
            return
        kind, cores = "reference", threads
        if args.workload == "conv":
            runs = [ref_conv(threads) for _ in range(max(args.steps, 1))]
            value, unit, note = statistics.median(r[0] for r in runs), "MAC/s", runs[-1][1]
            metric = "INT16 3x3 conv int16-MAC/s (BASELINE config 1 shape, 64 copies per step)"
            cfg = "config-1 conv 64x[1x64x88x160] 3x3 64->64 int32 bias, pad 1"
        elif args.workload == "warp":
            # the reference has no integer warp: its CPU path is this repository's restatement
            runs = [cpu_warp() for _ in range(max(args.steps, 1))]
            value, unit, note = statistics.median(r[0] for r in runs), "warps/s", runs[-1][1]
            metric = "INT16 backward bilinear warp calls/s (BASELINE config 2, 1x64x176x320)"
            cfg = "config 2: features 1x64x176x320, Q9 flow N(0,4^2)+(3.25,-1.5) px, border clamp, seed 1"
            kind, cores = "port", 1
        else:
            samples = [ref_decode_sample(threads) for _ in range(max(args.steps, 1))]
            t_p = statistics.median(s[0] for s in samples)
            t_i = statistics.median(s[1] for s in samples)
            value, unit, note = ref_fps_1080(t_p, t_i), "frames/s", ref_decode_note(t_p, t_i)
            metric = "INT16 HT-L decoded frames/s (1920x1088, BASELINE config 5)"
            cfg = "config 5: 64 seqs x 32 frames 1920x1088, I + 4 P packets each, qp_i 0 qp_p 20, reset 8, skip 0.2"
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "int16",
            "data": "synthetic (seeded)", "config": {"workload": cfg},
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind, "sample": note},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        # start barrier and timing reductions only: host scalars over gloo
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    if args.workload == "warp":
        res = bench_warp_ours(args, rank, world, local)
        if rank == 0 and world == 1:
            v, note = cpu_warp()
            res["cpu_baseline"] = {"value": v, "unit": "warps/s", "cores": 1, "kind": "port", "sample": note}
    elif args.workload == "conv":
        res = bench_conv_ours(args, rank, world, local)
        if rank == 0 and world == 1:
            v, note = ref_conv(1)
            res["cpu_baseline"] = {"value": v, "unit": "MAC/s", "cores": 1, "kind": "reference", "sample": note}
    else:
        res = bench_decode_ours(args, rank, world, local)
        if rank == 0 and world == 1:
            t_p, t_i = ref_decode_sample(threads)
            res["cpu_baseline"] = {"value": ref_fps_1080(t_p, t_i), "unit": "frames/s", "cores": threads,
                                   "kind": "reference", "sample": ref_decode_note(t_p, t_i)}
    if rank == 0:
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
