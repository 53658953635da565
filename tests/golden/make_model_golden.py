"""Generate the model-level golden digests at the benchmark sizes from the
reference's own CPU INT16 path.

Every value here comes from the UNMODIFIED reference sources compiled into
oracle/_ref/libufref.so (`make -C oracle ref REF_ROOT=<reference checkout>`):
``uf::IntegerModel`` (src/integer_model.cpp:295-359: compress, decompress,
reconstruct and the DPB states), ``uf::IntegerCodec`` (src/integer_codec.cpp:
215-292 encode loop, 405-493 decode loop with its decoded-YUV SHA-256) and
``IntegerCodec::raw_frame`` (src/integer_codec.cpp:294-323).  The models are
the seeded random-init prepared tables of ``synthetic.make_prepared`` (image
seed 1, HT-L seed 2) and the inputs come from ``synthetic.synthetic_video``;
SHA-256 digests of the inputs are stored too, so a test can tell an input
mismatch from an engine mismatch, and so are the reference's CPU seconds per
encode and decode (the thread count is recorded).

Cases (the reference's FFmpeg testsrc2 clip is not
available, the seeded synthetic scene stands in for it):

* ``config3`` -- 626x352, video seed 2: I packet (qp 0), then P packet 1
  (qp 20, reset: the reset_interval 8 case) and P packet 2 (qp 20, no reset)
  encoded by ``IntegerModel::compress`` with reconstruction, then all three
  decoded from their payloads by a fresh model pair through
  ``IntegerModel::decompress``.  Digests of payloads, int16 frames, YUV420
  frames (``raw_frame``) and the reference / memory / context states.
* ``config4`` -- the 120-frame GOP at 626x352, video seed 3, qp_i 0, qp_p 20,
  reset_interval 8, intra_period -1, skip 0.2: the archive written by
  ``IntegerCodec::encode`` and the decoded-YUV SHA-256 (plus per-frame
  digests) returned by ``IntegerCodec::decode_stream`` on it.
* ``config5`` -- one 1920x1088 stream (video seed 100): I packet and the first
  (reset) P packet encoded with reconstruction.  A reference decode of a 1080p
  packet takes over half an hour on CPU; its decoder reproduces these
  reconstructions by construction (the same ``reconstruct`` on the same
  ``y_hat``), which config3 checks at 626x352.

CPU cost on 8 threads: about 20 min (config3), 2 h (config4), 1 h (config5).

Run: python tests/golden/make_model_golden.py [--threads N] [config3 config4 config5]
Writes tests/golden/<case>.json; existing files are kept unless --force.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import __graft_entry__ as entry  # noqa: E402
import oracle  # noqa: E402
import oracle.stream as ost  # noqa: E402

SKIP = 0.2
IMAGE_SEED, VIDEO_SEED = 1, 2
IMAGE_SOURCE, VIDEO_SOURCE = "src-image", "src-htl"


def sha(a) -> str:
    if isinstance(a, (bytes, bytearray)):
        return hashlib.sha256(a).hexdigest()
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()).hexdigest()


def models(syn):
    return syn.prepared("image", IMAGE_SEED), syn.prepared("htl", VIDEO_SEED)


def states(model):
    out = {}
    for which in ("reference", "memory", "context"):
        s = model.state(which)
        out[which] = None if s is None else {"shape": [int(v) for v in s.shape], "sha256": sha(s)}
    return out


def frames_record(ref, frames, width, height):
    return {"int16": [sha(f) for f in frames],
            "yuv420": [sha(ref.raw_frame(f, height, width)) for f in frames]}


def packet_case(ref, ora, syn, width, height, seed, p_resets, decode, log):
    """I packet then P packets (one per entry of p_resets) at qp 0 / 20."""
    img_t, vid_t = models(syn)
    video = syn.synthetic_video(width, height, 1 + 8 * len(p_resets), seed)
    rec = {"width": width, "height": height, "video_seed": seed, "frames": int(video.shape[0]),
           "input_sha256": sha(video), "qp_i": 0, "qp_p": 20, "skip_threshold": SKIP, "packets": []}
    image, hv = ref.model("image", img_t), ref.model("htl", vid_t)
    for m in (image, hv):
        m.set_skip_threshold(SKIP)
    t = time.time()
    first, frames = image.compress(ora.from_bytes(video[0:1].reshape(1, 3, height, width)), 0)
    dt = time.time() - t
    log(f"  I encode {dt:.0f} s")
    rec["packets"].append({"type": "I", "payload_sha256": sha(first), "payload_bytes": len(first),
                           "frames": frames_record(ref, frames, width, height), "encode_seconds": round(dt, 2)})
    hv.add_ref_feature_from_frame(frames[0])
    payloads = []
    for k, reset in enumerate(p_resets):
        chunk = video[1 + 8 * k: 9 + 8 * k].reshape(1, 24, height, width)
        t = time.time()
        payload, frames = hv.compress(ora.from_bytes(chunk), 20, reset)
        dt = time.time() - t
        log(f"  P{k + 1} encode {dt:.0f} s")
        payloads.append(payload)
        rec["packets"].append({"type": "P", "reset": bool(reset), "payload_sha256": sha(payload),
                               "payload_bytes": len(payload), "frames": frames_record(ref, frames, width, height),
                               "states": states(hv), "encode_seconds": round(dt, 2)})
    if decode:
        image_d, hv_d = ref.model("image", img_t), ref.model("htl", vid_t)
        for m in (image_d, hv_d):
            m.set_skip_threshold(SKIP)
        t = time.time()
        frames = image_d.decompress(first, width, height, 0)
        dt = time.time() - t
        log(f"  I decode {dt:.0f} s")
        rec["packets"][0]["decoded"] = frames_record(ref, frames, width, height)
        rec["packets"][0]["decode_seconds"] = round(dt, 2)
        hv_d.add_ref_feature_from_frame(frames[0])
        for k, reset in enumerate(p_resets):
            pk = rec["packets"][1 + k]
            t = time.time()
            frames = hv_d.decompress(payloads[k], width, height, 20, reset)
            dt = time.time() - t
            log(f"  P{k + 1} decode {dt:.0f} s")
            pk["decoded"] = frames_record(ref, frames, width, height)
            pk["decode_seconds"] = round(dt, 2)
            pk["decoded_states"] = states(hv_d)
    return rec


def gop_case(ref, syn, width, height, frames, seed, threads, log):
    img_t, vid_t = models(syn)
    ii = ost.prepared_identity(img_t, "image", IMAGE_SOURCE)
    vi = ost.prepared_identity(vid_t, "htl", VIDEO_SOURCE)
    video = syn.synthetic_video(width, height, frames, seed)
    rec = {"width": width, "height": height, "video_seed": seed, "frames": frames, "input_sha256": sha(video),
           "qp_i": 0, "qp_p": 20, "reset_interval": 8, "intra_period": -1, "skip_threshold": SKIP,
           "image_identity": ii, "video_identity": vi}
    enc = ref.codec(img_t, ii, vid_t, vi, "htl", SKIP, threads=threads)
    t = time.time()
    data, nframes, packets = enc.encode(video, width, height, 0, 20, 8, -1)
    dt = time.time() - t
    log(f"  encode {dt:.0f} s, {packets} packets, {len(data)} bytes")
    rec.update({"archive_sha256": sha(data), "archive_bytes": len(data), "packets": packets,
                "encode_seconds": round(dt, 1)})
    dec = ref.codec(img_t, ii, vid_t, vi, "htl", SKIP, threads=threads)
    t = time.time()
    digest, yuv, dpk = dec.decode(data, frames, packets, width, height)
    dt = time.time() - t
    log(f"  decode {dt:.0f} s")
    rec["decode_seconds"] = round(dt, 1)
    assert dpk == packets
    rec.update({"decoded_yuv_sha256": digest, "frame_yuv_sha256": [sha(y) for y in yuv]})
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*", default=["config3", "config4", "config5"])
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    syn = entry.load_synthetic()
    ref, ora = oracle.ref_oracle(), oracle.c_oracle()

    def log(msg):
        print(msg, flush=True)

    for case in args.cases:
        path = os.path.join(HERE, f"{case}.json")
        if os.path.exists(path) and not args.force:
            log(f"{case}: {path} exists, kept")
            continue
        ref.set_threads(args.threads)
        log(f"{case}: {args.threads} threads")
        t0 = time.time()
        if case == "config3":
            rec = packet_case(ref, ora, syn, 626, 352, 2, [True, False], True, log)
        elif case == "config4":
            rec = gop_case(ref, syn, 626, 352, 120, 3, args.threads, log)
        elif case == "config5":
            rec = packet_case(ref, ora, syn, 1920, 1088, 100, [True], False, log)
        else:
            raise SystemExit(f"unknown case {case}")
        rec.update({"case": case, "image_seed": IMAGE_SEED, "htl_seed": VIDEO_SEED,
                    "generator": "tests/golden/make_model_golden.py",
                    "reference_cpu_seconds": round(time.time() - t0, 1), "threads": args.threads})
        with open(path + ".tmp", "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)
            f.write("\n")
        os.replace(path + ".tmp", path)
        log(f"{case}: wrote {path} ({time.time() - t0:.0f} s)")


if __name__ == "__main__":
    main()
