"""Command line for whole UF16 streams on the B200 engine: the encode, decode and
verify commands of the reference's CLI (src/main.cpp:663-744 over
uf::IntegerCodec, src/integer_codec.cpp:215-493) for raw YUV420 files.

    python dcvc-uf-int16-cpp_b200/cli.py encode --image img.npz --video vid.npz \\
        --input in.yuv --width 1920 --height 1088 --output video.bin
    python dcvc-uf-int16-cpp_b200/cli.py decode --image img.npz --video vid.npz \\
        --input video.bin --frames 32 --packets 5 --output out.yuv
    python dcvc-uf-int16-cpp_b200/cli.py verify --image img.npz --video vid.npz \\
        --input video.bin --frames 32 --packets 5 --expect-sha256 <hex>

Prepared models are .npz files of the prepared tensors by name (the
uf::PreparedModel table), with the 0-d string entries "__variant__" and
"__source_sha256__"; the stream preamble carries their identities
(uf::prepared_identity).  Raw input frames are YUV420 planar and are widened to
YUV444 by repeating each chroma sample over its 2 x 2 block, as the
reference's RawYuv420Reader does (src/integer_codec.cpp:125-148).  Each command
prints one JSON event line ({"event": "encode_completed", ...}); a digest
mismatch or any codec error exits with status 1 and an {"event": "error"} line.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

VARIANT_KEY = "__variant__"
SOURCE_KEY = "__source_sha256__"


def _package():
    """The engine package (this directory; its name is not an identifier)."""
    name = "ufb200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(HERE, "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def save_model_npz(path: str, tensors: dict, variant: str, source_sha256: str = "") -> None:
    np.savez(path, **tensors, **{VARIANT_KEY: np.array(variant), SOURCE_KEY: np.array(source_sha256)})


def load_model_npz(path: str):
    """-> (variant, source_sha256, {name: array})."""
    with np.load(path, allow_pickle=False) as z:
        if VARIANT_KEY not in z.files:
            raise ValueError(f"{path}: not a prepared model table (no {VARIANT_KEY})")
        variant = str(z[VARIANT_KEY])
        source = str(z[SOURCE_KEY]) if SOURCE_KEY in z.files else ""
        tensors = {k: z[k] for k in z.files if k not in (VARIANT_KEY, SOURCE_KEY)}
    return variant, source, tensors


def yuv420_to_444(planar: np.ndarray, width: int, height: int) -> np.ndarray:
    """One planar YUV420 frame -> uint8 [3, height, width] (chroma repeated 2 x 2)."""
    px = width * height
    y = planar[:px].reshape(height, width)
    u = planar[px: px + px // 4].reshape(height // 2, width // 2)
    v = planar[px + px // 4: px + px // 2].reshape(height // 2, width // 2)
    up = lambda c: np.repeat(np.repeat(c, 2, axis=0), 2, axis=1)  # noqa: E731
    return np.stack([y, up(u), up(v)])


def read_yuv420(path: str, width: int, height: int, max_frames=None) -> np.ndarray:
    """All frames of a raw YUV420 file as uint8 [T, 3, height, width]."""
    if width <= 0 or height <= 0 or width % 2 or height % 2:
        raise ValueError("Invalid UF encode settings")
    frame = width * height * 3 // 2
    data = np.fromfile(path, np.uint8)
    count = data.size // frame
    if data.size % frame:
        raise ValueError("Truncated raw YUV420 frame")
    if max_frames is not None:
        count = min(count, max_frames)
    return np.stack([yuv420_to_444(data[i * frame:(i + 1) * frame], width, height) for i in range(count)])


class Engine:
    """An image codec, a video codec and their stream codec on one GPU."""

    def __init__(self, image_npz: str, video_npz, device: int = 0, skip_threshold: float = 0.2):
        ufb = self.ufb = _package()
        iv, isrc, it = load_model_npz(image_npz)
        if iv != "image":
            raise ValueError(f"{image_npz}: image model expected, got {iv!r}")
        self.image_model = ufb.Model("image", it, device)
        self.image = ufb.Codec(self.image_model, 1)
        self.image.set_skip_threshold(skip_threshold)
        image_id = bytes.fromhex(ufb.prepared_identity(it, iv, isrc))
        self.video_model = self.video = None
        video_id = bytes(32)
        if video_npz:
            vv, vsrc, vt = load_model_npz(video_npz)
            if vv != "htl":
                raise ValueError(f"{video_npz}: HT-L video model expected, got {vv!r}")
            self.video_model = ufb.Model("htl", vt, device)
            self.video = ufb.Codec(self.video_model, 1)
            self.video.set_skip_threshold(skip_threshold)
            video_id = bytes.fromhex(ufb.prepared_identity(vt, vv, vsrc))
        self.stream = ufb.StreamCodec(self.image, self.video, image_id, video_id)


def cmd_encode(a) -> dict:
    eng = Engine(a.image, a.video, a.device, a.skip_threshold)
    frames = read_yuv420(a.input, a.width, a.height, a.max_frames)
    t0 = time.perf_counter()
    streams, packets = eng.stream.encode(frames[None], a.width, a.height, a.qp_i, a.qp_p, a.reset_interval,
                                         a.intra_period)
    seconds = time.perf_counter() - t0
    with open(a.output, "wb") as f:
        f.write(streams[0])
    return {"event": "encode_completed", "output": a.output, "frames": int(frames.shape[0]),
            "packets": int(packets), "bytes": len(streams[0]), "encode_seconds": seconds}


def cmd_decode(a, write: bool) -> dict:
    eng = Engine(a.image, a.video, a.device, a.skip_threshold)
    data = open(a.input, "rb").read()
    out = open(a.output, "wb") if write else None
    try:
        t0 = time.perf_counter()
        sink = (lambda _s, _f, y: out.write(y)) if out else None
        res = eng.stream.decode([data], a.frames, a.packets, a.width or 0, a.height or 0, sink=sink)
        seconds = time.perf_counter() - t0
    finally:
        if out:
            out.close()
    digest = res["sha256"][0]
    if a.expect_sha256 and a.expect_sha256.lower() != digest:
        raise RuntimeError("Decoded UF pixels differ from archive validation")
    return {"event": "decode_completed" if write else "verification_completed", "input": a.input,
            "decoded_frames": res["frames"], "packets": res["packets"], "decode_seconds": seconds,
            "decoded_yuv_sha256": digest}


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="cli.py", description=__doc__.split("\n\n")[0])
    sub = p.add_subparsers(dest="command", required=True)
    for name in ("encode", "decode", "verify"):
        s = sub.add_parser(name)
        s.add_argument("--image", required=True, help="prepared image model (.npz)")
        s.add_argument("--video", help="prepared HT-L video model (.npz); without it, encode needs --intra-period 1")
        s.add_argument("--input", required=True)
        s.add_argument("--device", type=int, default=0)
        s.add_argument("--skip-threshold", type=float, default=0.2)
        s.add_argument("--width", type=int, required=name == "encode")
        s.add_argument("--height", type=int, required=name == "encode")
        if name == "encode":
            s.add_argument("--output", required=True)
            s.add_argument("--qp-i", type=int, default=0)
            s.add_argument("--qp-p", type=int, default=20)
            s.add_argument("--reset-interval", type=int, default=8)
            s.add_argument("--intra-period", type=int, default=-1)
            s.add_argument("--max-frames", type=int)
        else:
            s.add_argument("--frames", type=int, required=True, help="frames in the archive metadata")
            s.add_argument("--packets", type=int, required=True, help="packets in the archive metadata")
            s.add_argument("--expect-sha256", help="the archive's decoded_yuv_sha256")
            if name == "decode":
                s.add_argument("--output", required=True, help="raw YUV420 output")
    return p


def main(argv=None) -> int:
    a = parser().parse_args(argv)
    try:
        if a.command == "encode":
            event = cmd_encode(a)
        else:
            event = cmd_decode(a, a.command == "decode")
    except Exception as e:  # noqa: BLE001 -- reported as the command's result
        print(json.dumps({"event": "error", "command": a.command, "message": str(e)}))
        return 1
    print(json.dumps(event))
    return 0


if __name__ == "__main__":
    sys.exit(main())
