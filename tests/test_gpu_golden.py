"""GPU: the engine against golden digests the reference's own CPU INT16 path
produced at the benchmark sizes (tests/golden/make_model_golden.py, run once on
CPU with oracle/_ref: uf::IntegerModel and uf::IntegerCodec compiled from the
reference's sources).

* config3 (626x352): I packet, a reset P packet and a non-reset P packet --
  payload bytes, reconstructed int16 frames, YUV420 frames (the reference's
  IntegerCodec::raw_frame) and reference / memory / context states after
  encoding, then the same after decoding the payloads with fresh codecs.
* config4 (626x352, 120 frames): the whole UF16 archive the reference's
  IntegerCodec::encode writes (qp_i 0, qp_p 20, reset_interval 8, skip 0.2)
  and the decoded-YUV SHA-256 its decode loop returns.
* config5 (1920x1088): I packet and the first reset P packet of one stream;
  decoding reproduces the reference encoder's reconstructions.

At these sizes every spatial conv spans many tiles and each stream's
spatial-prior positions span many 4096-position chunks (55 at 626x352, 510 at
1080p), so the multi-CTA count / scan / emit path is compared with the
reference's position order.
"""
import hashlib
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a) -> str:
    if isinstance(a, (bytes, bytearray)):
        return hashlib.sha256(a).hexdigest()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def golden(case):
    path = os.path.join(GOLDEN, f"{case}.json")
    if not os.path.exists(path):
        pytest.skip(f"{path} not generated")
    with open(path) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def engines(ufb, syn, dev):
    return ufb.Model("image", syn.prepared("image", 1)), ufb.Model("htl", syn.prepared("htl", 2))


def _codec(ufb, model, skip):
    c = ufb.Codec(model, 1)
    c.set_skip_threshold(skip)
    return c


def _check_frames(frames, yuv, want, what):
    assert [sha(frames[0, f]) for f in range(frames.shape[1])] == want["int16"], f"{what}: int16 frames"
    assert [sha(yuv[0, f]) for f in range(yuv.shape[1])] == want["yuv420"], f"{what}: yuv420 frames"


def _check_states(codec, want, what):
    for k in ("reference", "memory", "context"):
        w = want[k]
        assert codec.state_hash(k) == (None if w is None else w["sha256"]), f"{what}: {k} state"


def _packets_case(ufb, syn, engines, case):
    g = golden(case)
    W, H, skip = g["width"], g["height"], g["skip_threshold"]
    video = syn.synthetic_video(W, H, g["frames"], g["video_seed"])
    assert sha(video) == g["input_sha256"], "synthetic input differs from the one the fixture was made from"
    image, htl = engines
    packets = g["packets"]
    # encode: payload bytes, reconstructions and states
    ie, ve = _codec(ufb, image, skip), _codec(ufb, htl, skip)
    chunk = syn.frames_to_chunk(video[:1])
    payloads, rec = ie.compress(chunk, g["qp_i"], frames=True)
    assert sha(payloads[0]) == packets[0]["payload_sha256"], "I payload"
    assert [sha(rec[0, 0])] == packets[0]["frames"]["int16"], "I reconstruction"
    all_payloads = [payloads[0]]
    ve.set_reference_from(ie)
    for k, pk in enumerate(packets[1:]):
        chunk = syn.frames_to_chunk(video[1 + 8 * k: 9 + 8 * k])
        payloads, rec = ve.compress(chunk, g["qp_p"], pk["reset"], frames=True)
        assert sha(payloads[0]) == pk["payload_sha256"], f"P{k + 1} payload"
        assert [sha(rec[0, f]) for f in range(8)] == pk["frames"]["int16"], f"P{k + 1} reconstruction"
        _check_states(ve, pk["states"], f"P{k + 1} encode")
        all_payloads.append(payloads[0])
    # decode the (reference-identical) payloads with fresh codecs
    idc, vdc = _codec(ufb, image, skip), _codec(ufb, htl, skip)
    frames, yuv = idc.decompress([all_payloads[0]], W, H, g["qp_i"], frames=True, yuv=True)
    _check_frames(frames, yuv, packets[0].get("decoded", packets[0]["frames"]), "I decode")
    vdc.set_reference_from(idc)
    for k, pk in enumerate(packets[1:]):
        frames, yuv = vdc.decompress([all_payloads[1 + k]], W, H, g["qp_p"], pk["reset"], frames=True, yuv=True)
        _check_frames(frames, yuv, pk.get("decoded", pk["frames"]), f"P{k + 1} decode")
        _check_states(vdc, pk.get("decoded_states", pk["states"]), f"P{k + 1} decode")
    assert ufb.device_status(0) == 0


def test_config3_packets_match_reference(ufb, syn, engines):
    _packets_case(ufb, syn, engines, "config3")


def test_config5_fullsize_packets_match_reference(ufb, syn, engines):
    _packets_case(ufb, syn, engines, "config5")


def test_config4_gop_archive_matches_reference(ufb, syn, engines):
    g = golden("config4")
    W, H, skip = g["width"], g["height"], g["skip_threshold"]
    video = syn.synthetic_video(W, H, g["frames"], g["video_seed"])
    assert sha(video) == g["input_sha256"], "synthetic input differs from the one the fixture was made from"
    image, htl = engines
    ids = bytes.fromhex(g["image_identity"]), bytes.fromhex(g["video_identity"])
    enc = ufb.StreamCodec(_codec(ufb, image, skip), _codec(ufb, htl, skip), *ids)
    streams, packets = enc.encode(video[None], W, H, g["qp_i"], g["qp_p"], g["reset_interval"], g["intra_period"])
    assert packets == g["packets"]
    assert len(streams[0]) == g["archive_bytes"] and sha(streams[0]) == g["archive_sha256"], "archive bytes"
    dec = ufb.StreamCodec(_codec(ufb, image, skip), _codec(ufb, htl, skip), *ids)
    seen = []
    res = dec.decode(streams, g["frames"], packets, W, H, sink=lambda b, f, y: seen.append(sha(y)))
    assert res["frames"] == g["frames"] and res["packets"] == packets
    assert seen == g["frame_yuv_sha256"], "decoded YUV frames"
    assert res["sha256"][0] == g["decoded_yuv_sha256"]
