"""GPU: whole UF16 streams.  The engine's stream encoder must write the same
archive bytes as the reference's IntegerCodec::encode loop over its own CPU
models, and its stream decoder must reproduce the reference's decoded frames
and decoded-YUV SHA-256 (src/integer_codec.cpp:215-493).  64x64 frames keep
the CPU reference to seconds per packet."""
import hashlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

W, H = 64, 64
SKIP = 0.2


@pytest.fixture(scope="module")
def setup(ufb, syn, dev):
    import oracle.stream as st
    img_t, vid_t = syn.prepared("image", 1), syn.prepared("htl", 2)
    ids = (bytes.fromhex(ufb.prepared_identity(img_t, "image", "src-image")),
           bytes.fromhex(ufb.prepared_identity(vid_t, "htl", "src-htl")))
    assert ids[0].hex() == st.prepared_identity(img_t, "image", "src-image")
    return {"img_t": img_t, "vid_t": vid_t, "ids": ids,
            "image": ufb.Model("image", img_t), "htl": ufb.Model("htl", vid_t)}


def _engine(ufb, setup, batch=1, video=True):
    ic = ufb.Codec(setup["image"], batch)
    vc = ufb.Codec(setup["htl"], batch) if video else None
    for c in (ic, vc):
        if c is not None:
            c.set_skip_threshold(SKIP)
    return ufb.StreamCodec(ic, vc, *setup["ids"]), (ic, vc)


def _reference(ref, ora, setup):
    import oracle.stream as st
    return st.RefStreamCodec(ref, ora, setup["img_t"], setup["vid_t"], *setup["ids"], skip_threshold=SKIP)


@pytest.mark.parametrize("frames,reset_interval,intra_period", [
    (10, 16, -1),  # I + P + padded P; (9 + 8) % 16 == 1 resets the second P
    (17, 8, 8),    # I + P + I + P: intra_period 8 puts an I packet at frame 9; (1 + 8) % 8 == 1 resets the first P
])
def test_stream_bytes_and_digest_match_reference(ufb, ref, ora, syn, setup, frames, reset_interval, intra_period):
    video = syn.synthetic_video(W, H, frames, 11)
    want, want_packets = _reference(ref, ora, setup).encode(video, W, H, 0, 20, reset_interval, intra_period)
    sc, keep = _engine(ufb, setup)
    got, packets = sc.encode(video[None], W, H, 0, 20, reset_interval, intra_period)
    assert packets == want_packets
    assert got[0] == want, "archive bytes differ"
    info = ufb.scan_bitstream(got[0], "htl", frames)
    assert info["packets"] == packets and info["image_identity"] == setup["ids"][0]
    # decode: the reference's digest and frames, and the engine's
    digest, yuv, ref_packets = _reference(ref, ora, setup).decode(want, frames, packets)
    seen = []
    dec, keep2 = _engine(ufb, setup)
    res = dec.decode([want], frames, packets, W, H, sink=lambda b, f, y: seen.append((b, f, y)))
    assert res["frames"] == frames and res["packets"] == ref_packets
    assert res["sha256"][0] == digest
    assert [f for _, f, _ in seen] == list(range(frames))
    for (_, f, y), r in zip(seen, yuv):
        assert y == r.tobytes(), f"frame {f}"
    assert hashlib.sha256(b"".join(y for _, _, y in seen)).hexdigest() == digest


def test_batched_streams_match_single_streams(ufb, syn, setup):
    videos = np.stack([syn.synthetic_video(W, H, 9, s) for s in (21, 22)])
    both, _ = _engine(ufb, setup, batch=2)
    streams, packets = both.encode(videos, W, H, 0, 20, 0, -1)
    for b in range(2):
        one, _ = _engine(ufb, setup)
        single, _ = one.encode(videos[b:b + 1], W, H, 0, 20, 0, -1)
        assert single[0] == streams[b]
    dec, _ = _engine(ufb, setup, batch=2)
    res = dec.decode(streams, 9, packets)
    for b in range(2):
        one, _ = _engine(ufb, setup)
        assert one.decode([streams[b]], 9, packets)["sha256"][0] == res["sha256"][b]
    # streams of one batch must share their packet structure
    other, _ = _engine(ufb, setup)
    odd, _ = other.encode(videos[1:2], W, H, 0, 22, 0, -1)
    with pytest.raises(ufb.UfbError) as e:
        dec.decode([streams[0], odd[0]], 9, packets)
    assert "differ in packet structure" in str(e.value)


def test_image_only_stream(ufb, ref, ora, syn, setup):
    import oracle.stream as st
    video = syn.synthetic_video(W, H, 3, 31)
    r = st.RefStreamCodec(ref, ora, setup["img_t"], None, setup["ids"][0], skip_threshold=SKIP)
    want, packets = r.encode(video, W, H, 12, 20, 0, 1)
    assert packets == 3
    sc, _ = _engine(ufb, setup, video=False)
    got, _ = sc.encode(video[None], W, H, 12, 20, 0, 1)
    assert got[0] == want
    assert sc.decode(got, 3, 3)["sha256"][0] == r.decode(want, 3, 3)[0]
    with pytest.raises(ufb.UfbError) as e:
        sc.encode(video[None], W, H, 12, 20, 0, -1)
    assert "video model is required" in str(e.value)


def test_stream_decode_errors(ufb, syn, setup):
    video = syn.synthetic_video(W, H, 9, 41)
    sc, _ = _engine(ufb, setup)
    streams, packets = sc.encode(video[None], W, H, 0, 20, 0, -1)
    data = streams[0]
    dec, _ = _engine(ufb, setup)
    cases = [
        (lambda: dec.decode([data], 10, packets), "Incomplete UF integer bitstream"),
        (lambda: dec.decode([data], 9, packets + 1), "Incomplete UF integer bitstream"),
        (lambda: dec.decode([data], 1, packets), "Unexpected UF packet or unknown SPS"),
        (lambda: dec.decode([data[:-7]], 9, packets), "Truncated UF bitstream payload"),
        (lambda: dec.decode([data], 9, packets, W + 2, H), "Bitstream dimensions differ from archive metadata"),
    ]
    wrong = bytearray(data)
    wrong[9] ^= 1  # image identity
    cases.append((lambda: dec.decode([bytes(wrong)], 9, packets), "identity mismatch"))
    for call, message in cases:
        with pytest.raises(ufb.UfbError) as e:
            call()
        assert message in str(e.value)
    # the codec still decodes a valid stream after the errors
    assert dec.decode([data], 9, packets)["frames"] == 9


def test_invalid_encode_settings(ufb, syn, setup):
    sc, _ = _engine(ufb, setup)
    video = syn.synthetic_video(W, H, 2, 3)[None]
    for args in ((W, H, 64, 20, 0, -1), (W, H, 0, -1, 0, -1), (W, H, 0, 20, 0, 12)):
        with pytest.raises(ufb.UfbError) as e:
            sc.encode(video, *args)
        assert "Invalid UF encode settings" in str(e.value)


def test_interrupt_stops_coding(ufb, syn, setup):
    video = syn.synthetic_video(W, H, 9, 51)
    sc, _ = _engine(ufb, setup)
    streams, packets = sc.encode(video[None], W, H, 0, 20, 0, -1)
    dec, _ = _engine(ufb, setup)
    ufb.set_interrupt(True)
    try:
        for call in (lambda: dec.decode(streams, 9, packets), lambda: sc.encode(video[None], W, H, 0, 20, 0, -1)):
            with pytest.raises(ufb.UfbError) as e:
                call()
            assert e.value.code == -6 and str(e.value) == "UF operation interrupted"
    finally:
        ufb.set_interrupt(False)
    assert dec.decode(streams, 9, packets)["frames"] == 9


def test_state_hashes_match_reference(ufb, ref, ora, syn, setup):
    """check-int16 state records: SHA-256 of each DPB tensor's NCHW int16 bytes."""
    import oracle.stream as st
    video = syn.synthetic_video(W, H, 9, 61)
    r = st.RefStreamCodec(ref, ora, setup["img_t"], setup["vid_t"], *setup["ids"], skip_threshold=SKIP)
    data, packets = r.encode(video, W, H, 0, 20, 0, -1)
    # the reference models' states after decoding the archive's packets in
    # order, as IntegerCodec::decode_stream_impl does (src/integer_codec.cpp:445-461)
    image, vid = ref.model("image", setup["img_t"]), ref.model("htl", setup["vid_t"])
    for m in (image, vid):
        m.set_skip_threshold(SKIP)
    for u in ref.bs_parse(data)[1]:
        if u["type"] == 1:
            frames = image.decompress(u["payload"], W, H, u["qp"])
            vid.clear_dpb()
            vid.add_ref_feature_from_frame(frames[0])
        elif u["type"] == 2:
            vid.decompress(u["payload"], W, H, u["qp"], u["reset"])
    sc, (ic, vc) = _engine(ufb, setup)
    sc.decode([data], 9, packets)
    for k in ("reference", "memory", "context"):
        mine, want = vc.state_hash(k), vid.state(k)
        assert (mine is None) == (want is None), k
        if want is not None:
            assert mine == hashlib.sha256(np.ascontiguousarray(want, "<i2").tobytes()).hexdigest(), k
            assert mine == hashlib.sha256(vc.state(k).astype("<i2").tobytes()).hexdigest(), k


def test_cli_encode_decode_verify(ufb, syn, setup, tmp_path, capsys):
    """The command line (encode / decode / verify) over a raw YUV420 file."""
    import importlib.util
    import json
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("ufb200_cli", os.path.join(root, "dcvc-uf-int16-cpp_b200", "cli.py"))
    cli = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cli)
    img, vid = str(tmp_path / "image.npz"), str(tmp_path / "video.npz")
    cli.save_model_npz(img, setup["img_t"], "image", "src-image")
    cli.save_model_npz(vid, setup["vid_t"], "htl", "src-htl")
    video = syn.synthetic_video(W, H, 10, 81)
    yuv = tmp_path / "in.yuv"
    with open(yuv, "wb") as f:
        for fr in video:
            f.write(fr[0].tobytes() + fr[1, ::2, ::2].tobytes() + fr[2, ::2, ::2].tobytes())
    bits, out = str(tmp_path / "video.bin"), str(tmp_path / "out.yuv")

    def run(*argv):
        rc = cli.main(list(argv))
        return rc, json.loads(capsys.readouterr().out.strip().splitlines()[-1])

    rc, ev = run("encode", "--image", img, "--video", vid, "--input", str(yuv), "--width", str(W), "--height",
                 str(H), "--output", bits)
    assert rc == 0 and ev["frames"] == 10 and ev["packets"] == 3
    info = ufb.scan_bitstream(open(bits, "rb").read(), "htl", 10)
    assert info["image_identity"] == setup["ids"][0] and info["video_identity"] == setup["ids"][1]
    common = ("--image", img, "--video", vid, "--input", bits, "--frames", "10", "--packets", "3")
    rc, ev = run("decode", *common, "--output", out)
    assert rc == 0 and ev["decoded_frames"] == 10
    assert ev["decoded_yuv_sha256"] == hashlib.sha256(open(out, "rb").read()).hexdigest()
    assert os.path.getsize(out) == 10 * W * H * 3 // 2
    rc, ev2 = run("verify", *common, "--expect-sha256", ev["decoded_yuv_sha256"])
    assert rc == 0 and ev2["event"] == "verification_completed"
    rc, ev3 = run("verify", *common, "--expect-sha256", "0" * 64)
    assert rc == 1 and ev3["message"] == "Decoded UF pixels differ from archive validation"
