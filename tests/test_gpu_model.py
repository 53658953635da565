"""GPU parity of the model engine against the reference's own CPU path.

The reference's uf::Layers / uf::IntegerModel (oracle/_ref, compiled from its
sources) and the engine run the same seeded prepared models on the same
inputs; every module output, bitstream byte, reconstructed frame and DPB
state must be identical.  Sizes are small so the CPU reference finishes in
seconds (64x64 frames: latent 4x4, features 8x8).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

W, H = 64, 64


@pytest.fixture(scope="module")
def models(ufb, ref, syn, dev):
    img_t, vid_t = syn.prepared("image", 1), syn.prepared("htl", 2)
    return {
        "image": (ufb.Model("image", img_t), ref.model("image", img_t)),
        "htl": (ufb.Model("htl", vid_t), ref.model("htl", vid_t)),
    }


def rnd(rng, shape, lo=-3000, hi=3000):
    return rng.integers(lo, hi, shape).astype(np.int16)


@pytest.mark.parametrize("module,shapes,q", [
    ("feature_adaptor_i", [(1, 192, 8, 8)], None),
    ("feature_adaptor_m", [(1, 512, 8, 8), (1, 512, 8, 8)], None),
    ("feature_extractor", [(1, 512, 8, 10)], None),
    ("hyper_decoder", [(1, 128, 2, 3)], None),
    ("temporal_prior_encoder", [(1, 512, 8, 12)], "q_feature"),
    ("y_prior_fusion", [(1, 256, 4, 6), (1, 512, 4, 6)], None),
    ("y_spatial_prior_reduction", [(1, 768, 4, 5)], None),
    ("y_spatial_prior_adaptor_2", [(1, 512, 4, 4)], None),
    ("y_spatial_prior", [(1, 512, 3, 5)], None),
    ("decoder", [(1, 256, 4, 4), (1, 512, 8, 8)], "q_decoder"),
    ("recon_head.conv.3", [(1, 512, 8, 8)], None),
    ("hyper_encoder", [(1, 256, 8, 8)], None),
])
@pytest.mark.parametrize("ctas", [0, 1])
def test_htl_module_parity(ufb, models, module, shapes, q, ctas):
    """ctas=1 runs every convolution on one persistent CTA, so each one walks
    all its tiles and alternates between the two TMEM accumulator sets."""
    mine, theirs = models["htl"]
    rng = np.random.default_rng(abs(hash(module)) % 1000)
    args = [rnd(rng, s) for s in shapes]
    qp = 20
    want = theirs.run(module, *(args + ([theirs.parameter(q, qp)] if q else [])))
    ufb.set_conv_max_ctas(ctas)
    try:
        got = mine.run(module, *args, q_name=q, qp=qp)
    finally:
        ufb.set_conv_max_ctas(0)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("module,shapes,q", [
    ("hyper_dec", [(1, 128, 2, 2)], None),
    ("y_prior_fusion", [(1, 256, 4, 4)], None),
    ("y_spatial_prior", [(1, 512, 4, 4)], None),
    ("dec", [(1, 256, 4, 4)], "q_scale_dec"),
    ("enc", [(1, 3, 64, 64)], "q_scale_enc"),
])
def test_image_module_parity(models, module, shapes, q):
    mine, theirs = models["image"]
    rng = np.random.default_rng(7)
    args = [rnd(rng, s) for s in shapes]
    qp = 36
    want = theirs.run(module, *(args + ([theirs.parameter(q, qp)] if q else [])))
    got = mine.run(module, *args, q_name=q, qp=qp)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def _frames(syn, count, w=W, h=H, seed=3):
    return syn.synthetic_video(w, h, count, seed)


def _same_states(codec, refm):
    for k in ("reference", "memory", "context"):
        a, b = codec.state(k), refm.state(k)
        assert (a is None) == (b is None), k
        if a is not None:
            assert np.array_equal(a, b), k


@pytest.mark.parametrize("skip", [0.2, 0.0])
def test_image_compress_decompress_parity(ufb, ora, ref, syn, models, skip):
    mine, _ = models["image"]
    img_t = syn.prepared("image", 1)
    video = _frames(syn, 1)
    chunk = syn.frames_to_chunk(video[:1])
    r = ref.model("image", img_t)
    r.set_skip_threshold(skip)
    want_payload, want_frames = r.compress(ora.from_bytes(chunk), 0)
    c = ufb.Codec(mine, 1)
    c.set_skip_threshold(skip)
    payloads, frames = c.compress(chunk, 0, frames=True)
    assert payloads[0] == want_payload
    assert np.array_equal(frames[0, 0], want_frames[0][0])
    got, _ = c.decompress([want_payload], W, H, 0)
    r2 = ref.model("image", img_t)
    r2.set_skip_threshold(skip)
    dec = r2.decompress(want_payload, W, H, 0)
    assert np.array_equal(got[0, 0], dec[0][0])


@pytest.mark.parametrize("reset", [True, False])
@pytest.mark.parametrize("size", [(64, 64), (128, 128)])
def test_video_p_packet_parity(ufb, ora, ref, syn, models, reset, size):
    """At 128x128 a stream's latent holds 256 x 8 x 8 = 16384 positions, four
    4096-position chunks of the spatial-prior kernels, so the per-chunk counts,
    their per-stream scan and the emit offsets are compared with the
    reference's index_select order (src/integer_model.cpp:202-293)."""
    W, H = size
    mine, _ = models["htl"]
    vid_t = syn.prepared("htl", 2)
    video = _frames(syn, 17, w=W, h=H)
    iframe = ora.from_bytes(syn.frames_to_chunk(video[:1]))
    # the I frame reconstruction from the reference image path seeds both DPBs
    ri = ref.model("image", syn.prepared("image", 1))
    ri.set_skip_threshold(0.2)
    _, rec = ri.compress(iframe, 0)
    ref_frame = rec[0]
    enc_ref = ref.model("htl", vid_t)
    enc_ref.set_skip_threshold(0.2)
    enc_ref.add_ref_feature_from_frame(ref_frame)
    enc = ufb.Codec(mine, 1)
    enc.set_skip_threshold(0.2)
    enc.add_ref_frames(ref_frame)
    for packet in range(2):
        chunk = syn.frames_to_chunk(video[1 + 8 * packet: 9 + 8 * packet])
        want_payload, _ = enc_ref.compress(ora.from_bytes(chunk), 20, reset)
        got_payloads, _ = enc.compress(chunk, 20, reset)
        assert got_payloads[0] == want_payload, f"packet {packet}"
        _same_states(enc, enc_ref)
    # decode the reference's stream with a fresh engine codec
    dec_ref = ref.model("htl", vid_t)
    dec_ref.set_skip_threshold(0.2)
    dec_ref.add_ref_feature_from_frame(ref_frame)
    dec = ufb.Codec(mine, 1)
    dec.set_skip_threshold(0.2)
    dec.add_ref_frames(ref_frame)
    chunk = syn.frames_to_chunk(video[1:9])
    enc_ref2 = ref.model("htl", vid_t)
    enc_ref2.set_skip_threshold(0.2)
    enc_ref2.add_ref_feature_from_frame(ref_frame)
    payload, _ = enc_ref2.compress(ora.from_bytes(chunk), 20, reset)
    want = dec_ref.decompress(payload, W, H, 20, reset)
    got, yuv = dec.decompress([payload], W, H, 20, reset, frames=True, yuv=True)
    assert len(want) == 8
    for f in range(8):
        assert np.array_equal(got[0, f], want[f][0]), f"frame {f}"
        assert np.array_equal(yuv[0, f], ref.raw_frame(want[f][0], H, W)), f"yuv {f}"
    _same_states(dec, dec_ref)


def test_batched_streams_match_single(ufb, ora, ref, syn, models):
    """Two independent streams decoded as one batch equal two single decodes
    (frames and YUV420 output)."""
    mine, _ = models["htl"]
    vid_t = syn.prepared("htl", 2)
    payloads, refs = [], []
    for s in range(2):
        video = _frames(syn, 9, seed=40 + s)
        frame0 = ora.from_bytes(syn.frames_to_chunk(video[:1]))
        e = ref.model("htl", vid_t)
        e.set_skip_threshold(0.2)
        e.add_ref_feature_from_frame(frame0)
        p, _ = e.compress(ora.from_bytes(syn.frames_to_chunk(video[1:9])), 20, True)
        payloads.append(p)
        refs.append(frame0)
    batch = ufb.Codec(mine, 2)
    batch.set_skip_threshold(0.2)
    batch.add_ref_frames(np.concatenate(refs, 0))
    got, got_yuv = batch.decompress(payloads, W, H, 20, True, yuv=True)
    for s in range(2):
        one = ufb.Codec(mine, 1)
        one.set_skip_threshold(0.2)
        one.add_ref_frames(refs[s])
        single, single_yuv = one.decompress([payloads[s]], W, H, 20, True, yuv=True)
        assert np.array_equal(got[s], single[0])
        assert np.array_equal(got_yuv[s], single_yuv[0])  # stream s's frames land at its own offsets


def test_concurrent_codecs_match(ufb, syn, models):
    """Codecs decoding on their own CUDA streams from two host threads at once
    (how the bench overlaps one group's host rANS with another group's kernels)
    give the same frames as one after the other."""
    import threading
    import torch
    mine, _ = models["htl"]
    jobs = []
    for s in range(2):
        video = _frames(syn, 17, seed=70 + s)
        enc = ufb.Codec(mine, 1)
        enc.set_skip_threshold(0.2)
        enc.add_ref_frames(np.zeros((1, 3, H, W), np.int16))
        jobs.append([enc.compress(syn.frames_to_chunk(video[1 + 8 * k: 9 + 8 * k]), 20, k == 0)[0]
                     for k in range(2)])

    def decode(payloads, stream=None):
        c = ufb.Codec(mine, 1)
        c.set_skip_threshold(0.2)
        if stream is not None:
            c.set_stream(stream)
        c.add_ref_frames(np.zeros((1, 3, H, W), np.int16))
        return [c.decompress(p, W, H, 20, k == 0)[0] for k, p in enumerate(payloads)]

    want = [decode(j) for j in jobs]
    got = [None, None]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]

    def run(i):
        got[i] = decode(jobs[i], streams[i])

    threads = [threading.Thread(target=run, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for i in range(2):
        for a, b in zip(got[i], want[i]):
            assert np.array_equal(a, b)


def test_odd_size_padding(ufb, ora, ref, syn, models):
    """Width/height not multiples of 16: replicate padding and raw-frame crop."""
    mine, _ = models["htl"]
    vid_t = syn.prepared("htl", 2)
    w, h = 72, 40
    video = _frames(syn, 9, w=w, h=h, seed=9)
    frame0 = ora.from_bytes(syn.frames_to_chunk(video[:1]))
    frame0 = np.pad(frame0, ((0, 0), (0, 0), (0, 8), (0, 8)), mode="edge")  # reference frames are padded
    e = ref.model("htl", vid_t)
    e.set_skip_threshold(0.2)
    e.add_ref_feature_from_frame(frame0)
    want_payload, _ = e.compress(ora.from_bytes(syn.frames_to_chunk(video[1:9])), 30, False)
    c = ufb.Codec(mine, 1)
    c.set_skip_threshold(0.2)
    c.add_ref_frames(frame0)
    got_payloads, _ = c.compress(syn.frames_to_chunk(video[1:9]), 30, False)
    assert got_payloads[0] == want_payload


def test_truncated_payload_raises(ufb, syn, models):
    mine, _ = models["htl"]
    c = ufb.Codec(mine, 1)
    c.add_ref_frames(np.zeros((1, 3, H, W), np.int16))
    with pytest.raises(ufb.UfbError):
        c.decompress([b"\x00\x00\x80\x00\x01"], W, H, 20, False)


def test_p_frame_without_reference_raises(ufb, models):
    mine, _ = models["htl"]
    c = ufb.Codec(mine, 1)
    with pytest.raises(ufb.UfbError) as e:
        c.decompress([b"\x00\x00\x80\x00"], W, H, 20, False)
    assert "no reference" in str(e.value)


@pytest.mark.parametrize("table", ["random", "relu"])
def test_lut_tables_beyond_wsilu(ufb, ref, syn, table):
    """A WSiLU table with no narrow window (random: the kernels read the global
    table) and one that is max(v, 0) everywhere (a one-entry window) through the
    fused LUT and WSiLU4 epilogues."""
    t = dict(syn.prepared("htl", 2))
    rng = np.random.default_rng(5)
    v = np.arange(-32768, 32768)
    t["tables.wsilu"] = (rng.integers(-32768, 32768, 65536) if table == "random"
                         else np.maximum(v, 0)).astype(np.int16)
    mine, theirs = ufb.Model("htl", t), ref.model("htl", t)
    x = rng.integers(-6000, 6000, (1, 512, 6, 9)).astype(np.int16)
    assert np.array_equal(mine.run("feature_extractor", x), theirs.run("feature_extractor", x))


@pytest.mark.parametrize("extreme", [32639, 32767])
def test_signed_split_weight_extremes(ufb, ref, syn, extreme):
    """Weights at the edge of the signed byte split (<= 32639 uses it, 32767
    forces the unsigned split) must give identical module outputs."""
    t = dict(syn.prepared("htl", 2))
    rng = np.random.default_rng(extreme)
    for name in ("feature_extractor.conv.0.dc.0.weight", "feature_extractor.conv.0.ffn.0.weight",
                 "feature_extractor.conv.1.ffn.2.weight"):
        w = t[name].copy()
        flat = w.reshape(-1)
        idx = rng.choice(flat.size, flat.size // 3, replace=False)
        flat[idx] = rng.choice(np.array([extreme, -32768, -1, 127, -128, 128, 255, -255], np.int16), idx.size)
        t[name] = w
    mine, theirs = ufb.Model("htl", t), ref.model("htl", t)
    x = rng.integers(-6000, 6000, (1, 512, 6, 9)).astype(np.int16)
    assert np.array_equal(mine.run("feature_extractor", x), theirs.run("feature_extractor", x))


def _narrow_ok(w):
    """Host restatement of the engine's narrow-recombination bound: per output
    channel, 4096 + sum_k 32768 |wl| + 65280 |wh| <= 2^31 - 1 (signed byte
    split when every weight is <= 32639, else unsigned)."""
    w = w.astype(np.int64).reshape(w.shape[0], -1)
    lo = ((w + 128) & 255) - 128 if w.max() <= 32639 else (w & 255)
    hi = (w - lo) >> 8
    return bool((4096 + (32768 * np.abs(lo) + 65280 * np.abs(hi)).sum(1)).max() <= 2**31 - 1)


@pytest.mark.parametrize("module,shapes", [
    ("feature_extractor", [(1, 512, 8, 10)]),
    ("recon_head.conv.3", [(1, 512, 8, 8)]),
    ("y_spatial_prior", [(1, 512, 3, 5)]),
    ("decoder", [(1, 256, 4, 4), (1, 512, 8, 8)]),
])
def test_narrow_recombination_matches_general(ufb, syn, models, module, shapes):
    """Most HT-L layers (1x1 convolutions of up to 512 input channels) keep
    LL + 256 X + 4096 within 32 bits and use the narrow recombination; with the
    switch off every layer takes the general one.  Both must give the
    reference's outputs."""
    t = syn.prepared("htl", 2)
    assert sum(_narrow_ok(v) for k, v in t.items() if k.startswith(module) and k.endswith(".weight")
               and v.shape[1] > 1) > 0
    mine, theirs = models["htl"]
    rng = np.random.default_rng(17)
    args = [rnd(rng, s, -9000, 9000) for s in shapes]
    q = "q_decoder" if module == "decoder" else None
    want = theirs.run(module, *(args + ([theirs.parameter(q, 20)] if q else [])))
    got = mine.run(module, *args, q_name=q, qp=20)
    ufb.set_conv_narrow(False)
    try:
        general = mine.run(module, *args, q_name=q, qp=20)
    finally:
        ufb.set_conv_narrow(True)
    assert np.array_equal(got, want)
    assert np.array_equal(general, want)


@pytest.mark.parametrize("margin", ["inside", "outside"])
def test_narrow_bound_edges(ufb, ref, syn, margin):
    """Weights with |low byte| = 127 everywhere and a few high bytes put the
    narrow bound within 2^24 of int32's limit ("inside": narrow path) or just
    past it ("outside": general path); inputs of -32768 and 32767 then drive
    LL + 256 X + 4096 to that limit.  The module must match the reference."""
    t = dict(syn.prepared("htl", 2))
    rng = np.random.default_rng(23)
    sign_in = rng.choice(np.array([-1, 1]), 512)  # one sign pattern over the input channels
    for name in ("feature_extractor.conv.0.dc.0.weight", "feature_extractor.conv.0.ffn.0.weight",
                 "feature_extractor.conv.0.dc.3.weight"):
        co, ci = t[name].shape[:2]
        sign = np.broadcast_to(sign_in[:ci], (co, ci)).copy()
        sign[1::2] *= -1  # odd output channels take the opposite pattern
        w = sign * 127
        # 4096 + 512 * 127 * 32768 leaves 16,773,119 for the high bytes: 256
        # of them at |wh| = 1 fit (65280 each), 257 do not
        n_hi = 256 if margin == "inside" else 300
        w[:, :n_hi] += sign[:, :n_hi] * 256
        w = w.astype(np.int16).reshape(t[name].shape)
        assert _narrow_ok(w) == (margin == "inside")
        t[name] = w
    mine, theirs = ufb.Model("htl", t), ref.model("htl", t)
    # pixels whose channels follow the sign pattern (32767 / -32768): every
    # output channel of dc.0 sits at +-(the bound) before the rounding
    x = np.where(sign_in[None, :, None, None] > 0, np.int16(32767), np.int16(-32768))
    x = np.broadcast_to(x, (1, 512, 6, 9)).copy()
    x[..., 3:6] = rng.choice(np.array([-32768, 32767, -32767, 0, 255, -256], np.int16), (1, 512, 6, 3))
    x[..., 6:] = rng.integers(-32768, 32768, (1, 512, 6, 3))
    x[:, :, 3:] = -x[:, :, 3:]  # and the opposite signs (-(-32768) wraps to -32768)
    assert np.array_equal(mine.run("feature_extractor", x), theirs.run("feature_extractor", x))


def test_depthwise_narrow_many_tiles_per_cta(ufb, models):
    """The narrow depthwise instance (every dc.2 of the seeded model) with the
    grids capped at two CTAs: each depthwise CTA walks 12 of the 24 tiles
    (4 channel blocks x 3 x 2), refilling both window buffers behind the
    warps' release barriers."""
    mine, theirs = models["htl"]
    x = rnd(np.random.default_rng(43), (1, 512, 12, 36))
    want = theirs.run("feature_extractor", x)
    ufb.set_conv_max_ctas(2)
    try:
        got = mine.run("feature_extractor", x)
    finally:
        ufb.set_conv_max_ctas(0)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("margin", ["inside", "outside"])
def test_depthwise_narrow_bound_edges(ufb, ref, syn, margin):
    """The depthwise dc.2 sums run in one int32 when, per channel,
    32768 sum|w| + 4096 + 8192 |bias| fits ("inside": sum|w| = 57343 with
    |bias| at its maximum) and in split byte sums otherwise ("outside").  An
    identity table and an identity dc.0 hand the input to dc.2 unchanged, so
    inputs at 32767 / -32768 following the weight signs drive the sum to the
    bound; a wrapped sum would flip the sign of dc.3's result."""
    t = dict(syn.prepared("htl", 2))
    rng = np.random.default_rng(29)
    t["tables.wsilu"] = np.arange(-32768, 32768).astype(np.int16)
    pre = "feature_extractor.conv.0."
    t[pre + "dc.0.weight"] = (8192 * np.eye(512)).astype(np.int16).reshape(512, 512, 1, 1)
    t[pre + "dc.0.bias"] = np.zeros(512, np.int16)
    sign = rng.choice(np.array([-1, 1]), 512)
    taps = np.array([6371] * 8 + [6375 if margin == "inside" else 6432])
    t[pre + "dc.2.weight"] = (sign[:, None] * taps[None, :]).astype(np.int16).reshape(512, 1, 3, 3)
    t[pre + "dc.2.bias"] = np.where(np.arange(512) % 2, 32767, -32768).astype(np.int16)
    w = t[pre + "dc.2.weight"].astype(np.int64).reshape(512, 9)
    bound = 4096 + 8192 * np.abs(t[pre + "dc.2.bias"].astype(np.int64)) + 32768 * np.abs(w).sum(1)
    assert (bound.max() <= 2**31 - 1) == (margin == "inside")
    mine, theirs = ufb.Model("htl", t), ref.model("htl", t)
    x = np.where(sign[None, :, None, None] > 0, np.int16(32767), np.int16(-32768))
    x = np.broadcast_to(x, (1, 512, 8, 9)).copy()
    x[:, :, 4:6] = -x[:, :, 4:6]
    x[:, :, 6:] = rng.integers(-32768, 32768, (1, 512, 2, 9))
    assert np.array_equal(mine.run("feature_extractor", x), theirs.run("feature_extractor", x))
