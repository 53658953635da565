"""CPU: the oracle restatement is pinned to the reference's own known-answer
cases (golden fixtures made from the reference's compiled CPU path) and, when
oracle/_ref is built, to the reference on seeded random cases."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "model_free.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def test_bytes_all_values(ora, gold):
    assert np.array_equal(ora.from_bytes(gold["bytes_in"]), gold["bytes_out"])


def test_rna_ties(ora, gold):
    got = np.array([ora.divide_round(int(v), 512) for v in gold["ties_in"]], np.int64)
    assert np.array_equal(got, gold["ties_out"])
    assert list(got) == [-2, -2, -1, -1, -1, 0, 0, 1, 1, 1, 2, 2]


def test_elementwise_golden(ora, gold):
    v, o = gold["ew_values"], gold["ew_other"]
    assert np.array_equal(ora.add(v, o), gold["ew_add"])
    assert np.array_equal(ora.multiply(v, gold["ew_scale"]), gold["ew_mul"])
    assert np.array_equal(ora.lookup(v, gold["ew_lut"]), gold["ew_lookup"])
    assert np.array_equal(ora.wsilu4(v, gold["ew_lut"]), gold["ew_wsilu4"])


@pytest.mark.parametrize("i", range(8))
def test_conv_golden(ora, gold, i):
    ci, co, k, stride, pad, groups = [int(g) for g in gold[f"conv{i}_geom"]]
    got = ora.conv2d(gold[f"conv{i}_x"], gold[f"conv{i}_w"], gold[f"conv{i}_b"], stride, pad, groups)
    assert np.array_equal(got, gold[f"conv{i}_out"])


def test_conv_extremes_saturate(gold):
    # all-32767 inputs with +-full-scale weights saturate both ways (int64 accumulator)
    outs = [gold[f"conv{i}_out"] for i in range(4, 8)]
    assert (outs[0] == -32768).all() and (outs[1] == 32767).all()


@pytest.mark.parametrize("seed", range(4))
def test_conv_random_vs_reference(ora, ref, seed):
    rng = np.random.default_rng(100 + seed)
    ci, co = int(rng.integers(1, 40)), int(rng.integers(1, 40))
    k = int(rng.choice([1, 3]))
    stride = int(rng.choice([1, 2]))
    groups = 1 if seed % 2 == 0 else int(np.gcd(ci, co))
    h, w = int(rng.integers(k, 20)), int(rng.integers(k, 20))
    x = rng.integers(-32768, 32768, (2, ci, h, w)).astype(np.int16)
    wt = rng.integers(-32768, 32768, (co, ci // groups, k, k)).astype(np.int16)
    b = rng.integers(-32768, 32768, (co,)).astype(np.int16)
    assert np.array_equal(ora.conv2d(x, wt, b, stride, k // 2, groups), ref.conv2d(x, wt, b, stride, k // 2, groups))


def test_conv_int32_bias_vs_reference(ora, ref):
    rng = np.random.default_rng(0)
    x = rng.integers(-4096, 4097, (1, 16, 12, 20)).astype(np.int16)
    w = rng.integers(-256, 257, (16, 16, 3, 3)).astype(np.int16)
    b = rng.integers(-(1 << 16), (1 << 16) + 1, (16,)).astype(np.int32)
    assert np.array_equal(ora.conv2d(x, w, b, 1, 1), ref.conv2d(x, w, b, 1, 1))


def test_elementwise_random_vs_reference(ora, ref):
    rng = np.random.default_rng(7)
    a = rng.integers(-32768, 32768, (2, 8, 5, 6)).astype(np.int16)
    b = rng.integers(-32768, 32768, (2, 8, 5, 6)).astype(np.int16)
    c = rng.integers(-32768, 32768, (2, 8, 5, 6)).astype(np.int16)
    assert np.array_equal(ora.add(a, b, c), ref.add(a, b, c))
    for shape in [(1, 8, 1, 1), (2, 8, 5, 6), (1, 1, 5, 6)]:
        s = rng.integers(-32768, 32768, shape).astype(np.int16)
        assert np.array_equal(ora.multiply(a, s), ref.multiply(a, s))
    t8 = rng.integers(0, 256, 65536).astype(np.uint8)
    assert np.array_equal(ora.lookup(a, t8), ref.lookup(a, t8))
    assert np.array_equal(ora.symbols(a), ref.symbols(a))
    assert np.array_equal(ora.reciprocal(a), ref.reciprocal(a))
    for f in (2, 8):
        x = rng.integers(-32768, 32768, (1, 3 * f * f, 4, 5)).astype(np.int16)
        assert np.array_equal(ora.pixel_shuffle(x, f), ref.pixel_shuffle(x, f))
        y = rng.integers(-32768, 32768, (1, 3, 4 * f, 5 * f)).astype(np.int16)
        assert np.array_equal(ora.pixel_unshuffle(y, f), ref.pixel_shuffle(y, f, unshuffle=True))


def test_warp_identity_and_shift(ora):
    rng = np.random.default_rng(1)
    f = rng.integers(-4096, 4097, (1, 4, 9, 11)).astype(np.int16)
    zero = np.zeros((1, 2, 9, 11), np.int16)
    assert np.array_equal(ora.warp(f, zero), f)
    one = zero.copy()
    one[:, 0] = 512  # +1 px in x: out[x] = f[min(x+1, W-1)]
    want = np.concatenate([f[..., 1:], f[..., -1:]], axis=-1)
    assert np.array_equal(ora.warp(f, one), want)


def test_warp_close_to_float_semantics(ora):
    rng = np.random.default_rng(2)
    f = rng.integers(-4096, 4097, (1, 3, 16, 20)).astype(np.int16)
    flow = np.round(512 * (rng.normal(0, 4, (1, 2, 16, 20)) + np.array([3.25, -1.5])[None, :, None, None]))
    flow = flow.astype(np.int16)
    diff = np.abs(ora.warp(f, flow).astype(np.float64) - ora.warp_float(f, flow))
    assert diff.max() <= 1.0


@pytest.mark.parametrize("size", [(72, 80), (70, 78), (352, 626)])
def test_raw_frame_vs_reference_codec(ora, ref, size):
    """The C restatement of raw_frame equals the reference's own
    IntegerCodec::raw_frame (src/integer_codec.cpp:294-323) on cropped, padded
    and saturating frames, including every rounding tie of the luma formula."""
    h, w = size
    rng = np.random.default_rng(h * 1000 + w)
    fh, fw = (h + 15) // 16 * 16, (w + 15) // 16 * 16
    frame = rng.integers(-1400, 1400, (1, 3, fh, fw)).astype(np.int16)
    frame.reshape(-1)[: 65536] = np.arange(-32768, 32768, dtype=np.int64).astype(np.int16)[: min(65536, frame.size)]
    want = ref.raw_frame(frame, h, w)
    assert np.array_equal(ora.raw_frame(frame[0], h, w).reshape(-1), want)


def test_reference_codec_stream_roundtrip(ref, syn):
    """The reference's IntegerCodec decode loop over its own encoded archive:
    the decoded-YUV SHA-256 it returns is the hash of the frames its sink saw."""
    import hashlib

    import oracle.stream as st
    img_t, vid_t = syn.prepared("image", 1), syn.prepared("htl", 2)
    ii, vi = st.prepared_identity(img_t, "image", "a"), st.prepared_identity(vid_t, "htl", "b")
    video = syn.synthetic_video(64, 64, 9, 5)
    data, frames, packets = ref.codec(img_t, ii, vid_t, vi, "htl", 0.2).encode(video, 64, 64, 0, 20, 8, -1)
    assert (frames, packets) == (9, 2)
    digest, yuv, p = ref.codec(img_t, ii, vid_t, vi, "htl", 0.2).decode(data, 9, 2, 64, 64)
    assert p == 2 and len(yuv) == 9
    assert hashlib.sha256(b"".join(y.tobytes() for y in yuv)).hexdigest() == digest


def _raw_frame_int32(frame, h, w):
    """The 32-bit forms the GPU's raw_frame kernel evaluates (engine_kernels.cu):
    luma rna((v + 256) * 255 / 512) with the divide as shifts, chroma
    floor((s + 1024) * 255 / 2048) = ((s + 1024) * 255) >> 11 over each 2 x 2 block."""
    f = frame.reshape(3, frame.shape[-2], frame.shape[-1]).astype(np.int32)
    t = (f[0, :h, :w] + 256) * 255
    planes = [np.where(t < 0, -((256 - t) >> 9), (t + 256) >> 9)]
    ch, cw = h // 2, w // 2
    for comp in (1, 2):
        c = f[comp, :2 * ch, :2 * cw]
        s = c[0::2, 0::2] + c[1::2, 0::2] + c[0::2, 1::2] + c[1::2, 1::2]
        planes.append(((s + 1024) * 255) >> 11)
    return np.concatenate([np.clip(p, 0, 255).astype(np.uint8).reshape(-1) for p in planes])


@pytest.mark.parametrize("size", [(64, 64), (72, 80), (352, 626)])
def test_raw_frame_int32_forms_vs_reference(ref, size):
    """The GPU kernel's shift forms give the reference's IntegerCodec::raw_frame
    bytes: every int16 value in luma, chroma blocks at both saturation ends
    and at every rounding boundary region."""
    h, w = size
    rng = np.random.default_rng(h + 7 * w)
    fh, fw = (h + 15) // 16 * 16, (w + 15) // 16 * 16
    frame = rng.integers(-32768, 32768, (1, 3, fh, fw)).astype(np.int16)
    n = min(65536, h * w)
    frame[0, 0].reshape(-1)[:n] = np.arange(-32768, 32768, dtype=np.int64).astype(np.int16)[:n]
    frame[0, 1, : fh // 2] = 32767
    frame[0, 2, : fh // 2] = -32768
    frame[0, 1:, fh // 2:] = rng.integers(-1300, 1300, (2, fh - fh // 2, fw))
    assert np.array_equal(_raw_frame_int32(frame, h, w), ref.raw_frame(frame, h, w))


def test_q9_multiply_int32_form_vs_reference(ref):
    """sat(rna(v * q / 512)) as the GPU's multiply kernels evaluate it in 32
    bits (|v * q| <= 2^30) equals the reference's int16::multiply over every
    int16 v and multipliers at the extremes and around the rounding unit."""
    q = np.array([-32768, -32767, -513, -512, -511, -1, 0, 1, 255, 256, 511, 512, 513, 1024, 32766, 32767],
                 np.int16)
    x = np.arange(-32768, 32768, dtype=np.int64).astype(np.int16).reshape(1, 16, 64, 64)
    p = x.astype(np.int32) * q.astype(np.int32)[None, :, None, None]
    sg = p >> 31
    r = ((((p ^ sg) - sg) + 256) >> 9 ^ sg) - sg
    mine = np.clip(r, -32768, 32767).astype(np.int16)
    assert np.array_equal(mine, ref.multiply(x, q.reshape(1, 16, 1, 1)))


def test_depthwise_narrow_form_vs_reference(ref):
    """The narrow depthwise instance's arithmetic (dwconv.cu): per channel
    s = S + 4096 + 8192 bias in one int32 (every channel inside
    32768 sum|w| + 4096 + 8192 |bias| <= 2^31 - 1), output
    sat((s - [s < 4096 + 8192 bias]) >> 13), equals the reference's depthwise
    conv; the weights sit at the bound's edge and the inputs at the extremes."""
    rng = np.random.default_rng(5)
    c, h, w = 24, 9, 11
    bias = rng.integers(-32768, 32768, c).astype(np.int16)
    room = (2**31 - 1 - 4096 - 8192 * np.abs(bias.astype(np.int64))) // 32768  # largest sum|w| per channel
    wt = np.zeros((c, 1, 3, 3), np.int16)
    for ch in range(c):
        taps = rng.integers(0, 1 << 12, 9).astype(np.float64)
        taps = np.floor(taps / taps.sum() * min(room[ch], 9 * 32767)).astype(np.int64)
        wt[ch, 0] = (taps * rng.choice([-1, 1], 9)).reshape(3, 3).astype(np.int16)
    wsum = np.abs(wt.astype(np.int64)).reshape(c, 9).sum(1)
    assert (32768 * wsum + 4096 + 8192 * np.abs(bias.astype(np.int64)) <= 2**31 - 1).all()
    x = rng.choice(np.array([-32768, 32767, -1, 0, 1, 4096, -4096], np.int16), (2, c, h, w))
    xp = np.pad(x.astype(np.int64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    S = sum(xp[:, :, ky:ky + h, kx:kx + w] * wt[None, :, 0, ky, kx, None, None].astype(np.int64)
            for ky in range(3) for kx in range(3))
    s0 = (4096 + 8192 * bias.astype(np.int64))[None, :, None, None]
    s = S + s0
    assert (np.abs(s) <= 2**31 - 1).all()
    s = s.astype(np.int32)
    mine = np.clip((s - (s < s0).astype(np.int32)) >> 13, -32768, 32767).astype(np.int16)
    assert np.array_equal(mine, ref.conv2d(x, wt, bias, 1, 1, c))


def test_narrow_recombination_form_vs_reference(ref):
    """The tensor-core epilogue's narrow recombination (conv_tc.cu): with
    x = xl + 256 xh (xl unsigned, xh signed bytes) and w = wl + 256 wh (signed
    split), LL = sum xl wl, X = sum xl wh + xh wl, HH = sum xh wh and
    P = LL + 256 X inside int32 (4096 + sum 32768 |wl| + 65280 |wh| <= 2^31 - 1),
    rna(S / 8192) = 8 HH + ((P + 4096 + (fl >> 31)) >> 13) with
    fl = 8 HH + (P >> 13); plus the bias and saturation this equals the
    reference's 1x1 convolution at the bound's edge with inputs at the extremes."""
    rng = np.random.default_rng(9)
    ci, co, n = 512, 8, 64
    sign = rng.choice(np.array([-1, 1]), (co, ci))
    w = sign * 127
    w[:, :256] += sign[:, :256] * 256  # 4096 + 512 * 127 * 32768 + 256 * 65280 just below 2^31
    x = np.where(rng.random((n, ci)) < 0.5, 32767, -32768)
    x[: n // 2] = np.where(sign[0] > 0, 32767, -32768)  # rows that drive channel 0 to the bound
    x[n - 4:] = rng.integers(-32768, 32768, (4, ci))
    b = rng.integers(-32768, 32768, co)
    wl = ((w + 128) & 255) - 128
    wh = (w - wl) >> 8
    xl, xh = x & 255, x >> 8
    LL, HH = xl @ wl.T, xh @ wh.T
    X = xl @ wh.T + xh @ wl.T
    assert (4096 + (32768 * np.abs(wl) + 65280 * np.abs(wh)).sum(1) <= 2**31 - 1).all()
    P = LL + 256 * X
    assert (np.abs(P + 4096) <= 2**31 - 1).all()
    P = P.astype(np.int32)
    H8 = (8 * HH).astype(np.int32)
    fl = H8 + (P >> 13)
    r = H8 + ((P + 4096 + (fl >> 31)) >> 13) + b[None, :]
    mine = np.clip(r, -32768, 32767).astype(np.int16)
    want = ref.conv2d(x.astype(np.int16).reshape(n, ci, 1, 1), w.astype(np.int16).reshape(co, ci, 1, 1),
                      b.astype(np.int16), 1, 0)
    assert np.array_equal(mine, want.reshape(n, co))
