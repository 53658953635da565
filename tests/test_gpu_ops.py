"""GPU parity of the operator-level C ABI against the CPU oracle (bit-exact).

Mirrors the reference's CUDA checks in tests/model_free.cpp:580-621
(elementwise parity, four convolution geometries, int64-accumulator extremes
through all three convolution variants) and widens them to the HT-L layer
shapes, K/N tails and the config-1 convolution.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "model_free.npz")


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def N(t):
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def _status_clean(ufb):
    assert ufb.device_status(0) == 0


@pytest.mark.parametrize("variant", ["auto", "generic", "baseline"])
@pytest.mark.parametrize("i", range(8))
def test_conv_golden(ufb, dev, gold, i, variant):
    ci, co, k, stride, pad, groups = [int(g) for g in gold[f"conv{i}_geom"]]
    x, w, b = gold[f"conv{i}_x"], gold[f"conv{i}_w"], gold[f"conv{i}_b"]
    got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev), stride, stride, pad, pad, groups, variant=variant)
    assert np.array_equal(N(got), gold[f"conv{i}_out"])
    _status_clean(ufb)


def test_elementwise_golden(ufb, dev, gold):
    v, o = T(gold["ew_values"], dev), T(gold["ew_other"], dev)
    lut = T(gold["ew_lut"], dev)
    assert np.array_equal(N(ufb.add([v, o])), gold["ew_add"])
    assert np.array_equal(N(ufb.multiply(v, T(gold["ew_scale"], dev))), gold["ew_mul"])
    assert np.array_equal(N(ufb.lookup(v, lut)), gold["ew_lookup"])
    assert np.array_equal(N(ufb.wsilu4(v, lut)), gold["ew_wsilu4"])
    assert np.array_equal(N(ufb.from_bytes(T(gold["bytes_in"], dev))), gold["bytes_out"])


def test_elementwise_random(ufb, ora, dev):
    rng = np.random.default_rng(3)
    shape = (2, 16, 9, 13)
    a, b, c, d = (rng.integers(-32768, 32768, shape).astype(np.int16) for _ in range(4))
    for k in (2, 3, 4):
        ops = [a, b, c, d][:k]
        assert np.array_equal(N(ufb.add([T(x, dev) for x in ops])), ora.add(*ops))
    for sshape in [(1, 16, 1, 1), shape, (1, 1, 9, 13), (2, 1, 1, 1)]:
        s = rng.integers(-32768, 32768, sshape).astype(np.int16)
        assert np.array_equal(N(ufb.multiply(T(a, dev), T(s, dev))), ora.multiply(a, s))
    t16 = rng.integers(-32768, 32768, 65536).astype(np.int16)
    t8 = rng.integers(0, 256, 65536).astype(np.uint8)
    assert np.array_equal(N(ufb.lookup(T(a, dev), T(t16, dev))), ora.lookup(a, t16))
    assert np.array_equal(N(ufb.lookup(T(a, dev), T(t8, dev))), ora.lookup(a, t8))
    assert np.array_equal(N(ufb.wsilu4(T(a, dev), T(t16, dev))), ora.wsilu4(a, t16))


@pytest.mark.parametrize("ci,co,hw", [(16, 16, (7, 9)), (64, 64, (16, 16)), (128, 128, (11, 13)),
                                      (192, 512, (8, 10)), (512, 512, (9, 17)), (512, 2048, (4, 8)),
                                      (1024, 512, (6, 7)), (768, 256, (5, 8)), (256, 192, (12, 12)),
                                      (2048, 512, (3, 5)), (100, 40, (5, 5))])
def test_conv1x1_shapes(ufb, ora, dev, ci, co, hw):
    rng = np.random.default_rng(ci * 7 + co)
    x = rng.integers(-32768, 32768, (2, ci) + hw).astype(np.int16)
    w = rng.integers(-32768, 32768, (co, ci, 1, 1)).astype(np.int16)
    b = rng.integers(-32768, 32768, (co,)).astype(np.int16)
    got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev))
    assert np.array_equal(N(got), ora.conv2d(x, w, b))
    _status_clean(ufb)


@pytest.mark.parametrize("ci,co,hw", [(64, 64, (9, 20)), (256, 128, (10, 12)), (32, 80, (5, 33)),
                                      (256, 2048, (4, 6)), (8, 6, (7, 8))])
def test_conv3x3_shapes(ufb, ora, dev, ci, co, hw):
    rng = np.random.default_rng(ci + co)
    x = rng.integers(-32768, 32768, (1, ci) + hw).astype(np.int16)
    w = rng.integers(-32768, 32768, (co, ci, 3, 3)).astype(np.int16)
    b = rng.integers(-32768, 32768, (co,)).astype(np.int16)
    got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev), 1, 1, 1, 1)
    assert np.array_equal(N(got), ora.conv2d(x, w, b, 1, 1))
    _status_clean(ufb)


def test_conv_config1_int32_bias(ufb, ora, dev):
    rng = np.random.default_rng(0)
    x = rng.integers(-4096, 4097, (1, 64, 88, 160)).astype(np.int16)
    w = rng.integers(-256, 257, (64, 64, 3, 3)).astype(np.int16)
    b = rng.integers(-(1 << 16), (1 << 16) + 1, (64,)).astype(np.int32)
    got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev), 1, 1, 1, 1)
    assert np.array_equal(N(got), ora.conv2d(x, w, b, 1, 1))


@pytest.mark.parametrize("kernel", [1, 3])
@pytest.mark.parametrize("sign", [-1, 1])
@pytest.mark.parametrize("ci", [32, 2048])
def test_accumulator_extremes(ufb, ora, dev, kernel, sign, ci):
    x = np.full((1, ci, 5, 5), 32767, np.int16)
    w = np.full((32, ci, kernel, kernel), 32767 if sign == 1 else -32768, np.int16)
    # mix in the low-byte extremes too: alternate 32767 and -32768 / -1 / 255
    w.reshape(-1)[::3] = -1
    x.reshape(-1)[::5] = -32768
    b = np.zeros(32, np.int16)
    for variant in ("auto", "generic", "baseline"):
        got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev), 1, 1, kernel // 2, kernel // 2, variant=variant)
        assert np.array_equal(N(got), ora.conv2d(x, w, b, 1, kernel // 2))


@pytest.mark.parametrize("ci,kernel", [(910, 3), (8192, 1)])
def test_unsigned_low_byte_bound(ufb, ora, dev, ci, kernel):
    # low bytes 255 everywhere (value = 255 + 256 * hi) stress the u8 x u8
    # accumulator at the tensor-core path's longest reduction (K <= 8192)
    x = np.full((1, ci, 3, 3), 255, np.int16)
    w = np.full((16, ci, kernel, kernel), 255, np.int16)
    x.reshape(-1)[::7] = -32768
    got = ufb.conv2d(T(x, dev), T(w, dev), None, 1, 1, kernel // 2, kernel // 2)
    assert np.array_equal(N(got), ora.conv2d(x, w, None, 1, kernel // 2))


def test_large_reduction_uses_direct_path(ufb, ora, dev):
    rng = np.random.default_rng(5)
    x = rng.integers(-32768, 32768, (1, 4000, 3, 3)).astype(np.int16)  # 36000 > 8192
    w = rng.integers(-32768, 32768, (4, 4000, 3, 3)).astype(np.int16)
    got = ufb.conv2d(T(x, dev), T(w, dev), None, 1, 1, 1, 1)
    assert np.array_equal(N(got), ora.conv2d(x, w, None, 1, 1))


@pytest.mark.parametrize("ctas", [0, 3])
@pytest.mark.parametrize("kernel", [1, 3])
def test_conv_many_tiles(ufb, ora, dev, kernel, ctas):
    """Hundreds of output tiles per launch, so every CTA alternates between the
    two TMEM accumulator sets; about 1 in 8192 outputs is an exact rounding
    tie, so both tie signs occur many times."""
    rng = np.random.default_rng(11 + kernel)
    hw = (160, 128) if kernel == 1 else (48, 40)
    ci = 128 if kernel == 1 else 64
    x = rng.integers(-32768, 32768, (2, ci) + hw).astype(np.int16)
    w = rng.integers(-32768, 32768, (192, ci, kernel, kernel)).astype(np.int16)
    b = rng.integers(-32768, 32768, (192,)).astype(np.int16)
    ufb.set_conv_max_ctas(ctas)
    try:
        got = ufb.conv2d(T(x, dev), T(w, dev), T(b, dev), 1, 1, kernel // 2, kernel // 2)
    finally:
        ufb.set_conv_max_ctas(0)
    assert np.array_equal(N(got), ora.conv2d(x, w, b, 1, kernel // 2))
    _status_clean(ufb)


def test_depthwise_and_stride2(ufb, ora, dev):
    rng = np.random.default_rng(9)
    x = rng.integers(-32768, 32768, (1, 64, 10, 12)).astype(np.int16)
    wd = rng.integers(-32768, 32768, (64, 1, 3, 3)).astype(np.int16)
    b = rng.integers(-32768, 32768, (64,)).astype(np.int16)
    assert np.array_equal(N(ufb.conv2d(T(x, dev), T(wd, dev), T(b, dev), 1, 1, 1, 1, 64)),
                          ora.conv2d(x, wd, b, 1, 1, 64))
    w2 = rng.integers(-32768, 32768, (32, 64, 3, 3)).astype(np.int16)
    assert np.array_equal(N(ufb.conv2d(T(x, dev), T(w2, dev), None, 2, 2, 1, 1)), ora.conv2d(x, w2, None, 2, 1))


@pytest.mark.parametrize("n,ci,co,h,w,k,ctas", [
    (1, 512, 256, 68, 120, 3, 0),    # HT-L encoder.down at 1080p latent-feature scale /2
    (2, 384, 256, 45, 37, 3, 0),     # image enc.enc_2.6 shape, odd sizes, batch 2
    (1, 64, 40, 33, 70, 3, 3),       # channel tails (K and N), few CTAs walking many tiles
    (1, 128, 96, 21, 22, 1, 0),      # 1x1 stride 2 (spatial tensor map)
    (1, 16, 16, 3, 3, 3, 0),         # a single output row of two pixels
])
def test_stride2_tensor_core(ufb, ora, dev, n, ci, co, h, w, k, ctas):
    """Stride-2 convolutions (encoder.down, enc.enc_2.6) on the tensor cores:
    each tap's activation box is a 2x-sized TMA box with element stride 2."""
    rng = np.random.default_rng(ci + co + h)
    x = rng.integers(-32768, 32768, (n, ci, h, w)).astype(np.int16)
    wt = rng.integers(-32768, 32768, (co, ci, k, k)).astype(np.int16)
    b = rng.integers(-32768, 32768, (co,)).astype(np.int16)
    ufb.set_conv_max_ctas(ctas)
    try:
        got = ufb.conv2d(T(x, dev), T(wt, dev), T(b, dev), 2, 2, k // 2, k // 2)
    finally:
        ufb.set_conv_max_ctas(0)
    assert np.array_equal(N(got), ora.conv2d(x, wt, b, 2, k // 2))
    _status_clean(ufb)


@pytest.mark.parametrize("n,c,h,w", [(1, 64, 10, 12), (2, 256, 37, 45), (1, 192, 16, 33), (1, 512, 35, 50),
                                     (3, 4, 5, 7), (1, 132, 1, 1)])
def test_depthwise_split_kernel(ufb, ora, dev, n, c, h, w):
    """The engine's split-layout depthwise kernel (through conv2d's depthwise
    route): strip, column-block and channel-block edges, odd sizes, 1x1 images."""
    rng = np.random.default_rng(c * 31 + h)
    x = rng.integers(-32768, 32768, (n, c, h, w)).astype(np.int16)
    wd = rng.integers(-32768, 32768, (c, 1, 3, 3)).astype(np.int16)
    b = rng.integers(-32768, 32768, (c,)).astype(np.int16)
    for bias in (T(b, dev), None):
        got = ufb.conv2d(T(x, dev), T(wd, dev), bias, 1, 1, 1, 1, c)
        assert np.array_equal(N(got), ora.conv2d(x, wd, b if bias is not None else None, 1, 1, c))
    _status_clean(ufb)


@pytest.mark.parametrize("ctas", [1, 5])
def test_depthwise_many_tiles_per_cta(ufb, ora, dev, ctas):
    """With the grid capped every depthwise CTA walks many tiles, so both
    window buffers are refilled many times behind the warps' release
    barriers (60 tiles: 2 channel blocks x 3 x 5 per image, 2 images)."""
    rng = np.random.default_rng(41 + ctas)
    n, c, h, w = 2, 256, 37, 45
    x = rng.integers(-32768, 32768, (n, c, h, w)).astype(np.int16)
    wd = rng.integers(-32768, 32768, (c, 1, 3, 3)).astype(np.int16)
    b = rng.integers(-32768, 32768, (c,)).astype(np.int16)
    ufb.set_conv_max_ctas(ctas)
    try:
        got = ufb.conv2d(T(x, dev), T(wd, dev), T(b, dev), 1, 1, 1, 1, c)
    finally:
        ufb.set_conv_max_ctas(0)
    assert np.array_equal(N(got), ora.conv2d(x, wd, b, 1, 1, c))
    _status_clean(ufb)


@pytest.mark.parametrize("xv,wv", [(-32768, -32768), (32767, -32768), (-32768, 32767), (-1, 4096), (3, 4096),
                                   (-3, 4096), (255, 32767), (-256, -32768)])
def test_depthwise_extremes_and_ties(ufb, ora, dev, xv, wv):
    """Constant inputs and weights at the int16 extremes (the largest partial
    sums of the byte-plane dot products) and exact half-way cases (S = +-4096
    mod 8192, rounded away from zero), with and without a saturating bias."""
    c = 136
    x = np.full((2, c, 9, 19), xv, np.int16)
    wd = np.full((c, 1, 3, 3), wv, np.int16)
    wd[1::3, 0, 0, :] = 0  # some channels see fewer taps
    wd[2::5, 0, :, 1] = -wd[2::5, 0, :, 1]
    for b in (np.zeros(c, np.int16), np.full(c, -32768, np.int16), np.arange(c, dtype=np.int16) * 241):
        got = ufb.conv2d(T(x, dev), T(wd, dev), T(b, dev), 1, 1, 1, 1, c)
        assert np.array_equal(N(got), ora.conv2d(x, wd, b, 1, 1, c))
    _status_clean(ufb)


def _config2_flow(rng, n, h, w, sigma=4.0, shift=(3.25, -1.5)):
    """BASELINE config 2's flow: int16 Q9 of N(0, sigma^2) px per pixel plus a global translation."""
    flow = np.round(512 * (rng.normal(0, sigma, (n, 2, h, w)) + np.array(shift)[None, :, None, None]))
    return np.clip(flow, -32768, 32767).astype(np.int16)


@pytest.mark.parametrize("n,c,h,w,sigma,shift,lo,hi", [
    (1, 64, 176, 320, 4.0, (3.25, -1.5), -4096, 4097),        # BASELINE config 2 (TMA-staged windows)
    (1, 8, 44, 80, 4.0, (3.25, -1.5), -4096, 4097),
    (2, 6, 37, 72, 2.0, (-0.5, 0.75), -32768, 32768),         # batch 2, ragged tiles, full int16 range
    (1, 4, 40, 64, 40.0, (0.0, 0.0), -32768, 32768),          # wide spread: windows exceed the ring (global gathers)
    (1, 4, 30, 50, 4.0, (3.25, -1.5), -4096, 4097),           # W % 8 != 0: no tensor map (global gathers)
    (1, 3, 24, 64, 4.0, (3.25, -1.5), -4096, 4097),           # odd channel count: no tensor map
    (1, 2, 16, 16, 0.0, (100.0, -100.0), -4096, 4097),        # every sample clamped to the border
])
def test_warp_matches_oracle(ufb, ora, dev, n, c, h, w, sigma, shift, lo, hi):
    """The integer warp equals the fixed-point spec (ufo_warp) exactly; against
    the float semantics of src/dcvc_fm_motion.cu:41-58 it differs by at most
    one Q9 step (reported for config 2)."""
    rng = np.random.default_rng(c * 1000 + h)
    f = rng.integers(lo, hi, (n, c, h, w)).astype(np.int16)
    flow = _config2_flow(rng, n, h, w, sigma, shift)
    got = N(ufb.warp(T(f, dev), T(flow, dev)))
    assert np.array_equal(got, ora.warp(f, flow))
    if (c, h, w) == (64, 176, 320):
        delta = np.abs(got.astype(np.float64) - ora.warp_float(f, flow))
        print(f"config 2: max |integer - float| = {delta.max():.4f} Q9 steps")
        assert delta.max() <= 1.0
    _status_clean(ufb)


def test_errors_are_raised_not_computed(ufb, dev):
    x = torch.zeros((1, 8, 4, 4), dtype=torch.int16, device=dev)
    with pytest.raises(ufb.UfbError):
        ufb.conv2d(x, torch.zeros((8, 3, 1, 1), dtype=torch.int16, device=dev))
    with pytest.raises(ufb.UfbError):
        ufb.add([x])
    with pytest.raises(ufb.UfbError):
        ufb.multiply(x, torch.zeros((1, 3, 1, 1), dtype=torch.int16, device=dev))
