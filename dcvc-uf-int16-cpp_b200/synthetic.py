"""Seeded synthetic prepared models and inputs (no checkpoints exist offline).

The reference has no random-model generator: its prepared ``.int16.pt`` files
come from real checkpoints.  This module builds prepared-model tensor tables
with exactly the names, shapes and dtypes the reference loader expects
(tensor topology of ``src/model_schema.cpp:77-144``), drawing the integer
parameters from a seeded generator, and building the lookup tables and CDFs
with the formulas of ``src/prepare.cpp:110-267`` (CDFs) and
``src/prepare.cpp:335-349`` (WSiLU and scale-index tables).

Weights are Q13 (``*.weight``), biases and ``q_*`` tables Q9, as produced by
``src/prepare.cpp:327-333``.  Weight magnitudes are variance-preserving
(about 8192 * gain / sqrt(fan_in)) so activations neither vanish nor saturate
through the residual blocks.
"""
from __future__ import annotations

import math
from collections import OrderedDict

import numpy as np

FEATURE_SCALE = 512
WEIGHT_SCALE = 8192


class _Schema:
    """Parameter table following the helper structure of src/model_schema.cpp:15-75."""

    def __init__(self):
        self.shapes: "OrderedDict[str, tuple]" = OrderedDict()

    def parameter(self, name, dims):
        if name in self.shapes:
            raise ValueError(f"duplicate parameter {name}")
        self.shapes[name] = tuple(int(d) for d in dims)

    def conv(self, name, cin, cout, kernel=1, bias=True, groups=1):
        self.parameter(name + ".weight", (cout, cin // groups, kernel, kernel))
        if bias:
            self.parameter(name + ".bias", (cout,))

    def depth(self, name, cin, cout, dcb2=False, force_adaptor=False):
        hidden = cout // (2 if dcb2 else 1)
        if cin != cout or force_adaptor:
            self.conv(name + ".adaptor", cin, cout)
        self.conv(name + ".dc.0", cout, hidden)
        self.conv(name + ".dc.2", hidden, hidden, 3, True, hidden)
        self.conv(name + ".dc.3", hidden, cout)
        self.conv(name + ".ffn.0", cout, hidden * 4)
        self.conv(name + ".ffn.2", hidden, cout)

    def depths(self, name, count, cin, cout, dcb2=False):
        for i in range(count):
            self.depth(f"{name}.{i}", cout if i else cin, cout, dcb2)

    def subpel(self, name, cin, cout, kernel=1, force_bias=False):
        self.conv(name + ".conv.0", cin, cout * 4, kernel, kernel > 1 or force_bias)

    def up(self, name, cin, cout, dcb2=False, force_bias=False):
        self.subpel(name + ".up", cin, cout, 1, force_bias)
        self.depth(name + ".conv", cout, cout, dcb2)

    def down(self, name, cin, cout, dcb2=False):
        self.conv(name + ".down", cin * 4, cout)
        self.depth(name + ".conv", cout, cout, dcb2)

    def prior(self, name, cin, hidden, cout, blocks, dcb2=False):
        self.depths(name, blocks, cin, hidden, dcb2)
        self.conv(f"{name}.{blocks}", hidden, cout)

    def entropy(self):
        self.parameter("bit_estimator_z.h", (64, 128, 4))
        self.parameter("bit_estimator_z.b", (64, 128, 4))
        self.parameter("bit_estimator_z.a", (64, 128, 3))


def image_schema() -> _Schema:
    """Image (I-frame) model topology: src/model_schema.cpp:77-103."""
    s = _Schema()
    s.entropy()
    s.depth("enc.enc_1", 192, 384)
    s.depths("enc.enc_2", 6, 384, 384)
    s.conv("enc.enc_2.6", 384, 256, 3)
    s.depth("hyper_enc.conv.0", 256, 128)
    s.down("hyper_enc.conv.1", 128, 128)
    s.down("hyper_enc.conv.2", 128, 128)
    s.up("hyper_dec.conv.0", 128, 128)
    s.up("hyper_dec.conv.1", 128, 128)
    s.depth("hyper_dec.conv.2", 128, 256)
    s.prior("y_prior_fusion.conv", 256, 512, 512, 3)
    s.conv("y_spatial_prior_reduction", 512, 256)
    for i in range(1, 4):
        s.depth(f"y_spatial_prior_adaptor_{i}", 512, 512, False, True)
    s.prior("y_spatial_prior.conv", 512, 512, 512, 3)
    s.up("dec.dec_1.0", 256, 384)
    for i in range(1, 13):
        s.depth(f"dec.dec_1.{i}", 384, 384)
    s.depth("dec.dec_2", 384, 192)
    s.parameter("q_scale_enc", (64, 384))
    s.parameter("q_scale_dec", (64, 384))
    s.parameter("q_scale_y_enc", (64, 256))
    s.parameter("q_scale_y_dec", (64, 256))
    return s


def htl_schema() -> _Schema:
    """HT-L video model topology: src/model_schema.cpp:105-144 with hts = false."""
    s = _Schema()
    s.entropy()
    s.depths("feature_adaptor_i.conv", 3, 192, 512)
    s.depths("feature_adaptor_m.conv", 10, 1024, 512)
    s.depths("feature_extractor.conv", 2, 512, 512)
    s.depths("encoder.conv1", 7, 2048, 512)
    s.conv("encoder.down", 512, 256, 3)
    s.depth("hyper_encoder.conv.0", 256, 256)
    s.down("hyper_encoder.conv.1", 256, 256)
    s.down("hyper_encoder.conv.2", 256, 128)
    s.up("hyper_decoder.conv.0", 128, 256, False, True)
    s.up("hyper_decoder.conv.1", 256, 256, False, True)
    s.depth("hyper_decoder.conv.2", 256, 256)
    s.down("temporal_prior_encoder.conv", 512, 512)
    s.prior("y_prior_fusion.conv", 768, 768, 768, 3)
    s.conv("y_spatial_prior_reduction", 768, 256)
    for i in range(1, 4):
        s.depth(f"y_spatial_prior_adaptor_{i}", 512, 512, False, True)
    s.prior("y_spatial_prior.conv", 512, 512, 512, 3)
    s.subpel("decoder.up", 256, 512, 3, True)
    s.depths("decoder.conv1", 11, 1024, 512)
    for i in range(8):
        s.prior(f"recon_head.conv.{i}", 512, 256, 192, 5)
    s.parameter("q_encoder", (64, 512))
    s.parameter("q_decoder", (64, 512))
    s.parameter("q_feature", (64, 512))
    return s


# ---------------------------------------------------------------- tables ----

def wsilu_table() -> np.ndarray:
    """src/prepare.cpp:335-338: quantize(v * sigmoid(4 v), 512), v = i / 512."""
    v = np.arange(-32768, 32768, dtype=np.float64) / FEATURE_SCALE
    y = v / (1.0 + np.exp(-4.0 * v))
    return np.clip(np.round(y * FEATURE_SCALE), -32768, 32767).astype(np.int16)


def scale_index_table() -> np.ndarray:
    """src/prepare.cpp:339-345: floor((log(clamp(v, .11, 16)) - log .11) * 127 / (log 16 - log .11))."""
    v = np.arange(-32768, 32768, dtype=np.float64) / FEATURE_SCALE
    s = np.clip(v, 0.11, 16.0)
    lo, hi = math.log(0.11), math.log(16.0)
    idx = np.floor((np.log(s) - lo) * (127.0 / (hi - lo)))
    return np.clip(idx, 0, 127).astype(np.uint8)


def _quantized_cdf(pmf: np.ndarray) -> list:
    """src/prepare.cpp:110-151: 16-bit CDF with zero-frequency repair."""
    maximum = 1 << 16
    cdf = [0] * (len(pmf) + 1)
    for i, p in enumerate(pmf):
        cdf[i + 1] = int(np.float32(p) * np.float32(maximum) + 0.5)
    total = sum(cdf)
    if not total:
        raise ValueError("empty pmf")
    cdf = [maximum * v // total for v in cdf]
    for i in range(1, len(cdf)):
        cdf[i] += cdf[i - 1]
    cdf[-1] = maximum
    for i in range(len(cdf) - 1):
        if cdf[i] + 1 <= cdf[i + 1]:
            continue
        best, donor = None, None
        for j in range(len(cdf) - 1):
            f = cdf[j + 1] - cdf[j]
            if f >= 2 and (best is None or f < best):
                donor, best = j, f
        if donor is None or donor == i:
            raise ValueError("CDF repair failed")
        if donor < i:
            for j in range(donor + 1, i + 1):
                cdf[j] -= 1
        else:
            for j in range(i + 1, donor + 1):
                cdf[j] += 1
    return cdf


def _make_cdf(pmf: np.ndarray, tail: np.ndarray, lengths: np.ndarray):
    """src/prepare.cpp:153-191: reorder (centre, +1, -1, +2, -2, ..., tail)."""
    rows, max_length = pmf.shape
    width = max_length + 2
    cdf = np.zeros((rows, width), np.int32)
    out_len = np.zeros(rows, np.int32)
    for r in range(rows):
        length = int(lengths[r])
        center = length // 2
        re = np.zeros(length + 1, np.float32)
        re[0] = pmf[r, center]
        for i in range(1, center + 1):
            re[2 * i - 1] = pmf[r, center + i]
            re[2 * i] = pmf[r, center - i]
        re[length] = tail[r]
        vals = _quantized_cdf(re)
        cdf[r, : len(vals)] = vals
        out_len[r] = length + 2
    return cdf, out_len


def _erf(x):
    from scipy.special import erf
    return erf(x)


def _normal_cdf(x, scale):
    return 0.5 * (1.0 + _erf(x / scale / math.sqrt(2.0)))


def gaussian_cdf():
    """src/prepare.cpp:200-223: 128 Gaussian rows, scales exp(linspace(log .11, log 16))."""
    levels, maximum = 128, 8
    scales = np.exp(np.linspace(math.log(0.11), math.log(16.0), levels)).astype(np.float32)
    rng_ = np.full(levels, maximum, np.int32)
    for i in range(maximum, 1, -1):
        rng_ = np.where(_normal_cdf(np.float32(i), scales) > 0.999, i, rng_)
    lengths = 2 * rng_ + 1
    samples = (np.arange(2 * maximum + 1)[None, :] - rng_[:, None]).astype(np.float32)
    sc = scales[:, None]
    upper = _normal_cdf(samples + 0.5, sc).astype(np.float32)
    lower = _normal_cdf(samples - 0.5, sc).astype(np.float32)
    return _make_cdf(upper - lower, 2 * lower[:, 0], lengths)


def _softplus(x):
    return np.log1p(np.exp(-np.abs(x))) + np.maximum(x, 0)


def _bit_forward(x, h, b, a):
    """src/prepare.cpp:225-239 (factorized bit estimator)."""
    for i in range(4):
        x = x * _softplus(h[..., i])[..., None] + b[..., i][..., None]
        if i != 3:
            x = x + np.tanh(x) * np.tanh(a[..., i])[..., None]
    return 1.0 / (1.0 + np.exp(-x))


def bit_estimator_cdf(h, b, a):
    """src/prepare.cpp:241-267: 64 x 128 rows (qp-major), range search to 8."""
    maximum = 8
    zeros = np.zeros((64, 128, 1), np.float32)
    rng_ = zeros + maximum
    for i in range(maximum, 1, -1):
        neg = _bit_forward(zeros - i, h, b, a)
        pos = _bit_forward(zeros + i, h, b, a)
        rng_ = np.where(np.logical_and(neg < 0.001, pos > 0.999), i, rng_)
    rng_ = rng_.astype(np.int32)
    lengths = (rng_ * 2 + 1).reshape(-1)
    samples = (np.arange(2 * maximum + 1)[None, None, :] - rng_).astype(np.float32)
    lower = _bit_forward(samples - 0.5, h, b, a)
    upper = _bit_forward(samples + 0.5, h, b, a)
    pmf = (upper - lower).reshape(-1, 2 * maximum + 1).astype(np.float32)
    tail = (lower[..., :1] + (1.0 - _bit_forward(rng_.astype(np.float32), h, b, a))).reshape(-1)
    return _make_cdf(pmf, tail.astype(np.float32), lengths)


# ---------------------------------------------------------------- models ----

def _fan_in(shape):
    return int(np.prod(shape[1:]))


def make_prepared(variant: str, seed: int, gain: float = 0.55) -> dict:
    """Seeded prepared-model tensor table {name: ndarray} for 'htl' or 'image'."""
    schema = htl_schema() if variant == "htl" else image_schema() if variant == "image" else None
    if schema is None:
        raise ValueError(f"unsupported variant {variant}")
    rng = np.random.default_rng(seed)
    tensors = {}
    for name, shape in schema.shapes.items():
        if name.endswith(".weight"):
            fan = _fan_in(shape)
            std = WEIGHT_SCALE * gain / math.sqrt(fan)
            tensors[name] = np.clip(np.round(rng.normal(0.0, std, shape)), -32768, 32767).astype(np.int16)
        elif name.endswith(".bias"):
            tensors[name] = np.clip(np.round(rng.normal(0.0, 0.05 * FEATURE_SCALE, shape)),
                                    -32768, 32767).astype(np.int16)
        elif name.startswith("q_"):
            # per-qp scales near unit (Q9 512), finer quantisation at low qp
            qp = np.arange(64, dtype=np.float64)[:, None]
            base = 0.6 + 0.9 * qp / 63.0
            if "dec" in name or name == "q_feature" or name == "q_scale_y_dec":
                val = base
            else:
                val = 1.0 / base
            noise = rng.uniform(0.9, 1.1, shape)
            tensors[name] = np.clip(np.round(val * noise * FEATURE_SCALE), 1, 32767).astype(np.int16)
    h = rng.normal(0.0, 0.6, (64, 128, 4)).astype(np.float32)
    b = rng.normal(0.0, 0.6, (64, 128, 4)).astype(np.float32)
    a = rng.normal(0.0, 0.6, (64, 128, 3)).astype(np.float32)
    tensors["tables.wsilu"] = wsilu_table()
    tensors["tables.scale_index"] = scale_index_table()
    zc, zl = bit_estimator_cdf(h, b, a)
    yc, yl = gaussian_cdf()
    tensors["tables.z_cdf"], tensors["tables.z_lengths"] = zc, zl
    tensors["tables.y_cdf"], tensors["tables.y_lengths"] = yc, yl
    return tensors


_CACHE: dict = {}


def prepared(variant: str, seed: int) -> dict:
    key = (variant, seed)
    if key not in _CACHE:
        _CACHE[key] = make_prepared(variant, seed)
    return _CACHE[key]


# ---------------------------------------------------------------- inputs ----

def synthetic_video(width: int, height: int, frames: int, seed: int) -> np.ndarray:
    """YUV444 8-bit frames [frames, 3, height, width]: smooth gradient background,
    six textured rectangles moving at constant velocities of 0-4 px/frame, and
    N(0, 2^2) noise.  Stands in for the reference's FFmpeg testsrc2 clip."""
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:height, 0:width].astype(np.float64)
    base = np.stack([60 + 120 * xx / max(width - 1, 1) + 30 * yy / max(height - 1, 1),
                     128 + 40 * np.sin(xx / 37.0),
                     128 + 40 * np.cos(yy / 29.0)])
    rects = []
    for _ in range(6):
        rw, rh = rng.integers(width // 10 + 4, width // 4 + 8), rng.integers(height // 10 + 4, height // 4 + 8)
        x0, y0 = rng.uniform(0, width - rw), rng.uniform(0, height - rh)
        speed, ang = rng.uniform(0, 4), rng.uniform(0, 2 * math.pi)
        color = rng.uniform(20, 235, 3)
        freq = rng.uniform(0.2, 0.8)
        rects.append((rw, rh, x0, y0, speed * math.cos(ang), speed * math.sin(ang), color, freq))
    out = np.empty((frames, 3, height, width), np.uint8)
    for f in range(frames):
        img = base.copy()
        for rw, rh, x0, y0, vx, vy, color, freq in rects:
            cx, cy = int(round(x0 + vx * f)) % width, int(round(y0 + vy * f)) % height
            ys, xs = slice(cy, min(cy + rh, height)), slice(cx, min(cx + rw, width))
            tex = 25 * np.sin(freq * (xx[ys, xs] + yy[ys, xs]))
            for c in range(3):
                img[c, ys, xs] = color[c] + (tex if c == 0 else 0.3 * tex)
        img += rng.normal(0, 2.0, img.shape)
        out[f] = np.clip(np.round(img), 0, 255).astype(np.uint8)
    return out


def frames_to_chunk(frames_u8: np.ndarray) -> np.ndarray:
    """[F, 3, H, W] uint8 -> [1, 3F, H, W] uint8 (channel order frame-major, as
    src/integer_codec.cpp:183-213 concatenates each frame's 3 planes)."""
    f, c, h, w = frames_u8.shape
    return np.ascontiguousarray(frames_u8.reshape(1, f * c, h, w))


def synthetic_video_gpu(width: int, height: int, frames: int, seed: int, device="cuda"):
    """The synthetic_video scene (same background, six moving textured
    rectangles, N(0, 2^2) noise) generated with torch on a GPU for the
    large benchmark workloads.  Rectangle parameters come from the same numpy
    generator; the noise comes from a torch generator seeded with `seed`, so
    the pixels differ from synthetic_video() but are equally reproducible.
    Returns uint8 [frames, 3, height, width] on `device`."""
    import torch
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    yy, xx = torch.meshgrid(torch.arange(height, device=device, dtype=torch.float32),
                            torch.arange(width, device=device, dtype=torch.float32), indexing="ij")
    base = torch.stack([60 + 120 * xx / max(width - 1, 1) + 30 * yy / max(height - 1, 1),
                        128 + 40 * torch.sin(xx / 37.0), 128 + 40 * torch.cos(yy / 29.0)])
    rects = []
    for _ in range(6):
        rw, rh = int(rng.integers(width // 10 + 4, width // 4 + 8)), int(rng.integers(height // 10 + 4, height // 4 + 8))
        x0, y0 = rng.uniform(0, width - rw), rng.uniform(0, height - rh)
        speed, ang = rng.uniform(0, 4), rng.uniform(0, 2 * math.pi)
        color = rng.uniform(20, 235, 3)
        freq = rng.uniform(0.2, 0.8)
        rects.append((rw, rh, x0, y0, speed * math.cos(ang), speed * math.sin(ang), color, freq))
    out = torch.empty((frames, 3, height, width), dtype=torch.uint8, device=device)
    for f in range(frames):
        img = base.clone()
        for rw, rh, x0, y0, vx, vy, color, freq in rects:
            cx, cy = int(round(x0 + vx * f)) % width, int(round(y0 + vy * f)) % height
            ys, xs = slice(cy, min(cy + rh, height)), slice(cx, min(cx + rw, width))
            tex = 25 * torch.sin(freq * (xx[ys, xs] + yy[ys, xs]))
            for c in range(3):
                img[c, ys, xs] = float(color[c]) + (tex if c == 0 else 0.3 * tex)
        img += torch.randn(img.shape, generator=gen, device=device) * 2.0
        out[f] = img.round().clamp(0, 255).to(torch.uint8)
    return out
