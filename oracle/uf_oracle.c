/* TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference INT16 path.
 *
 * This file is the checker, never the product: only tests/, the smoke check
 * and bench.py's CPU arm load it.  Each function names the reference
 * file:line whose behaviour it restates.  It is pinned against the reference's
 * own known-answer cases (tests/model_free.cpp:570-621 of the reference, turned
 * into tests/golden fixtures) and against the reference CPU path itself
 * compiled from its sources (oracle/_ref, see oracle/Makefile).
 *
 * The integer warp (ufo_warp) has no reference counterpart (the reference's
 * only warp is the float DCVC-FM kernel, src/dcvc_fm_motion.cu:29-76), so its
 * parity is UNPINNED: it restates this repository's own fixed-point spec.
 */
#include "uf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/int16_ops.cpp:48-56 -- round to nearest, ties away from zero:
 * sign(v) * floor((|v| + floor(d/2)) / d) for a positive denominator. */
int64_t ufo_divide_round(int64_t value, int64_t denominator) {
    const int64_t half = denominator / 2;
    if (value < 0) return -((-value + half) / denominator);
    return (value + half) / denominator;
}

/* src/int16_ops.cpp:34-36 */
int16_t ufo_saturate(int64_t value) {
    return (int16_t)(value < -32768 ? -32768 : (value > 32767 ? 32767 : value));
}

/* src/int16_ops.cpp:132-171 (conv2d_reference): exact int64 dot products over
 * zero-padded input, rna(sum / 8192), then + bias (widened to int64), then
 * saturate.  bias_bits: 0 = no bias, 16 = int16 bias, 32 = int32 bias. */
int ufo_conv2d(const int16_t* x, int64_t n, int64_t ci, int64_t h, int64_t w,
               const int16_t* weight, int64_t co, int64_t kh, int64_t kw,
               const void* bias, int bias_bits, int64_t sh, int64_t sw, int64_t ph,
               int64_t pw, int64_t groups, int16_t* out) {
    if (groups <= 0 || ci % groups || co % groups || sh <= 0 || sw <= 0) return -1;
    const int64_t oh = (h + 2 * ph - kh) / sh + 1, ow = (w + 2 * pw - kw) / sw + 1;
    if (oh <= 0 || ow <= 0) return -2;
    const int64_t cig = ci / groups, cog = co / groups;
    for (int64_t b = 0; b < n; ++b) {
        for (int64_t oc = 0; oc < co; ++oc) {
            const int64_t first = (oc / cog) * cig;
            int64_t bias_value = 0;
            if (bias_bits == 16) bias_value = ((const int16_t*)bias)[oc];
            if (bias_bits == 32) bias_value = ((const int32_t*)bias)[oc];
            for (int64_t oy = 0; oy < oh; ++oy) {
                for (int64_t ox = 0; ox < ow; ++ox) {
                    int64_t sum = 0;
                    for (int64_t c = 0; c < cig; ++c) {
                        const int16_t* plane = x + ((b * ci + first + c) * h) * w;
                        const int16_t* taps = weight + ((oc * cig + c) * kh) * kw;
                        for (int64_t ky = 0; ky < kh; ++ky) {
                            const int64_t iy = oy * sh + ky - ph;
                            if (iy < 0 || iy >= h) continue;
                            for (int64_t kx = 0; kx < kw; ++kx) {
                                const int64_t ix = ox * sw + kx - pw;
                                if (ix < 0 || ix >= w) continue;
                                sum += (int64_t)plane[iy * w + ix] * taps[ky * kw + kx];
                            }
                        }
                    }
                    out[((b * co + oc) * oh + oy) * ow + ox] =
                        ufo_saturate(ufo_divide_round(sum, 8192) + bias_value);
                }
            }
        }
    }
    return 0;
}

/* src/int16_ops.cpp:65-75: saturate(sum of int64-widened operands). */
int ufo_add(int count, const int16_t* const* values, int64_t numel, int16_t* out) {
    if (count < 1) return -1;
    for (int64_t i = 0; i < numel; ++i) {
        int64_t sum = 0;
        for (int k = 0; k < count; ++k) sum += values[k][i];
        out[i] = ufo_saturate(sum);
    }
    return 0;
}

/* src/int16_ops.cpp:77-83: saturate(rna(x * scale / 512)) with 4-D broadcast
 * of the scale (every scale extent is 1 or equal to the input's). */
int ufo_multiply(const int16_t* x, const int64_t* xs, const int16_t* scale, const int64_t* ss,
                 int16_t* out) {
    for (int d = 0; d < 4; ++d)
        if (ss[d] != 1 && ss[d] != xs[d]) return -1;
    for (int64_t b = 0; b < xs[0]; ++b)
        for (int64_t c = 0; c < xs[1]; ++c)
            for (int64_t y = 0; y < xs[2]; ++y)
                for (int64_t z = 0; z < xs[3]; ++z) {
                    const int64_t i = ((b * xs[1] + c) * xs[2] + y) * xs[3] + z;
                    const int64_t s = ((((ss[0] == 1 ? 0 : b) * ss[1] + (ss[1] == 1 ? 0 : c)) * ss[2] +
                                        (ss[2] == 1 ? 0 : y)) * ss[3]) + (ss[3] == 1 ? 0 : z);
                    out[i] = ufo_saturate(ufo_divide_round((int64_t)x[i] * scale[s], 512));
                }
    return 0;
}

/* src/int16_ops.cpp:107-115: table[x + 32768]. */
int ufo_lookup_i16(const int16_t* x, int64_t numel, const int16_t* table, int16_t* out) {
    for (int64_t i = 0; i < numel; ++i) out[i] = table[(int32_t)x[i] + 32768];
    return 0;
}

int ufo_lookup_u8(const int16_t* x, int64_t numel, const uint8_t* table, uint8_t* out) {
    for (int64_t i = 0; i < numel; ++i) out[i] = table[(int32_t)x[i] + 32768];
    return 0;
}

/* src/int16_ops.cpp:117-130: out[:, c] = saturate(sum_k lut[x[:, 4c + k]]),
 * k = 0..3 (the CPU path sums the slices x[:, k::4]). */
int ufo_wsilu4(const int16_t* x, int64_t n, int64_t c4, int64_t hw, const int16_t* table,
               int16_t* out) {
    if (c4 % 4) return -1;
    const int64_t c = c4 / 4;
    for (int64_t b = 0; b < n; ++b)
        for (int64_t ch = 0; ch < c; ++ch)
            for (int64_t p = 0; p < hw; ++p) {
                int64_t sum = 0;
                for (int k = 0; k < 4; ++k) sum += table[(int32_t)x[((b * c4) + 4 * ch + k) * hw + p] + 32768];
                out[(b * c + ch) * hw + p] = ufo_saturate(sum);
            }
    return 0;
}

/* src/int16_ops.cpp:99-105: saturate(rna((2v - 255) * 512 / 510)). */
int ufo_from_bytes(const uint8_t* x, int64_t numel, int16_t* out) {
    for (int64_t i = 0; i < numel; ++i)
        out[i] = ufo_saturate(ufo_divide_round((2 * (int64_t)x[i] - 255) * 512, 510));
    return 0;
}

/* src/int16_ops.cpp:91-93: clamp(rna(v / 512), -128, 127) as int8. */
int ufo_symbols(const int16_t* x, int64_t numel, int8_t* out) {
    for (int64_t i = 0; i < numel; ++i) {
        int64_t v = ufo_divide_round(x[i], 512);
        out[i] = (int8_t)(v < -128 ? -128 : (v > 127 ? 127 : v));
    }
    return 0;
}

/* src/int16_ops.cpp:95-97 */
int ufo_from_symbols(const int8_t* x, int64_t numel, int16_t* out) {
    for (int64_t i = 0; i < numel; ++i) out[i] = ufo_saturate((int64_t)x[i] * 512);
    return 0;
}

/* src/int16_ops.cpp:85-89: saturate(rna(512^2 / max(q, 256))). */
int ufo_reciprocal(const int16_t* x, int64_t numel, int16_t* out) {
    for (int64_t i = 0; i < numel; ++i) {
        const int64_t q = x[i] < 256 ? 256 : x[i];
        out[i] = ufo_saturate(ufo_divide_round(512 * 512, q));
    }
    return 0;
}

/* ATen pixel_shuffle / pixel_unshuffle as called by src/layers.cpp:25-33:
 * shuffle   out[c, y*f + i, x*f + j] = in[c*f*f + i*f + j, y, x]
 * unshuffle out[c*f*f + i*f + j, y, x] = in[c, y*f + i, x*f + j]
 * (c, h, w) are the INPUT extents. */
int ufo_pixel_shuffle(const int16_t* x, int64_t n, int64_t c, int64_t h, int64_t w,
                      int64_t f, int unshuffle, int16_t* out) {
    if (!unshuffle) {
        if (c % (f * f)) return -1;
        const int64_t oc = c / (f * f), oh = h * f, ow = w * f;
        for (int64_t b = 0; b < n; ++b)
            for (int64_t ch = 0; ch < c; ++ch) {
                const int64_t o = ch / (f * f), i = (ch / f) % f, j = ch % f;
                for (int64_t y = 0; y < h; ++y)
                    for (int64_t z = 0; z < w; ++z)
                        out[((b * oc + o) * oh + y * f + i) * ow + z * f + j] = x[((b * c + ch) * h + y) * w + z];
            }
    } else {
        if (h % f || w % f) return -1;
        const int64_t oc = c * f * f, oh = h / f, ow = w / f;
        for (int64_t b = 0; b < n; ++b)
            for (int64_t ch = 0; ch < oc; ++ch) {
                const int64_t s = ch / (f * f), i = (ch / f) % f, j = ch % f;
                for (int64_t y = 0; y < oh; ++y)
                    for (int64_t z = 0; z < ow; ++z)
                        out[((b * oc + ch) * oh + y) * ow + z] = x[((b * c + s) * h + y * f + i) * w + z * f + j];
            }
    }
    return 0;
}

/* src/integer_codec.cpp:294-323 (IntegerCodec::raw_frame): frame is a
 * 3 x h x w int16 YUV444 tensor cropped to height x width; output is 8-bit
 * YUV420: Y = clamp(rna((v + 256) * 255 / 512), 0, 255); each chroma sample is
 * clamp(floor((sum of a 2x2 block + 1024) * 255 / 2048), 0, 255). */
int ufo_raw_frame(const int16_t* frame, int64_t h, int64_t w, int64_t height, int64_t width,
                  uint8_t* out) {
    if (height > h || width > w || height % 2 || width % 2) return -1;
    uint8_t* y_out = out;
    for (int64_t y = 0; y < height; ++y)
        for (int64_t x = 0; x < width; ++x) {
            int64_t v = ufo_divide_round(((int64_t)frame[y * w + x] + 256) * 255, 512);
            y_out[y * width + x] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
        }
    uint8_t* uv = out + height * width;
    const int64_t ch = height / 2, cw = width / 2;
    for (int c = 1; c < 3; ++c) {
        const int16_t* plane = frame + (int64_t)c * h * w;
        for (int64_t y = 0; y < ch; ++y)
            for (int64_t x = 0; x < cw; ++x) {
                int64_t s = (int64_t)plane[(2 * y) * w + 2 * x] + plane[(2 * y + 1) * w + 2 * x] +
                            plane[(2 * y) * w + 2 * x + 1] + plane[(2 * y + 1) * w + 2 * x + 1];
                int64_t num = (s + 1024) * 255;
                int64_t v = num >= 0 ? num / 2048 : -((-num + 2047) / 2048); /* floor */
                uv[(c - 1) * ch * cw + y * cw + x] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
            }
    }
    return 0;
}

/* Integer backward bilinear warp (this repository's fixed-point spec; no
 * reference counterpart -- parity UNPINNED).  It mirrors the semantics of the
 * float kernel src/dcvc_fm_motion.cu:41-70: sample position = pixel + flow,
 * clamped to the border; x0 = floor, x1 = min(x0 + 1, W - 1); bilinear weights.
 * Flow is int16 Q9 (1/512 px, channel 0 = x, channel 1 = y).  Weights are the
 * 9-bit fractions, products Q18, result rna(sum / 2^18) saturated to int16. */
int ufo_warp(const int16_t* feature, const int16_t* flow, int64_t n, int64_t c, int64_t h,
             int64_t w, int16_t* out) {
    for (int64_t b = 0; b < n; ++b)
        for (int64_t y = 0; y < h; ++y)
            for (int64_t x = 0; x < w; ++x) {
                const int64_t fx = flow[((b * 2 + 0) * h + y) * w + x];
                const int64_t fy = flow[((b * 2 + 1) * h + y) * w + x];
                int64_t px = x * 512 + fx, py = y * 512 + fy;
                px = px < 0 ? 0 : (px > (w - 1) * 512 ? (w - 1) * 512 : px);
                py = py < 0 ? 0 : (py > (h - 1) * 512 ? (h - 1) * 512 : py);
                const int64_t x0 = px >> 9, y0 = py >> 9;
                const int64_t x1 = x0 + 1 < w ? x0 + 1 : w - 1, y1 = y0 + 1 < h ? y0 + 1 : h - 1;
                const int64_t ax = px & 511, ay = py & 511;
                const int64_t wa = (512 - ax) * (512 - ay), wb = (512 - ax) * ay;
                const int64_t wc = ax * (512 - ay), wd = ax * ay;
                for (int64_t ch = 0; ch < c; ++ch) {
                    const int16_t* p = feature + (b * c + ch) * h * w;
                    const int64_t s = wa * p[y0 * w + x0] + wb * p[y1 * w + x0] + wc * p[y0 * w + x1] +
                                      wd * p[y1 * w + x1];
                    out[((b * c + ch) * h + y) * w + x] = ufo_saturate(ufo_divide_round(s, 1 << 18));
                }
            }
    return 0;
}

/* The float semantics of src/dcvc_fm_motion.cu:41-70 on the same Q9 flow, for
 * the max |delta| report of the integer warp (not a parity target). */
int ufo_warp_float(const int16_t* feature, const int16_t* flow, int64_t n, int64_t c, int64_t h,
                   int64_t w, float* out) {
    for (int64_t b = 0; b < n; ++b)
        for (int64_t y = 0; y < h; ++y)
            for (int64_t x = 0; x < w; ++x) {
                float xp = (float)flow[((b * 2 + 0) * h + y) * w + x] / 512.0f + (float)x;
                float yp = (float)flow[((b * 2 + 1) * h + y) * w + x] / 512.0f + (float)y;
                xp = fminf(fmaxf(xp, 0.f), (float)(w - 1));
                yp = fminf(fmaxf(yp, 0.f), (float)(h - 1));
                const int64_t x0 = (int64_t)floorf(xp), y0 = (int64_t)floorf(yp);
                const int64_t x1 = x0 + 1 < w ? x0 + 1 : w - 1, y1 = y0 + 1 < h ? y0 + 1 : h - 1;
                const float wr = xp - (float)x0, wl = 1.f - wr, wbt = yp - (float)y0, wt = 1.f - wbt;
                const float wa = wl * wt, wb = wl * wbt, wc = wr * wt, wd = wr * wbt;
                for (int64_t ch = 0; ch < c; ++ch) {
                    const int16_t* p = feature + (b * c + ch) * h * w;
                    float r = 0.f;
                    r = fmaf((float)p[y0 * w + x0], wa, r);
                    r = fmaf((float)p[y1 * w + x0], wb, r);
                    r = fmaf((float)p[y0 * w + x1], wc, r);
                    r = fmaf((float)p[y1 * w + x1], wd, r);
                    out[((b * c + ch) * h + y) * w + x] = r;
                }
            }
    return 0;
}
