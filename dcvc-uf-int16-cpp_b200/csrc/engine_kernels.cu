// Model-level memory-bound kernels on split-NHWC views: channel copies (cat),
// symbol <-> feature conversions, multiply / unshuffle fusions, the
// entropy-parameter kernels of IntegerModel::prior, and raw-frame output.
#include "engine_kernels.h"
#include "uf_common.cuh"

namespace ufb {

namespace {

constexpr int kBlock = 256;

unsigned grid_for(long long n) {
    const long long b = (n + kBlock - 1) / kBlock;
    const long long cap = 148ll * 32;
    return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

#define GRID_LOOP(i, total) \
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < (total); \
         i += static_cast<long long>(gridDim.x) * blockDim.x)

__device__ __forceinline__ void px_of(const Act& a, long long p, int& b, int& y, int& x) {
    x = static_cast<int>(p % a.w);
    p /= a.w;
    y = static_cast<int>(p % a.h);
    b = static_cast<int>(p / a.h);
}

// dst[:, :, :, 0:c] = src (same n, h, w); 16 channels per thread.
__global__ void copy_channels_kernel(Act src, Act dst) {
    const int groups = (src.c + 15) / 16;
    GRID_LOOP(i, src.pixels() * groups) {
        const int g = static_cast<int>(i % groups);
        int b, y, x;
        px_of(src, i / groups, b, y, x);
        const long long sp = src.pixel(b, y, x), dp = dst.pixel(b, y, x);
        const int c0 = g * 16;
        if (c0 + 16 <= src.c) {
            *reinterpret_cast<uint4*>(dst.lo(dp) + c0) = *reinterpret_cast<const uint4*>(src.lo(sp) + c0);
            *reinterpret_cast<uint4*>(dst.hi(dp) + c0) = *reinterpret_cast<const uint4*>(src.hi(sp) + c0);
        } else {
            for (int c = c0; c < src.c; ++c) {
                dst.lo(dp)[c] = src.lo(sp)[c];
                dst.hi(dp)[c] = src.hi(sp)[c];
            }
        }
    }
}

__global__ void fill_zero_kernel(Act dst) {
    const int groups = (dst.c + 15) / 16;
    GRID_LOOP(i, dst.pixels() * groups) {
        const int g = static_cast<int>(i % groups);
        int b, y, x;
        px_of(dst, i / groups, b, y, x);
        const long long dp = dst.pixel(b, y, x);
        for (int c = g * 16; c < dst.c && c < g * 16 + 16; ++c) {
            dst.lo(dp)[c] = 0;
            dst.hi(dp)[c] = 0;
        }
    }
}

// int16::from_symbols (src/int16_ops.cpp:95-97) of NHWC int8 symbols.
__global__ void symbols_to_split_kernel(const int8_t* __restrict__ s, Act out) {
    GRID_LOOP(i, out.pixels() * out.c) {
        const int c = static_cast<int>(i % out.c);
        int b, y, x;
        px_of(out, i / out.c, b, y, x);
        const int16_t v = sat16i(static_cast<int32_t>(s[i]) * kFeatureScale);
        const long long p = out.pixel(b, y, x);
        out.lo(p)[c] = static_cast<uint8_t>(v & 0xff);
        out.hi(p)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// int16::symbols (src/int16_ops.cpp:91-93) into NHWC int8: clamp(rna(v/512)).
__global__ void split_to_symbols_kernel(Act in, int8_t* __restrict__ s) {
    GRID_LOOP(i, in.pixels() * in.c) {
        const int c = static_cast<int>(i % in.c);
        int b, y, x;
        px_of(in, i / in.c, b, y, x);
        const long long p = in.pixel(b, y, x);
        int64_t v = rna_div(join16(in.lo(p)[c], in.hi(p)[c]), kFeatureScale);
        s[i] = static_cast<int8_t>(v < -128 ? -128 : (v > 127 ? 127 : v));
    }
}

// out = pixel_unshuffle(multiply(in, q), 2): out channel 4c + 2i + j of
// pixel (y, x) = sat(rna(in[(2y + i, 2x + j), c] * q[c] / 512)); q may be null.
__global__ void mul_unshuffle2_kernel(Act in, const int16_t* __restrict__ q, Act out) {
    GRID_LOOP(i, in.pixels() * in.c) {
        const int c = static_cast<int>(i % in.c);
        int b, y, x;
        px_of(in, i / in.c, b, y, x);
        const long long p = in.pixel(b, y, x);
        int16_t v = join16(in.lo(p)[c], in.hi(p)[c]);
        if (q) v = sat16(rna_shift(static_cast<int64_t>(v) * q[c], 9));
        const long long op = out.pixel(b, y >> 1, x >> 1);
        const int oc = c * 4 + (y & 1) * 2 + (x & 1);
        out.lo(op)[oc] = static_cast<uint8_t>(v & 0xff);
        out.hi(op)[oc] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// out = sat(rna(in * q / 512)); q per channel (q_img_stride == 0) or a view.
__global__ void mul_channels_kernel(Act in, const int16_t* __restrict__ q, Act out) {
    GRID_LOOP(i, in.pixels() * in.c) {
        const int c = static_cast<int>(i % in.c);
        int b, y, x;
        px_of(in, i / in.c, b, y, x);
        const long long p = in.pixel(b, y, x), op = out.pixel(b, y, x);
        const int16_t v = sat16(rna_shift(static_cast<int64_t>(join16(in.lo(p)[c], in.hi(p)[c])) * q[c], 9));
        out.lo(op)[c] = static_cast<uint8_t>(v & 0xff);
        out.hi(op)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// out = lut[in] (groups == 1) or out[c] = sat(sum_{k<4} lut[in[4c + k]])
// (groups == 4): int16::lookup / int16::wsilu4 (src/int16_ops.cpp:107-130) on
// split views, for tables the convolution epilogue cannot window.
__global__ void lut_split_kernel(Act in, const int16_t* __restrict__ lut, int groups, Act out) {
    GRID_LOOP(i, out.pixels() * out.c) {
        const int c = static_cast<int>(i % out.c);
        int b, y, x;
        px_of(out, i / out.c, b, y, x);
        const long long p = in.pixel(b, y, x), op = out.pixel(b, y, x);
        int32_t v = 0;
        for (int k = 0; k < groups; ++k) {
            const int ic = c * groups + k;
            v += lut[join16(in.lo(p)[ic], in.hi(p)[ic]) + 32768];
        }
        const int16_t r = sat16(v);
        out.lo(op)[c] = static_cast<uint8_t>(r & 0xff);
        out.hi(op)[c] = static_cast<uint8_t>((r >> 8) & 0xff);
    }
}

// IntegerModel::prior tail (src/integer_model.cpp:209-210, 292):
// out = multiply(restored, max(q_raw, 256)) elementwise.
__global__ void yhat_kernel(Act restored, Act qraw, Act out) {
    GRID_LOOP(i, restored.pixels() * restored.c) {
        const int c = static_cast<int>(i % restored.c);
        int b, y, x;
        px_of(restored, i / restored.c, b, y, x);
        const long long p = restored.pixel(b, y, x), qp = qraw.pixel(b, y, x), op = out.pixel(b, y, x);
        int32_t q = join16(qraw.lo(qp)[c], qraw.hi(qp)[c]);
        q = q < kFeatureScale / 2 ? kFeatureScale / 2 : q;
        const int16_t v =
            sat16(rna_shift(static_cast<int64_t>(join16(restored.lo(p)[c], restored.hi(p)[c])) * q, 9));
        out.lo(op)[c] = static_cast<uint8_t>(v & 0xff);
        out.hi(op)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// ---- entropy-parameter kernels (src/integer_model.cpp:136-293) ----
//
// Positions of part p: every (c, y, x) of one stream, in NCHW order, whose
// micro position (y & 1) * 2 + (x & 1) equals four[p][c / (C / 4)] with
// four = {{0,1,2,3},{3,2,1,0},{2,3,0,1},{1,0,3,2}} (src/integer_model.cpp:146-168).
// A position is active when skip_thr == 0 or its scale > skip_thr.
// Each CTA owns kChunk consecutive NCHW positions of one stream; the count /
// scan / emit passes recompute the same flags, so ranks agree everywhere.

constexpr int kChunk = 4096;           // positions per CTA
constexpr int kPriorThreads = 256;     // 16 positions per thread

__device__ __forceinline__ int part_of(int c, int channels, int y, int x) {
    const int group = c / (channels / 4);
    const int micro = (y & 1) * 2 + (x & 1);
    // inverse of four[p][group] == micro
    const int inv[4][4] = {{0, 3, 2, 1}, {3, 0, 1, 2}, {2, 1, 0, 3}, {1, 2, 3, 0}};
    return inv[group][micro];
}

struct PriorGeom {
    int channels, h, w;   // per stream NCHW extents
    long long elems;      // channels * h * w
};

__device__ __forceinline__ bool prior_flag(const PriorGeom& g, int b, long long e, int part, const Act& scales,
                                           int thr, int16_t& scale_out, int& c_out, int& y_out, int& x_out) {
    const int x = static_cast<int>(e % g.w);
    const int y = static_cast<int>((e / g.w) % g.h);
    const int c = static_cast<int>(e / (static_cast<long long>(g.w) * g.h));
    c_out = c;
    y_out = y;
    x_out = x;
    if (part_of(c, g.channels, y, x) != part) return false;
    const long long p = scales.pixel(b, y, x);
    const int16_t s = join16(scales.lo(p)[c], scales.hi(p)[c]);
    scale_out = s;
    return thr == 0 || s > thr;
}

// Block-wide exclusive scan of one count per thread; returns the prefix and
// writes the block total.
__device__ __forceinline__ int block_scan(int v, int* total) {
    __shared__ int warp_sums[kPriorThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int s = lane < kPriorThreads / 32 ? warp_sums[lane] : 0;
        int si = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, si, o);
            if (lane >= o) si += n;
        }
        if (lane < kPriorThreads / 32) warp_sums[lane] = si - s;
        if (lane == kPriorThreads / 32 - 1) *total = si;
    }
    __syncthreads();
    const int r = warp_sums[warp] + incl - v;
    __syncthreads();
    return r;
}

__global__ void prior_count_kernel(PriorGeom g, int part, Act scales, int thr, int* __restrict__ block_counts,
                                   int blocks_per_stream) {
    const int b = blockIdx.y, blk = blockIdx.x;
    const long long base = static_cast<long long>(blk) * kChunk;
    int count = 0;
    for (int k = threadIdx.x; k < kChunk; k += kPriorThreads) {
        const long long e = base + k;
        if (e >= g.elems) break;
        int16_t s;
        int c, y, x;
        count += prior_flag(g, b, e, part, scales, thr, s, c, y, x) ? 1 : 0;
    }
    __shared__ int total;
    // reduce via the scan helper
    block_scan(count, &total);
    if (threadIdx.x == 0) block_counts[b * blocks_per_stream + blk] = total;
}

// One CTA per stream: exclusive scan of its block counts, stream total.
__global__ void prior_scan_kernel(int* __restrict__ block_counts, int blocks_per_stream, int* __restrict__ totals) {
    const int b = blockIdx.x;
    int* bc = block_counts + static_cast<long long>(b) * blocks_per_stream;
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < blocks_per_stream; base += kPriorThreads) {
        const int i = base + threadIdx.x;
        const int v = i < blocks_per_stream ? bc[i] : 0;
        __shared__ int total;
        const int ex = block_scan(v, &total);
        if (i < blocks_per_stream) bc[i] = carry + ex;
        __syncthreads();
        if (threadIdx.x == 0) carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) totals[b] = carry;
}

// Visits the active positions of a CTA's chunk in order; fn(rank, c, y, x, scale).
template <class Fn>
__device__ __forceinline__ void prior_visit(const PriorGeom& g, int part, const Act& scales, int thr, int b,
                                            long long base, int block_offset, Fn fn) {
    // each thread takes 16 consecutive positions so per-thread ranks are local
    constexpr int kPer = kChunk / kPriorThreads;
    const long long first = base + static_cast<long long>(threadIdx.x) * kPer;
    uint32_t mask = 0;
    int16_t sc[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const long long e = first + k;
        int c, y, x;
        sc[k] = 0;
        if (e < g.elems && prior_flag(g, b, e, part, scales, thr, sc[k], c, y, x)) mask |= 1u << k;
    }
    __shared__ int total;
    int rank = block_offset + block_scan(__popc(mask), &total);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const long long e = first + k;
        if (e >= g.elems) break;
        const int x = static_cast<int>(e % g.w);
        const int y = static_cast<int>((e / g.w) % g.h);
        const int c = static_cast<int>(e / (static_cast<long long>(g.w) * g.h));
        const bool in_part = part_of(c, g.channels, y, x) == part;
        const bool active = (mask >> k) & 1u;
        fn(in_part, active, active ? rank : -1, c, y, x, sc[k]);
        if (active) ++rank;
    }
}

// Decode pass 1: indexes[stream * cap + rank] = scale_index[scale] (u8).
__global__ void prior_indexes_kernel(PriorGeom g, int part, Act scales, int thr, const int* __restrict__ offsets,
                                     int blocks_per_stream, const uint8_t* __restrict__ scale_index,
                                     uint8_t* __restrict__ indexes, long long cap) {
    const int b = blockIdx.y, blk = blockIdx.x;
    const long long base = static_cast<long long>(blk) * kChunk;
    uint8_t* out = indexes + b * cap;
    prior_visit(g, part, scales, thr, b, base, offsets[b * blocks_per_stream + blk],
                [&](bool, bool active, int rank, int, int, int, int16_t s) {
                    if (active) out[rank] = scale_index[static_cast<int32_t>(s) + 32768];
                });
}

// Decode pass 2: restored[pos] = sat(sym * 512 + mean) for every position of
// the part (inactive positions take symbol 0).
__global__ void prior_restore_kernel(PriorGeom g, int part, Act scales, Act means, int thr,
                                     const int* __restrict__ offsets, int blocks_per_stream,
                                     const int8_t* __restrict__ symbols, long long cap, Act restored) {
    const int b = blockIdx.y, blk = blockIdx.x;
    const long long base = static_cast<long long>(blk) * kChunk;
    const int8_t* sy = symbols + b * cap;
    prior_visit(g, part, scales, thr, b, base, offsets[b * blocks_per_stream + blk],
                [&](bool in_part, bool active, int rank, int c, int y, int x, int16_t) {
                    if (!in_part) return;
                    const long long mp = means.pixel(b, y, x);
                    const int32_t mean = join16(means.lo(mp)[c], means.hi(mp)[c]);
                    const int32_t sym = active ? sy[rank] : 0;
                    const int16_t v = sat16i(sym * kFeatureScale + mean);
                    const long long rp = restored.pixel(b, y, x);
                    restored.lo(rp)[c] = static_cast<uint8_t>(v & 0xff);
                    restored.hi(rp)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
                });
}

// Encode: symbols of active positions, packed (sym << 8 | index) for rANS,
// and the restored value (src/integer_model.cpp:250-256, 277-290).
__global__ void prior_encode_kernel(PriorGeom g, int part, Act scales, Act means, Act yenc, int thr,
                                    const int* __restrict__ offsets, int blocks_per_stream,
                                    const uint8_t* __restrict__ scale_index, int16_t* __restrict__ packed,
                                    long long cap, Act restored) {
    const int b = blockIdx.y, blk = blockIdx.x;
    const long long base = static_cast<long long>(blk) * kChunk;
    int16_t* pk = packed + b * cap;
    prior_visit(g, part, scales, thr, b, base, offsets[b * blocks_per_stream + blk],
                [&](bool in_part, bool active, int rank, int c, int y, int x, int16_t s) {
                    if (!in_part) return;
                    const long long mp = means.pixel(b, y, x);
                    const int32_t mean = join16(means.lo(mp)[c], means.hi(mp)[c]);
                    int32_t sym = 0;
                    if (active) {
                        const long long yp = yenc.pixel(b, y, x);
                        const int64_t resid = static_cast<int64_t>(join16(yenc.lo(yp)[c], yenc.hi(yp)[c])) - mean;
                        int64_t q = rna_div(resid, kFeatureScale);
                        q = q < -128 ? -128 : (q > 127 ? 127 : q);
                        sym = static_cast<int32_t>(q);
                        const int idx = scale_index[static_cast<int32_t>(s) + 32768];
                        pk[rank] = static_cast<int16_t>(sym * 256 + idx);
                    }
                    const int16_t v = sat16i(sym * kFeatureScale + mean);
                    const long long rp = restored.pixel(b, y, x);
                    restored.lo(rp)[c] = static_cast<uint8_t>(v & 0xff);
                    restored.hi(rp)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
                });
}

// IntegerCodec::raw_frame (src/integer_codec.cpp:294-323) on the shuffle(8)
// layout of a recon head output: full-resolution pixel (Y, X) of component k
// is channel k * 64 + (Y % 8) * 8 + X % 8 of head pixel (Y / 8, X / 8).
__global__ void raw_frame_kernel(Act head, int height, int width, uint8_t* __restrict__ out, long long frame_bytes) {
    const long long luma = static_cast<long long>(height) * width;
    const int ch = height / 2, cw = width / 2;
    const long long chroma = static_cast<long long>(ch) * cw;
    const long long per_img = luma + 2 * chroma;
    GRID_LOOP(i, head.n * per_img) {
        const int b = static_cast<int>(i / per_img);
        long long r = i - static_cast<long long>(b) * per_img;
        uint8_t* o = out + b * frame_bytes;
        auto sample = [&](int comp, int Y, int X) -> int32_t {
            const long long p = head.pixel(b, Y >> 3, X >> 3);
            const int c = comp * 64 + (Y & 7) * 8 + (X & 7);
            return join16(head.lo(p)[c], head.hi(p)[c]);
        };
        if (r < luma) {
            const int Y = static_cast<int>(r / width), X = static_cast<int>(r % width);
            int64_t v = rna_div((static_cast<int64_t>(sample(0, Y, X)) + kFeatureScale / 2) * 255, kFeatureScale);
            o[r] = static_cast<uint8_t>(v < 0 ? 0 : (v > 255 ? 255 : v));
        } else {
            r -= luma;
            const int comp = 1 + static_cast<int>(r / chroma);
            const long long q = r % chroma;
            const int y = static_cast<int>(q / cw), x = static_cast<int>(q % cw);
            const int64_t s = sample(comp, 2 * y, 2 * x) + sample(comp, 2 * y + 1, 2 * x) +
                              sample(comp, 2 * y, 2 * x + 1) + sample(comp, 2 * y + 1, 2 * x + 1);
            const int64_t num = (s + 2 * kFeatureScale) * 255;
            int64_t v = num >= 0 ? num / (4 * kFeatureScale) : -((-num + 4 * kFeatureScale - 1) / (4 * kFeatureScale));
            o[luma + r] = static_cast<uint8_t>(v < 0 ? 0 : (v > 255 ? 255 : v));
        }
    }
}

// uint8 YUV444 frames [n][3F][H][W] -> int16 (from_bytes) split view with
// pixel_unshuffle(f) (the encoder's input unshuffle; f = 1 keeps resolution).
__global__ void bytes_to_split_kernel(const uint8_t* __restrict__ x, int n, int c, int h, int w, int f, Act out) {
    const long long total = static_cast<long long>(n) * c * h * w;
    GRID_LOOP(i, total) {
        const int xx = static_cast<int>(i % w);
        long long t = i / w;
        const int yy = static_cast<int>(t % h);
        t /= h;
        const int chn = static_cast<int>(t % c);
        const int b = static_cast<int>(t / c);
        const int16_t v = static_cast<int16_t>(rna_div((2 * static_cast<int32_t>(x[i]) - 255) * kFeatureScale, 510));
        const int oy = yy / f, ox = xx / f;
        const int och = chn * f * f + (yy - oy * f) * f + (xx - ox * f);
        const long long px = out.pixel(b, oy, ox);
        out.lo(px)[och] = static_cast<uint8_t>(v & 0xff);
        out.hi(px)[och] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}


// int16::reciprocal of max(q_raw, 256) (src/integer_model.cpp:209-212,
// src/int16_ops.cpp:85-89): sat(rna(512^2 / max(q, 256))).
__global__ void reciprocal_q_kernel(Act qraw, Act out) {
    GRID_LOOP(i, qraw.pixels() * qraw.c) {
        const int c = static_cast<int>(i % qraw.c);
        int b, y, x;
        px_of(qraw, i / qraw.c, b, y, x);
        const long long p = qraw.pixel(b, y, x), op = out.pixel(b, y, x);
        int32_t q = join16(qraw.lo(p)[c], qraw.hi(p)[c]);
        q = q < kFeatureScale / 2 ? kFeatureScale / 2 : q;
        const int16_t v = sat16(rna_div(static_cast<int64_t>(kFeatureScale) * kFeatureScale, q));
        out.lo(op)[c] = static_cast<uint8_t>(v & 0xff);
        out.hi(op)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// out = sat(rna(x * q / 512)) with q an elementwise view (int16::multiply).
__global__ void mul_elementwise_kernel(Act x, Act q, Act out) {
    GRID_LOOP(i, x.pixels() * x.c) {
        const int c = static_cast<int>(i % x.c);
        int b, y, xx;
        px_of(x, i / x.c, b, y, xx);
        const long long p = x.pixel(b, y, xx), qp = q.pixel(b, y, xx), op = out.pixel(b, y, xx);
        const int16_t v = sat16(rna_shift(static_cast<int64_t>(join16(x.lo(p)[c], x.hi(p)[c])) *
                                              join16(q.lo(qp)[c], q.hi(qp)[c]),
                                          9));
        out.lo(op)[c] = static_cast<uint8_t>(v & 0xff);
        out.hi(op)[c] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// pad_right_bottom (src/integer_model.cpp:59-81): replicate the last row and
// column of src into the larger dst.
__global__ void pad_replicate_kernel(Act src, Act dst) {
    const int groups = (dst.c + 15) / 16;
    GRID_LOOP(i, dst.pixels() * groups) {
        const int g = static_cast<int>(i % groups);
        int b, y, x;
        px_of(dst, i / groups, b, y, x);
        const long long sp = src.pixel(b, y < src.h ? y : src.h - 1, x < src.w ? x : src.w - 1);
        const long long dp = dst.pixel(b, y, x);
        for (int c = g * 16; c < dst.c && c < g * 16 + 16; ++c) {
            dst.lo(dp)[c] = src.lo(sp)[c];
            dst.hi(dp)[c] = src.hi(sp)[c];
        }
    }
}

// uint8 frames [n][c][h][w] -> from_bytes -> pad_right_bottom to (hp, wp) ->
// pixel_unshuffle(f), written into a split view (n, hp/f, wp/f, c*f*f).
__global__ void bytes_to_split_padded_kernel(const uint8_t* __restrict__ x, int n, int c, int h, int w, int hp,
                                             int wp, int f, Act out) {
    const long long total = static_cast<long long>(n) * c * hp * wp;
    GRID_LOOP(i, total) {
        const int xx = static_cast<int>(i % wp);
        long long t = i / wp;
        const int yy = static_cast<int>(t % hp);
        t /= hp;
        const int chn = static_cast<int>(t % c);
        const int b = static_cast<int>(t / c);
        const int sy = yy < h ? yy : h - 1, sx = xx < w ? xx : w - 1;
        const uint8_t u = x[((static_cast<long long>(b) * c + chn) * h + sy) * w + sx];
        const int16_t v = static_cast<int16_t>(rna_div((2 * static_cast<int32_t>(u) - 255) * kFeatureScale, 510));
        const int oy = yy / f, ox = xx / f;
        const int och = chn * f * f + (yy - oy * f) * f + (xx - ox * f);
        const long long px = out.pixel(b, oy, ox);
        out.lo(px)[och] = static_cast<uint8_t>(v & 0xff);
        out.hi(px)[och] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

}  // namespace

cudaError_t copy_channels(const Act& src, const Act& dst, cudaStream_t s) {
    copy_channels_kernel<<<grid_for(src.pixels() * ((src.c + 15) / 16)), kBlock, 0, s>>>(src, dst);
    return cudaGetLastError();
}

cudaError_t fill_zero(const Act& dst, cudaStream_t s) {
    fill_zero_kernel<<<grid_for(dst.pixels() * ((dst.c + 15) / 16)), kBlock, 0, s>>>(dst);
    return cudaGetLastError();
}

cudaError_t symbols_to_split(const int8_t* sym, const Act& out, cudaStream_t s) {
    symbols_to_split_kernel<<<grid_for(out.pixels() * out.c), kBlock, 0, s>>>(sym, out);
    return cudaGetLastError();
}

cudaError_t split_to_symbols(const Act& in, int8_t* sym, cudaStream_t s) {
    split_to_symbols_kernel<<<grid_for(in.pixels() * in.c), kBlock, 0, s>>>(in, sym);
    return cudaGetLastError();
}

cudaError_t mul_unshuffle2(const Act& in, const int16_t* q, const Act& out, cudaStream_t s) {
    mul_unshuffle2_kernel<<<grid_for(in.pixels() * in.c), kBlock, 0, s>>>(in, q, out);
    return cudaGetLastError();
}

cudaError_t mul_channels(const Act& in, const int16_t* q, const Act& out, cudaStream_t s) {
    mul_channels_kernel<<<grid_for(in.pixels() * in.c), kBlock, 0, s>>>(in, q, out);
    return cudaGetLastError();
}

cudaError_t lut_split(const Act& in, const int16_t* lut, int groups, const Act& out, cudaStream_t s) {
    lut_split_kernel<<<grid_for(out.pixels() * out.c), kBlock, 0, s>>>(in, lut, groups, out);
    return cudaGetLastError();
}

cudaError_t yhat(const Act& restored, const Act& qraw, const Act& out, cudaStream_t s) {
    yhat_kernel<<<grid_for(restored.pixels() * restored.c), kBlock, 0, s>>>(restored, qraw, out);
    return cudaGetLastError();
}

int prior_blocks_per_stream(int channels, int h, int w) {
    const long long e = static_cast<long long>(channels) * h * w;
    return static_cast<int>((e + kChunk - 1) / kChunk);
}

cudaError_t prior_scan(int channels, int h, int w, int n, int part, const Act& scales, int thr, int* block_counts,
                       int* totals, cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_count_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, thr, block_counts, bps);
    prior_scan_kernel<<<n, kPriorThreads, 0, s>>>(block_counts, bps, totals);
    return cudaGetLastError();
}

cudaError_t prior_indexes(int channels, int h, int w, int n, int part, const Act& scales, int thr,
                          const int* offsets, const uint8_t* scale_index, uint8_t* indexes, long long cap,
                          cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_indexes_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, thr, offsets, bps, scale_index,
                                                                  indexes, cap);
    return cudaGetLastError();
}

cudaError_t prior_restore(int channels, int h, int w, int n, int part, const Act& scales, const Act& means, int thr,
                          const int* offsets, const int8_t* symbols, long long cap, const Act& restored,
                          cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_restore_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, means, thr, offsets, bps, symbols,
                                                                  cap, restored);
    return cudaGetLastError();
}

cudaError_t prior_encode(int channels, int h, int w, int n, int part, const Act& scales, const Act& means,
                         const Act& yenc, int thr, const int* offsets, const uint8_t* scale_index, int16_t* packed,
                         long long cap, const Act& restored, cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_encode_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, means, yenc, thr, offsets, bps,
                                                                 scale_index, packed, cap, restored);
    return cudaGetLastError();
}

cudaError_t raw_frame(const Act& head, int height, int width, uint8_t* out, long long frame_bytes, cudaStream_t s) {
    const long long per = static_cast<long long>(height) * width * 3 / 2;
    raw_frame_kernel<<<grid_for(head.n * per), kBlock, 0, s>>>(head, height, width, out, frame_bytes);
    return cudaGetLastError();
}

cudaError_t bytes_to_split(const uint8_t* x, int n, int c, int h, int w, int f, const Act& out, cudaStream_t s) {
    bytes_to_split_kernel<<<grid_for(static_cast<long long>(n) * c * h * w), kBlock, 0, s>>>(x, n, c, h, w, f, out);
    return cudaGetLastError();
}

cudaError_t reciprocal_q(const Act& qraw, const Act& out, cudaStream_t s) {
    reciprocal_q_kernel<<<grid_for(qraw.pixels() * qraw.c), kBlock, 0, s>>>(qraw, out);
    return cudaGetLastError();
}

cudaError_t mul_elementwise(const Act& x, const Act& q, const Act& out, cudaStream_t s) {
    mul_elementwise_kernel<<<grid_for(x.pixels() * x.c), kBlock, 0, s>>>(x, q, out);
    return cudaGetLastError();
}

cudaError_t pad_replicate(const Act& src, const Act& dst, cudaStream_t s) {
    pad_replicate_kernel<<<grid_for(dst.pixels() * ((dst.c + 15) / 16)), kBlock, 0, s>>>(src, dst);
    return cudaGetLastError();
}

cudaError_t bytes_to_split_padded(const uint8_t* x, int n, int c, int h, int w, int hp, int wp, int f, const Act& out,
                                  cudaStream_t s) {
    bytes_to_split_padded_kernel<<<grid_for(static_cast<long long>(n) * c * hp * wp), kBlock, 0, s>>>(x, n, c, h, w,
                                                                                                      hp, wp, f, out);
    return cudaGetLastError();
}

}  // namespace ufb
