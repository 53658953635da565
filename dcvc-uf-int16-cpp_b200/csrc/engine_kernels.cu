// Model-level memory-bound kernels on split-NHWC views: channel copies (cat),
// symbol <-> feature conversions, multiply / unshuffle fusions, the
// entropy-parameter kernels of IntegerModel::prior, and raw-frame output.
#include "engine_kernels.h"
#include "uf_common.cuh"

#include <climits>

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
// One thread per output pixel and 16 output channels (input channels c0 ..
// c0 + 3 of the four input pixels), stored as one 16-byte word per plane
// where the views allow; the multiplier product is the 32-bit one of
// mul_channels_kernel (defined below).
__device__ __forceinline__ int16_t mul_q9(int32_t v, int32_t q);

__global__ void mul_unshuffle2_kernel(Act in, const int16_t* __restrict__ q, Act out) {
    const int groups = (in.c + 3) / 4;
    GRID_LOOP(i, out.pixels() * groups) {
        const int g = static_cast<int>(i % groups);
        int b, oy, ox;
        px_of(out, i / groups, b, oy, ox);
        const int c0 = 4 * g;
        const long long op = out.pixel(b, oy, ox);
        uint8_t* ol = out.lo(op) + 4 * c0;
        uint8_t* oh = out.hi(op) + 4 * c0;
        long long ip[4];  // input pixel of sub-position ij = 2 i + j
#pragma unroll
        for (int ij = 0; ij < 4; ++ij) ip[ij] = in.pixel(b, 2 * oy + (ij >> 1), 2 * ox + (ij & 1));
        uintptr_t align = reinterpret_cast<uintptr_t>(ol) | reinterpret_cast<uintptr_t>(oh);
#pragma unroll
        for (int ij = 0; ij < 4; ++ij)
            align |= (reinterpret_cast<uintptr_t>(in.lo(ip[ij]) + c0) | reinterpret_cast<uintptr_t>(in.hi(ip[ij]) + c0)) &
                     3;
        if (c0 + 4 <= in.c && 2 * oy + 1 < in.h && 2 * ox + 1 < in.w && (align & 15) == 0) {
            uint32_t lw[4], hw[4];
#pragma unroll
            for (int ij = 0; ij < 4; ++ij) {
                lw[ij] = *reinterpret_cast<const uint32_t*>(in.lo(ip[ij]) + c0);
                hw[ij] = *reinterpret_cast<const uint32_t*>(in.hi(ip[ij]) + c0);
            }
            uint32_t rl[4], rh[4];  // output word cc holds channels 4 (c0 + cc) + ij
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                rl[cc] = rh[cc] = 0;
#pragma unroll
                for (int ij = 0; ij < 4; ++ij) {
                    int16_t v = static_cast<int16_t>(((lw[ij] >> (8 * cc)) & 0xffu) |
                                                     (((hw[ij] >> (8 * cc)) & 0xffu) << 8));
                    if (q) v = mul_q9(v, q[c0 + cc]);
                    const uint16_t u = static_cast<uint16_t>(v);
                    rl[cc] |= static_cast<uint32_t>(u & 0xffu) << (8 * ij);
                    rh[cc] |= static_cast<uint32_t>(u >> 8) << (8 * ij);
                }
            }
            *reinterpret_cast<uint4*>(ol) = make_uint4(rl[0], rl[1], rl[2], rl[3]);
            *reinterpret_cast<uint4*>(oh) = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        } else {
            for (int k = 0; k < 16; ++k) {
                const int c = c0 + (k >> 2), ij = k & 3;
                const int iy = 2 * oy + (ij >> 1), ix = 2 * ox + (ij & 1);
                if (c >= in.c || iy >= in.h || ix >= in.w) continue;
                int16_t v = join16(in.lo(ip[ij])[c], in.hi(ip[ij])[c]);
                if (q) v = mul_q9(v, q[c]);
                ol[k] = static_cast<uint8_t>(v & 0xff);
                oh[k] = static_cast<uint8_t>((v >> 8) & 0xff);
            }
        }
    }
}

// sat(rna(v * q / 512)) in 32 bits (|v * q| <= 2^30).
__device__ __forceinline__ int16_t mul_q9(int32_t v, int32_t q) {
    const int32_t pr = v * q;
    const int32_t sg = pr >> 31;
    const int32_t r = (((pr ^ sg) - sg) + 256) >> 9;
    return sat16i((r ^ sg) - sg);
}

// out = sat(rna(in * q / 512)) with one multiplier per channel; 16 channels
// of one pixel per thread, in 16-byte words where the views allow.
__global__ void mul_channels_kernel(Act in, const int16_t* __restrict__ q, Act out) {
    const int groups = (in.c + 15) / 16;
    GRID_LOOP(i, in.pixels() * groups) {
        const int g = static_cast<int>(i % groups);
        int b, y, x;
        px_of(in, i / groups, b, y, x);
        const long long p = in.pixel(b, y, x), op = out.pixel(b, y, x);
        const int c0 = g * 16;
        const uint8_t* il = in.lo(p) + c0;
        const uint8_t* ih = in.hi(p) + c0;
        uint8_t* ol = out.lo(op) + c0;
        uint8_t* oh = out.hi(op) + c0;
        const uintptr_t align = reinterpret_cast<uintptr_t>(il) | reinterpret_cast<uintptr_t>(ih) |
                                reinterpret_cast<uintptr_t>(ol) | reinterpret_cast<uintptr_t>(oh);
        if (c0 + 16 <= in.c && (align & 15) == 0) {
            const uint4 l4 = *reinterpret_cast<const uint4*>(il), h4 = *reinterpret_cast<const uint4*>(ih);
            const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
            uint32_t rl[4], rh[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                rl[w] = rh[w] = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int32_t v = static_cast<int16_t>(((lw[w] >> (8 * k)) & 0xffu) | (((hw[w] >> (8 * k)) & 0xffu) << 8));
                    const uint16_t r = static_cast<uint16_t>(mul_q9(v, q[c0 + 4 * w + k]));
                    rl[w] |= static_cast<uint32_t>(r & 0xffu) << (8 * k);
                    rh[w] |= static_cast<uint32_t>(r >> 8) << (8 * k);
                }
            }
            *reinterpret_cast<uint4*>(ol) = make_uint4(rl[0], rl[1], rl[2], rl[3]);
            *reinterpret_cast<uint4*>(oh) = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        } else {
            const int n = in.c - c0 < 16 ? in.c - c0 : 16;
            for (int k = 0; k < n; ++k) {
                const int16_t v = mul_q9(join16(il[k], ih[k]), q[c0 + k]);
                ol[k] = static_cast<uint8_t>(v & 0xff);
                oh[k] = static_cast<uint8_t>((v >> 8) & 0xff);
            }
        }
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
    long long elems;      // channels * h * w (below 2^31, checked by the launchers)
};

// (c, y, x) of NCHW position e of one stream (32-bit divisions), and the
// position after (c, y, x).
__device__ __forceinline__ void prior_pos(const PriorGeom& g, long long e, int& c, int& y, int& x) {
    const uint32_t u = static_cast<uint32_t>(e);
    const uint32_t t = u / static_cast<uint32_t>(g.w);
    x = static_cast<int>(u - t * static_cast<uint32_t>(g.w));
    const uint32_t cc = t / static_cast<uint32_t>(g.h);
    y = static_cast<int>(t - cc * static_cast<uint32_t>(g.h));
    c = static_cast<int>(cc);
}

__device__ __forceinline__ void prior_next(const PriorGeom& g, int& c, int& y, int& x) {
    if (++x == g.w) {
        x = 0;
        if (++y == g.h) {
            y = 0;
            ++c;
        }
    }
}

__device__ __forceinline__ bool prior_flag(const PriorGeom& g, int b, int c, int y, int x, int part,
                                           const Act& scales, int thr, int16_t& scale_out) {
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
        prior_pos(g, e, c, y, x);
        count += prior_flag(g, b, c, y, x, part, scales, thr, s) ? 1 : 0;
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
    int c0 = 0, y0 = 0, x0 = 0;
    if (first < g.elems) prior_pos(g, first, c0, y0, x0);
    uint32_t mask = 0, parts = 0;  // active positions; positions of this part
    int16_t sc[kPer];
    int c = c0, y = y0, x = x0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const long long e = first + k;
        sc[k] = 0;
        if (e < g.elems && part_of(c, g.channels, y, x) == part) {
            parts |= 1u << k;
            const long long p = scales.pixel(b, y, x);
            sc[k] = join16(scales.lo(p)[c], scales.hi(p)[c]);
            if (thr == 0 || sc[k] > thr) mask |= 1u << k;
        }
        prior_next(g, c, y, x);
    }
    __shared__ int total;
    int rank = block_offset + block_scan(__popc(mask), &total);
    c = c0, y = y0, x = x0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const long long e = first + k;
        if (e >= g.elems) break;
        const bool in_part = (parts >> k) & 1u;
        const bool active = (mask >> k) & 1u;
        fn(in_part, active, active ? rank : -1, c, y, x, sc[k]);
        if (active) ++rank;
        prior_next(g, c, y, x);
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
// is channel k * 64 + (Y % 8) * 8 + X % 8 of head pixel (Y / 8, X / 8).  The
// grid is x over columns, y over the rows of one output image (height luma
// rows, then height / 2 rows of U and as many of V), z over images, so no
// thread divides; every sum fits int32 and the divisions by powers of two are
// shifts: luma rna((v + 256) * 255 / 512), chroma floor((s + 1024) * 255 / 2048)
// over the four samples s of a 2 x 2 block.
static_assert(kFeatureScale == 512, "raw_frame's shifts are written for a feature scale of 512");
__global__ void raw_frame_kernel(Act head, int height, int width, uint8_t* __restrict__ out, long long frame_bytes) {
    const int b = blockIdx.z, row = blockIdx.y;
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    uint8_t* o = out + b * frame_bytes;
    auto sample = [&](int comp, int Y, int X) -> int32_t {
        const long long p = head.pixel(b, Y >> 3, X >> 3);
        const int c = comp * 64 + (Y & 7) * 8 + (X & 7);
        return join16(head.lo(p)[c], head.hi(p)[c]);
    };
    if (row < height) {
        if (x >= width) return;
        const int32_t t = (sample(0, row, x) + 256) * 255;
        const int32_t v = t < 0 ? -((256 - t) >> 9) : (t + 256) >> 9;
        o[static_cast<long long>(row) * width + x] = static_cast<uint8_t>(min(max(v, 0), 255));
    } else {
        const int ch = height / 2, cw = width / 2;
        if (x >= cw) return;
        const int r = row - height;
        const int comp = r < ch ? 1 : 2;
        const int y = r - (comp - 1) * ch;
        const int32_t sum = sample(comp, 2 * y, 2 * x) + sample(comp, 2 * y + 1, 2 * x) +
                            sample(comp, 2 * y, 2 * x + 1) + sample(comp, 2 * y + 1, 2 * x + 1);
        const int32_t v = ((sum + 1024) * 255) >> 11;
        const long long at = static_cast<long long>(height) * width + static_cast<long long>(comp - 1) * ch * cw +
                             static_cast<long long>(y) * cw + x;
        o[at] = static_cast<uint8_t>(min(max(v, 0), 255));
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
    mul_unshuffle2_kernel<<<grid_for(out.pixels() * ((in.c + 3) / 4)), kBlock, 0, s>>>(in, q, out);
    return cudaGetLastError();
}

cudaError_t mul_channels(const Act& in, const int16_t* q, const Act& out, cudaStream_t s) {
    mul_channels_kernel<<<grid_for(in.pixels() * ((in.c + 15) / 16)), kBlock, 0, s>>>(in, q, out);
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
    if (g.elems > INT_MAX) return cudaErrorInvalidValue;
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_count_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, thr, block_counts, bps);
    prior_scan_kernel<<<n, kPriorThreads, 0, s>>>(block_counts, bps, totals);
    return cudaGetLastError();
}

cudaError_t prior_indexes(int channels, int h, int w, int n, int part, const Act& scales, int thr,
                          const int* offsets, const uint8_t* scale_index, uint8_t* indexes, long long cap,
                          cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    if (g.elems > INT_MAX) return cudaErrorInvalidValue;
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_indexes_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, thr, offsets, bps, scale_index,
                                                                  indexes, cap);
    return cudaGetLastError();
}

cudaError_t prior_restore(int channels, int h, int w, int n, int part, const Act& scales, const Act& means, int thr,
                          const int* offsets, const int8_t* symbols, long long cap, const Act& restored,
                          cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    if (g.elems > INT_MAX) return cudaErrorInvalidValue;
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_restore_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, means, thr, offsets, bps, symbols,
                                                                  cap, restored);
    return cudaGetLastError();
}

cudaError_t prior_encode(int channels, int h, int w, int n, int part, const Act& scales, const Act& means,
                         const Act& yenc, int thr, const int* offsets, const uint8_t* scale_index, int16_t* packed,
                         long long cap, const Act& restored, cudaStream_t s) {
    PriorGeom g{channels, h, w, static_cast<long long>(channels) * h * w};
    if (g.elems > INT_MAX) return cudaErrorInvalidValue;
    const int bps = prior_blocks_per_stream(channels, h, w);
    prior_encode_kernel<<<dim3(bps, n), kPriorThreads, 0, s>>>(g, part, scales, means, yenc, thr, offsets, bps,
                                                                 scale_index, packed, cap, restored);
    return cudaGetLastError();
}

cudaError_t raw_frame(const Act& head, int height, int width, uint8_t* out, long long frame_bytes, cudaStream_t s) {
    if (head.n <= 0 || height <= 0 || width <= 0) return cudaSuccess;
    const int rows = height + 2 * (height / 2);
    if (head.n > 65535 || rows > 65535) return cudaErrorInvalidValue;
    const dim3 grid((width + 255) / 256, rows, head.n);
    raw_frame_kernel<<<grid, 256, 0, s>>>(head, height, width, out, frame_bytes);
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
