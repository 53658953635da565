// Depthwise 3x3, stride 1, zero padding 1 on split views (DepthConvBlock dc.2,
// src/layers.cpp:96; the reference runs it through its scalar `general`
// kernel, src/cuda/conv.cu:44-60).
//
// Persistent CTAs walk output tiles of 128 channels x 16 columns x 8 rows.
// Each tile's input window (18 x 10 pixels with the halo, both byte planes,
// 45 KB) arrives by TMA into one of two shared-memory buffers while the
// previous tile is computed from the other; the halo outside the image is the
// TMA's zero fill, which is exactly the convolution's padding.  Each warp
// releases a buffer with one arrival on its `empty` mbarrier, and only warp 0,
// which issues the next window load into it, waits for all eight, so the other
// warps run on into the next tile without a CTA-wide barrier.  A thread owns
// four channels (one 32-bit word of each plane) of two adjacent output columns
// and slides down the tile's rows, reading each input row once from shared
// memory (a warp reads one 128-byte pixel line).  The arithmetic stays on the
// byte planes as they are stored: with x = 256 h + l (l unsigned, h signed
// bytes), S = 256 sum(h w) + sum(l w), and each partial sum of nine taps fits
// in 32 bits (|sum(l w)| <= 9 * 255 * 2^15).  Two-way dot-product instructions
// (16-bit weight pair times two bytes) take taps (0, 1) of a weight row in one
// instruction and tap 2 in another, and the output is rna(S / 8192) recombined
// exactly in 32-bit arithmetic, as the tensor-core epilogue does.
#include "kernels.h"

#include "conv_epi.cuh"
#include "conv_tc.h"
#include "umma.cuh"

#include <cuda.h>
#include <cuda_runtime.h>
#include <climits>
#include <cstdlib>
#include <string>

namespace ufb {

namespace {

constexpr int kQuads = 32;                        // channel quads per tile (128 channels)
constexpr int kColThreads = 8;                    // threads along x
constexpr int kCols = 2;                          // output columns per thread
constexpr int kTileW = kColThreads * kCols;       // 16 output columns
constexpr int kTileH = 8;                         // output rows
constexpr int kInW = kTileW + 2, kInH = kTileH + 2;
constexpr uint32_t kLine = 4 * kQuads;            // bytes of one plane of one pixel in the window
constexpr uint32_t kPlane = kInW * kInH * kLine;  // 23040: one byte plane of the window
constexpr uint32_t kBuffer = 2 * kPlane;          // both planes
constexpr int kThreads = kQuads * kColThreads;    // 256
constexpr size_t kSmem = 2 * size_t(kBuffer) + 128;  // two buffers, 128-byte alignment slack

// Exact sums of one output row: S = 256 h + l over the two byte planes of the
// input (l: unsigned low bytes, h: signed high bytes) for [column][channel].
struct DwAcc {
    int32_t l[kCols][4], h[kCols][4];
};

__device__ __forceinline__ void dw_zero(DwAcc& a) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) a.l[j][c] = a.h[j][c] = 0;
}

// Two-way dot products: signed 16-bit pair a times two bytes of b (unsigned
// or signed) plus c; .lo takes bytes 0 and 1 of b, .hi bytes 2 and 3.
__device__ __forceinline__ int32_t dp2_lo_u(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dp2_hi_u(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dp2_lo_s(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dp2_hi_s(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One input row in the forms the dot products take: for output column j,
// pair[j][g] interleaves the bytes of pixels j and j + 1 for channels 2g and
// 2g + 1 (taps kx = 0, 1), one[j][s] holds pixel j + 2 shifted by 8 s bits
// (tap kx = 2: channel s in byte 0 and channel s + 2 in byte 2).
struct DwRow {
    uint32_t pair[kCols][2], one[kCols][2];
};

__device__ __forceinline__ void dw_prep(const uint32_t (&v)[kCols + 2], DwRow& r) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
        r.pair[j][0] = __byte_perm(v[j], v[j + 1], 0x5140);
        r.pair[j][1] = __byte_perm(v[j], v[j + 1], 0x7362);
        r.one[j][0] = v[j + 2];
        r.one[j][1] = v[j + 2] >> 8;
    }
}

// Adds one input row into an output row through weight row ky: wp[c] packs
// taps (0, 1) of channel c as int16 halves, ws[c] tap 2 with a zero high half.
// The sums start (FRESH: the row's first input row) from l = 4096, the
// rounding half of rna(S / 8192), and h = 32 bias, which adds the bias to
// h >> 5 without touching h & 31, so the store needs neither.
template <bool FRESH>
__device__ __forceinline__ void dw_add(DwAcc& a, const DwRow& lo, const DwRow& hi, const uint32_t (&wp)[4],
                                       const uint32_t (&ws)[4], const int32_t (&h0)[4]) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
        int32_t l[4], h[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            l[c] = FRESH ? 4096 : a.l[j][c];
            h[c] = FRESH ? h0[c] : a.h[j][c];
        }
        a.l[j][0] = dp2_lo_u(ws[0], lo.one[j][0], dp2_lo_u(wp[0], lo.pair[j][0], l[0]));
        a.l[j][1] = dp2_lo_u(ws[1], lo.one[j][1], dp2_hi_u(wp[1], lo.pair[j][0], l[1]));
        a.l[j][2] = dp2_hi_u(ws[2], lo.one[j][0], dp2_lo_u(wp[2], lo.pair[j][1], l[2]));
        a.l[j][3] = dp2_hi_u(ws[3], lo.one[j][1], dp2_hi_u(wp[3], lo.pair[j][1], l[3]));
        a.h[j][0] = dp2_lo_s(ws[0], hi.one[j][0], dp2_lo_s(wp[0], hi.pair[j][0], h[0]));
        a.h[j][1] = dp2_lo_s(ws[1], hi.one[j][1], dp2_hi_s(wp[1], hi.pair[j][0], h[1]));
        a.h[j][2] = dp2_hi_s(ws[2], hi.one[j][0], dp2_lo_s(wp[2], hi.pair[j][1], h[2]));
        a.h[j][3] = dp2_hi_s(ws[3], hi.one[j][1], dp2_hi_s(wp[3], hi.pair[j][1], h[3]));
    }
}

// sat(rna(S / 8192) + bias) of two output columns, stored as one 32-bit word
// per plane.  With l = 4096 + sum(l w) and h = 32 bias + sum(h w):
// U = l + 256 (h & 31) and T = (h >> 5) + (U >> 13) = floor((S + 4096) / 8192)
// + bias, and an exact tie (U % 8192 == 0) with S < 0, i.e. T <= bias, rounds
// away from zero to T - 1 (the recombination of conv_epi.cuh, recombine32).
// The output pixel of column j sits at lo + j * px_bytes (low plane) and
// pitch bytes further (high plane); columns from ncols on are outside the image.
__device__ __forceinline__ void dw_store(const DwAcc& a, const int32_t (&b)[4], uint8_t* lo, long long px_bytes,
                                         int pitch, int ncols) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
        if (j >= ncols) break;
        int32_t r[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int32_t U = a.l[j][c] + ((a.h[j][c] & 31) << 8);
            const int32_t T = (a.h[j][c] >> 5) + (U >> 13);
            r[c] = T - static_cast<int32_t>(((U & 8191) == 0) & (T <= b[c]));
        }
        const uint32_t p0 = pack2_sat(r[0], r[1]), p1 = pack2_sat(r[2], r[3]);
        uint8_t* dst = lo + j * px_bytes;
        *reinterpret_cast<uint32_t*>(dst) = __byte_perm(p0, p1, 0x6420);
        *reinterpret_cast<uint32_t*>(dst + pitch) = __byte_perm(p0, p1, 0x7531);
    }
}

// Narrow layers (every channel: 32768 sum|w| + 4096 + 8192 |bias| < 2^31, see
// dw_narrow_ok): the whole sum S + 4096 + 8192 bias fits one int32, so each tap
// is one multiply-add of full int16 values and the store needs one compare.
struct DwAccN {
    int32_t s[kCols][4];
};

// Window row r as int16 values sign-extended to 32 bits: x[p][c] for window
// columns 2t + p and channels 4q + c (one byte permute per value).
struct DwRowN {
    int32_t x[kCols + 2][4];
};

// prmt.b32 in its default mode: a selector nibble with bit 3 set fills the
// byte with the sign of the selected source byte.
__device__ __forceinline__ int32_t prmt_sx(uint32_t a, uint32_t b, uint32_t sel) {
    int32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void dw_row_n(const uint8_t* buf, int r, int t, int q, DwRowN& row) {
#pragma unroll
    for (int p = 0; p < kCols + 2; ++p) {
        const uint32_t off = (static_cast<uint32_t>(r) * kInW + kCols * t + p) * kLine + 4 * q;
        const uint32_t lw = *reinterpret_cast<const uint32_t*>(buf + off);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(buf + kPlane + off);
        // bytes [lo c, hi c, sign(hi c), sign(hi c)]: selector nibbles 8-15 replicate a byte's sign
        row.x[p][0] = prmt_sx(lw, hw, 0xCC40);
        row.x[p][1] = prmt_sx(lw, hw, 0xDD51);
        row.x[p][2] = prmt_sx(lw, hw, 0xEE62);
        row.x[p][3] = prmt_sx(lw, hw, 0xFF73);
    }
}

// Adds one input row through weight row w[kx][c]; FRESH starts the sums from
// 4096 + 8192 bias (held in s0).
template <bool FRESH>
__device__ __forceinline__ void dw_add_n(DwAccN& a, const DwRowN& row, const int32_t (&w)[3][4],
                                         const int32_t (&s0)[4]) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            int32_t v = FRESH ? s0[c] : a.s[j][c];
            v += row.x[j][c] * w[0][c];
            v += row.x[j + 1][c] * w[1][c];
            v += row.x[j + 2][c] * w[2][c];
            a.s[j][c] = v;
        }
}

// sat(rna(S / 8192) + bias) from s = S + 4096 + 8192 bias: rna(S / 8192) =
// floor((S + 4096 - [S < 0]) / 8192), and S < 0 exactly when s < s0.
// (stored as dw_store does).
__device__ __forceinline__ void dw_store_n(const DwAccN& a, const int32_t (&s0)[4], uint8_t* lo, long long px_bytes,
                                           int pitch, int ncols) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
        if (j >= ncols) break;
        int32_t r[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) r[c] = (a.s[j][c] - static_cast<int32_t>(a.s[j][c] < s0[c])) >> 13;
        const uint32_t p0 = pack2_sat(r[0], r[1]), p1 = pack2_sat(r[2], r[3]);
        uint8_t* dst = lo + j * px_bytes;
        *reinterpret_cast<uint32_t*>(dst) = __byte_perm(p0, p1, 0x6420);
        *reinterpret_cast<uint32_t*>(dst + pitch) = __byte_perm(p0, p1, 0x7531);
    }
}

// Window row r, columns 2t .. 2t + 3, channels 4q .. 4q + 3 of both planes.
__device__ __forceinline__ void dw_row(const uint8_t* buf, int r, int t, int q, DwRow& lo, DwRow& hi) {
    uint32_t lw[kCols + 2], hw[kCols + 2];
#pragma unroll
    for (int p = 0; p < kCols + 2; ++p) {
        const uint32_t off = (static_cast<uint32_t>(r) * kInW + kCols * t + p) * kLine + 4 * q;
        lw[p] = *reinterpret_cast<const uint32_t*>(buf + off);
        hw[p] = *reinterpret_cast<const uint32_t*>(buf + kPlane + off);
    }
    dw_prep(lw, lo);
    dw_prep(hw, hi);
}

template <bool NARROW>
__global__ void __launch_bounds__(kThreads, 2)
dwconv3x3_kernel(const __grid_constant__ CUtensorMap map, Act out, const int16_t* __restrict__ weight,
                     const int16_t* __restrict__ bias, int channels, int tiles_x, int tiles_y, int images,
                     int total_tiles, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    // full[b]: the window load into buffer b landed; empty[b]: every warp is
    // done reading buffer b (one arrival per warp)
    __shared__ __align__(8) uint64_t full[2], empty[2];
    const int q = threadIdx.x % kQuads, t = threadIdx.x / kQuads;  // t is also the warp index
    const int per_block = tiles_x * tiles_y * images;  // tiles of one channel block

    auto issue = [&](int tile, int b) {
        const int cb = tile / per_block;
        int r = tile - cb * per_block;
        const int tx = r % tiles_x;
        r /= tiles_x;
        const int ty = r % tiles_y;
        const int img = r / tiles_y;
        uint8_t* dst = smem + b * kBuffer;
        mbar_arrive_expect_tx(&full[b], kBuffer);
        tma_load_5d(dst, &map, &full[b], cb * 4 * kQuads, 0, tx * kTileW - 1, ty * kTileH - 1, img);
        tma_load_5d(dst + kPlane, &map, &full[b], cb * 4 * kQuads, 1, tx * kTileW - 1, ty * kTileH - 1, img);
    };

    if (threadIdx.x == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        mbar_init(&empty[0], kThreads / 32);
        mbar_init(&empty[1], kThreads / 32);
        fence_mbar_init();
        prefetch_tmap(&map);
    }
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x < total_tiles) issue(blockIdx.x, 0);

    uint32_t wp[3][4], ws[3][4];  // general: taps (0, 1) packed, tap 2
    int32_t wn[3][3][4];           // narrow: [ky][kx][channel]
    int32_t bv[4];
    int loaded_cb = -1;
    int i = 0;
    bool next_issued = false;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++i) {
        const int b = i & 1;
        next_issued = tile + static_cast<int>(gridDim.x) < total_tiles;
        if (t == 0) {
            // warp 0 refills the other buffer once every warp has released its
            // previous use (tile i - 1); the other warps run on meanwhile
            int ok = 1;
            if (q == 0 && next_issued) {
                ok = i == 0 || mbar_wait(&empty[b ^ 1], ((i - 1) >> 1) & 1, status, 11);
                if (ok) issue(tile + gridDim.x, b ^ 1);
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
                // abort: the load into this tile's buffer must land before the CTA exits
                if (q == 0) mbar_wait(&full[b], (i >> 1) & 1, status, 10);
                break;
            }
        }
        const int cb = tile / per_block;
        int r = tile - cb * per_block;
        const int tx = r % tiles_x;
        r /= tiles_x;
        const int ty = r % tiles_y;
        const int img = r / tiles_y;
        const int c0 = cb * 4 * kQuads + 4 * q;
        if (cb != loaded_cb) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const bool ok = c0 + c < channels;
#pragma unroll
                for (int ky = 0; ky < 3; ++ky) {
                    if (NARROW) {
#pragma unroll
                        for (int kx = 0; kx < 3; ++kx) wn[ky][kx][c] = ok ? weight[(c0 + c) * 9 + 3 * ky + kx] : 0;
                    } else {
                        const uint32_t w0 = ok ? static_cast<uint16_t>(weight[(c0 + c) * 9 + 3 * ky]) : 0;
                        const uint32_t w1 = ok ? static_cast<uint16_t>(weight[(c0 + c) * 9 + 3 * ky + 1]) : 0;
                        const uint32_t w2 = ok ? static_cast<uint16_t>(weight[(c0 + c) * 9 + 3 * ky + 2]) : 0;
                        wp[ky][c] = w0 | (w1 << 16);
                        ws[ky][c] = w2;
                    }
                }
                bv[c] = ok && bias ? bias[c0 + c] : 0;
            }
            loaded_cb = cb;
        }
        const bool ready = mbar_wait(&full[b], (i >> 1) & 1, status, 9);
        if (!__all_sync(0xffffffffu, ready)) {
            // abort (every wait is bounded, so the other warps give up too): the
            // window load of the next tile must land before the CTA exits
            if (threadIdx.x == 0 && next_issued) mbar_wait(&full[b ^ 1], ((i + 1) >> 1) & 1, status, 10);
            break;
        }
        const uint8_t* buf = smem + b * kBuffer;
        const int oy0 = ty * kTileH, ox = tx * kTileW + kCols * t;
        const bool active = c0 < channels && ox < out.w;
        // low-plane address of this thread's first output of the next row to store
        const long long px_bytes = 2ll * out.pitch, row_bytes = px_bytes * out.row_px;
        const int ncols = min(kCols, out.w - ox);
        uint8_t* dst = active ? out.lo(out.pixel(img, oy0, ox)) + c0 : nullptr;
        if (active && NARROW) {
            // the general path's row schedule with whole-value sums
            const int32_t s0[4] = {4096 + 8192 * bv[0], 4096 + 8192 * bv[1], 4096 + 8192 * bv[2],
                                   4096 + 8192 * bv[3]};
            DwAccN a0, a1, a2;
            DwRowN row;
            auto step = [&](DwAccN& next, DwAccN& mid, DwAccN& done, int wr) {
                dw_row_n(buf, wr, t, q, row);
                dw_add_n<true>(next, row, wn[0], s0);
                if (wr >= 1) dw_add_n<false>(mid, row, wn[1], s0);
                if (wr >= 2) {
                    dw_add_n<false>(done, row, wn[2], s0);
                    if (oy0 + wr - 2 < out.h) dw_store_n(done, s0, dst, px_bytes, out.pitch, ncols);
                    dst += row_bytes;
                }
            };
#pragma unroll 1
            for (int wr = 0; wr < kInH; wr += 3) {
                step(a0, a1, a2, wr);
                if (wr + 1 >= kInH) break;
                step(a2, a0, a1, wr + 1);
                if (wr + 2 >= kInH) break;
                step(a1, a2, a0, wr + 2);
            }
        } else if (active) {
            // output rows r - 2, r - 1, r take window row r through weight rows
            // 2, 1, 0; row r starts there (the rows -1 and -2 of the first two
            // steps are never stored)
            const int32_t h0[4] = {32 * bv[0], 32 * bv[1], 32 * bv[2], 32 * bv[3]};
            DwAcc a0, a1, a2;
            dw_zero(a1);
            dw_zero(a2);
            DwRow lo, hi;
            auto step = [&](DwAcc& next, DwAcc& mid, DwAcc& done, int wr) {
                dw_row(buf, wr, t, q, lo, hi);
                dw_add<true>(next, lo, hi, wp[0], ws[0], h0);
                dw_add<false>(mid, lo, hi, wp[1], ws[1], h0);
                dw_add<false>(done, lo, hi, wp[2], ws[2], h0);
                if (wr >= 2) {
                    if (oy0 + wr - 2 < out.h) dw_store(done, bv, dst, px_bytes, out.pitch, ncols);
                    dst += row_bytes;
                }
            };
#pragma unroll 1
            for (int wr = 0; wr < kInH; wr += 3) {
                step(a0, a1, a2, wr);
                if (wr + 1 >= kInH) break;
                step(a2, a0, a1, wr + 1);
                if (wr + 2 >= kInH) break;
                step(a1, a2, a0, wr + 2);
            }
        }
        __syncwarp();
        if (q == 0) mbar_arrive(&empty[b]);  // this warp is done with the buffer
    }
}

}  // namespace

bool dw_narrow_ok(const int16_t* weight_host, const int16_t* bias_host, int channels) {
    for (int c = 0; c < channels; ++c) {
        long long bound = 4096 + 8192ll * (bias_host ? std::abs(static_cast<int>(bias_host[c])) : 0);
        for (int k = 0; k < 9; ++k) bound += 32768ll * std::abs(static_cast<int>(weight_host[c * 9 + k]));
        if (bound > INT32_MAX) return false;
    }
    return true;
}

cudaError_t dwconv3x3(const Act& in, const Act& out, const int16_t* weight, const int16_t* bias, int* status,
                      cudaStream_t s, bool narrow) {
    if (in.c % 4 || in.c != out.c || in.h != out.h || in.w != out.w || in.n != out.n || in.pitch % 16 ||
        out.pitch % 16 || reinterpret_cast<uintptr_t>(in.base) % 16 || reinterpret_cast<uintptr_t>(out.base) % 16 ||
        !status)
        return cudaErrorInvalidValue;
    // window map over the split view {channel, plane, x, y, image}; the box is
    // one tile's window of one plane, zero filled outside the view
    CUtensorMap map;
    const cuuint64_t dims[5] = {static_cast<cuuint64_t>(in.c), 2, static_cast<cuuint64_t>(in.w),
                                static_cast<cuuint64_t>(in.h), static_cast<cuuint64_t>(in.n)};
    const cuuint64_t strides[4] = {static_cast<cuuint64_t>(in.pitch), static_cast<cuuint64_t>(2 * in.pitch),
                                   static_cast<cuuint64_t>(2 * in.pitch) * in.row_px,
                                   static_cast<cuuint64_t>(2 * in.pitch) * in.img_px};
    const cuuint32_t box[5] = {4 * kQuads, 1, kInW, kInH, 1};
    std::string err;
    if (!tc_encode_map(&map, in.base, 5, dims, strides, box, err, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    const int ch_blocks = (in.c + 4 * kQuads - 1) / (4 * kQuads);
    const int tiles_x = (in.w + kTileW - 1) / kTileW, tiles_y = (in.h + kTileH - 1) / kTileH;
    const long long total = static_cast<long long>(ch_blocks) * tiles_x * tiles_y * in.n;
    if (total > INT32_MAX) return cudaErrorInvalidValue;
    narrow = narrow && tc_narrow_enabled();
    auto kernel = narrow ? dwconv3x3_kernel<true> : dwconv3x3_kernel<false>;
    // per device; always the same value, so concurrent callers cannot disagree
    const cudaError_t attr =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
    if (attr != cudaSuccess) return attr;
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    long long grid = total < 2ll * sms ? total : 2ll * sms;
    const int cap = tc_max_ctas();
    if (cap > 0 && grid > cap) grid = cap;
    kernel<<<static_cast<unsigned>(grid), kThreads, kSmem, s>>>(map, out, weight, bias, in.c, tiles_x, tiles_y, in.n,
                                                                 static_cast<int>(total), status);
    return cudaGetLastError();
}

}  // namespace ufb
