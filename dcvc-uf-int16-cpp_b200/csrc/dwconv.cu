// Depthwise 3x3, stride 1, zero padding 1 on split views (DepthConvBlock dc.2,
// src/layers.cpp:96; the reference runs it through its scalar `general`
// kernel, src/cuda/conv.cu:44-60).
//
// The kernel is bound by HBM: every input and output byte moves once, and the
// nine multiply-adds per value are cheap next to that.  Persistent CTAs walk
// output tiles of 128 channels x 16 columns x 8 rows.  Each tile's input window
// (18 x 10 pixels with the halo, both byte planes, 45 KB) arrives by TMA into
// one of two shared-memory buffers while the previous tile is computed from
// the other, so every SM keeps tens of KB of loads in flight; the halo outside
// the image is the TMA's zero fill, which is exactly the convolution's
// padding.  A thread owns four channels (one 32-bit word of each plane) of two
// adjacent output columns and slides down the tile's rows: each input row is
// read once from shared memory (a warp reads one 128-byte pixel line), joined
// back into int16 values and multiplied into the three output rows it feeds,
// one wide multiply-add per tap into an exact int64 sum (|S| < 2^34).
#include "kernels.h"

#include "conv_epi.cuh"
#include "conv_tc.h"
#include "umma.cuh"

#include <cuda.h>
#include <cuda_runtime.h>
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

struct DwAcc {
    int64_t s[kCols][4];  // [column][channel]: exact sum of x * w
};

__device__ __forceinline__ void dw_zero(DwAcc& a) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) a.s[j][c] = 0;
}

// Adds one input row (window columns 2t .. 2t + 3 as int16 values x) into the
// accumulator of an output row through weight row w[kx][channel].
__device__ __forceinline__ void dw_add(DwAcc& a, const int32_t (&x)[kCols + 2][4], const int32_t (&w)[3][4]) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx)
#pragma unroll
            for (int c = 0; c < 4; ++c) a.s[j][c] += static_cast<int64_t>(x[j + kx][c]) * w[kx][c];
}

// sat(rna(S / 8192) + bias) of two output columns, stored as one 32-bit word
// per plane (columns outside the image are skipped).
__device__ __forceinline__ void dw_store(const DwAcc& a, const int32_t (&b)[4], const Act& out, int img, int oy,
                                         int ox, int c0) {
#pragma unroll
    for (int j = 0; j < kCols; ++j) {
        if (ox + j >= out.w) break;
        int32_t r[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            // rna(S / 8192) = floor((S + 4096 - [S < 0]) / 8192)
            const int64_t S = a.s[j][c];
            r[c] = static_cast<int32_t>((S + 4096 + (S >> 63)) >> 13) + b[c];
        }
        const uint32_t p0 = pack2_sat(r[0], r[1]), p1 = pack2_sat(r[2], r[3]);
        const long long px = out.pixel(img, oy, ox + j);
        *reinterpret_cast<uint32_t*>(out.lo(px) + c0) = __byte_perm(p0, p1, 0x6420);
        *reinterpret_cast<uint32_t*>(out.hi(px) + c0) = __byte_perm(p0, p1, 0x7531);
    }
}

// Window row r, columns 2t .. 2t + 3, channels 4q .. 4q + 3 from the buffer.
__device__ __forceinline__ void dw_row(const uint8_t* buf, int r, int t, int q, int32_t (&x)[kCols + 2][4]) {
#pragma unroll
    for (int p = 0; p < kCols + 2; ++p) {
        const uint32_t off = (static_cast<uint32_t>(r) * kInW + kCols * t + p) * kLine + 4 * q;
        const uint32_t lw = *reinterpret_cast<const uint32_t*>(buf + off);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(buf + kPlane + off);
        uint32_t q0, q1;  // channels (0, 1) and (2, 3) as int16 pairs
        join_bytes(lw, hw, q0, q1);
        x[p][0] = lo16(q0);
        x[p][1] = hi16(q0);
        x[p][2] = lo16(q1);
        x[p][3] = hi16(q1);
    }
}

__global__ void __launch_bounds__(kThreads, 2)
dwconv3x3_tma_kernel(const __grid_constant__ CUtensorMap map, Act out, const int16_t* __restrict__ weight,
                     const int16_t* __restrict__ bias, int channels, int tiles_x, int tiles_y, int images,
                     int total_tiles, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    __shared__ __align__(8) uint64_t full[2];
    const int q = threadIdx.x % kQuads, t = threadIdx.x / kQuads;
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
        fence_mbar_init();
        prefetch_tmap(&map);
    }
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x < total_tiles) issue(blockIdx.x, 0);

    int32_t w[3][3][4], bv[4];
    int loaded_cb = -1;
    int i = 0;
    bool next_issued = false;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++i) {
        const int b = i & 1;
        // the other buffer was released by the barrier that ended the previous tile
        next_issued = tile + static_cast<int>(gridDim.x) < total_tiles;
        if (threadIdx.x == 0 && next_issued) issue(tile + gridDim.x, b ^ 1);
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
                for (int k = 0; k < 9; ++k) w[k / 3][k % 3][c] = ok ? weight[(c0 + c) * 9 + k] : 0;
                bv[c] = ok && bias ? bias[c0 + c] : 0;
            }
            loaded_cb = cb;
        }
        const bool ready = mbar_wait(&full[b], (i >> 1) & 1, status, 9);
        if (!__syncthreads_and(ready)) {
            // abort: the window load of the next tile must land before the CTA exits
            if (threadIdx.x == 0 && next_issued) mbar_wait(&full[b ^ 1], ((i + 1) >> 1) & 1, status, 10);
            break;
        }
        const uint8_t* buf = smem + b * kBuffer;
        const int oy0 = ty * kTileH, ox = tx * kTileW + kCols * t;
        const bool active = c0 < channels && ox < out.w;
        if (active) {
            // output rows r - 2, r - 1, r take window row r through weight rows 2, 1, 0
            DwAcc a0, a1, a2;
            dw_zero(a0);
            dw_zero(a1);
            dw_zero(a2);
            int32_t xv[kCols + 2][4];
            auto step = [&](DwAcc& next, DwAcc& mid, DwAcc& done, int wr) {
                dw_row(buf, wr, t, q, xv);
                dw_add(next, xv, w[0]);
                dw_add(mid, xv, w[1]);
                dw_add(done, xv, w[2]);
                if (wr >= 2 && oy0 + wr - 2 < out.h) dw_store(done, bv, out, img, oy0 + wr - 2, ox, c0);
                dw_zero(done);
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
        __syncthreads();  // every thread is done with this buffer before it is refilled
    }
}

}  // namespace

cudaError_t dwconv3x3(const Act& in, const Act& out, const int16_t* weight, const int16_t* bias, int* status,
                      cudaStream_t s) {
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
    // per device; always the same value, so concurrent callers cannot disagree
    const cudaError_t attr =
        cudaFuncSetAttribute(dwconv3x3_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
    if (attr != cudaSuccess) return attr;
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const long long grid = total < 2ll * sms ? total : 2ll * sms;
    dwconv3x3_tma_kernel<<<static_cast<unsigned>(grid), kThreads, kSmem, s>>>(
        map, out, weight, bias, in.c, tiles_x, tiles_y, in.n, static_cast<int>(total), status);
    return cudaGetLastError();
}

}  // namespace ufb
