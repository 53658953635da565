// Memory-bound INT16 kernels: layout conversion between
// the reference's NCHW tensors and split NHWC, the direct (grouped / strided /
// depthwise) convolution, the elementwise operators of the reference's CUDA
// extension (src/cuda/elementwise.cu:16-46) and the fixed-point warp.
#include "kernels.h"
#include "conv_epi.cuh"
#include "uf_common.cuh"

#include <cuda_runtime.h>

namespace ufb {

namespace {

constexpr int kBlock = 256;

inline unsigned blocks_for(long long n, int per_thread = 1) {
    const long long t = (n + per_thread - 1) / per_thread;
    return static_cast<unsigned>((t + kBlock - 1) / kBlock);
}

// NCHW int16 (n, c, h, w) -> split view of (n, h/f, w/f, c*f*f):
// out channel c*f*f + i*f + j of pixel (y, x) <- x[c, y*f + i, x*f + j]
// (pixel_unshuffle(f); f = 1 is a plain layout change).
__global__ void nchw_to_split_kernel(const int16_t* __restrict__ x, int n, int c, int h, int w, int f, Act out) {
    const int oh = h / f, ow = w / f, oc = c * f * f;
    const long long total = static_cast<long long>(n) * oc * oh * ow;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        // i enumerates the NCHW input so reads are coalesced
        const int xx = static_cast<int>(i % w);
        long long t = i / w;
        const int yy = static_cast<int>(t % h);
        t /= h;
        const int ch = static_cast<int>(t % c);
        const int b = static_cast<int>(t / c);
        const int16_t v = x[i];
        const int oy = yy / f, ox = xx / f;
        const int och = ch * f * f + (yy - oy * f) * f + (xx - ox * f);
        const long long px = out.pixel(b, oy, ox);
        out.lo(px)[och] = static_cast<uint8_t>(v & 0xff);
        out.hi(px)[och] = static_cast<uint8_t>((v >> 8) & 0xff);
    }
}

// split view (n, h, w, C) -> NCHW int16 (n, C/(f*f), h*f, w*f) (pixel_shuffle(f)).
__global__ void split_to_nchw_kernel(Act in, int f, int16_t* __restrict__ out) {
    const int oc = in.c / (f * f), oh = in.h * f, ow = in.w * f;
    const long long total = static_cast<long long>(in.n) * oc * oh * ow;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int xx = static_cast<int>(i % ow);
        long long t = i / ow;
        const int yy = static_cast<int>(t % oh);
        t /= oh;
        const int ch = static_cast<int>(t % oc);
        const int b = static_cast<int>(t / oc);
        const int y = yy / f, x = xx / f;
        const int ich = ch * f * f + (yy - y * f) * f + (xx - x * f);
        const long long px = in.pixel(b, y, x);
        out[i] = join16(in.lo(px)[ich], in.hi(px)[ich]);
    }
}

// Direct convolution with int64 accumulation, any stride / padding / groups
// (the reference's `general` kernel semantics, src/cuda/conv.cu:44-60).
__global__ void conv_direct_kernel(int16_t* __restrict__ out, const int16_t* __restrict__ x,
                                   const int16_t* __restrict__ weight, const void* bias, int bias32, long long count,
                                   int ci, int co, int h, int w, int oh, int ow, int kh, int kw, int sh, int sw,
                                   int ph, int pw, int groups) {
    for (long long index = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; index < count;
         index += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ox = static_cast<int>(index % ow);
        const int oy = static_cast<int>((index / ow) % oh);
        const int oc = static_cast<int>((index / (static_cast<long long>(ow) * oh)) % co);
        const long long b = index / (static_cast<long long>(ow) * oh * co);
        const int cg = ci / groups, first = (oc / (co / groups)) * cg;
        int64_t sum = 0;
        for (int c = 0; c < cg; ++c)
            for (int ky = 0; ky < kh; ++ky) {
                const int iy = oy * sh + ky - ph;
                if (iy < 0 || iy >= h) continue;
                for (int kx = 0; kx < kw; ++kx) {
                    const int ix = ox * sw + kx - pw;
                    if (ix < 0 || ix >= w) continue;
                    sum += static_cast<int64_t>(x[((b * ci + first + c) * h + iy) * w + ix]) *
                           weight[((static_cast<long long>(oc) * cg + c) * kh + ky) * kw + kx];
                }
            }
        int64_t v = rna_div(sum, kWeightScale);
        if (bias) v += bias32 ? static_cast<const int32_t*>(bias)[oc] : static_cast<const int16_t*>(bias)[oc];
        out[index] = sat16(v);
    }
}

// Depthwise 3x3, stride 1, zero padding 1 on split views (DepthConvBlock dc.2,
// src/layers.cpp:96; the reference runs it through its scalar `general`
// kernel, src/cuda/conv.cu:44-60).  A thread owns four channels (one 32-bit
// word of each byte plane) of kDwCols adjacent output columns and slides down a
// strip of rows: each input row is read once per thread (warp-coalesced
// 128-byte rows; neighbouring columns meet again in L1), its byte planes are
// joined back into int16 values, and it is multiplied into the three output
// rows it feeds with the 36 weights held in registers, one wide multiply-add
// per tap into an exact int64 sum (|S| < 2^34).  Two blocks of 256 threads per
// SM (128 registers) measured fastest: the kernel is latency-bound.
constexpr int kDwQuads = 32;     // channel quads per block (128 channels)
constexpr int kDwColThreads = 8; // threads along x per block
constexpr int kDwRows = 16;      // output rows per strip
constexpr int kDwThreads = kDwQuads * kDwColThreads;  // 256
constexpr int kDwCols = 2;       // output columns per thread (two blocks per SM: the best measured layout)

struct DwAcc {
    int64_t s[kDwCols][4];  // [column][channel]: exact sum of x * w
};

__device__ __forceinline__ void dw_zero(DwAcc& a) {
#pragma unroll
    for (int j = 0; j < kDwCols; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) a.s[j][c] = 0;
}

// Adds one input row (pixels x0-1 .. x0+kDwCols as int16 values x) into the
// accumulator of an output row through weight row w[kx][channel]: one wide
// multiply-add per tap (|x w| <= 2^30, nine taps need more than 32 bits).
__device__ __forceinline__ void dw_add(DwAcc& a, const int32_t (&x)[kDwCols + 2][4], const int32_t (&w)[3][4]) {
#pragma unroll
    for (int j = 0; j < kDwCols; ++j)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx)
#pragma unroll
            for (int c = 0; c < 4; ++c) a.s[j][c] += static_cast<int64_t>(x[j + kx][c]) * w[kx][c];
}

__device__ __forceinline__ void dw_store(const DwAcc& a, const int32_t (&b)[4], const Act& out, int img, int oy,
                                         int x0, int c0) {
#pragma unroll
    for (int j = 0; j < kDwCols; ++j) {
        if (x0 + j >= out.w) break;
        int32_t r[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            // rna(S / 8192) = floor((S + 4096 - [S < 0]) / 8192); |S| < 2^34
            const int64_t S = a.s[j][c];
            r[c] = static_cast<int32_t>((S + 4096 + (S >> 63)) >> 13) + b[c];
        }
        const uint32_t p0 = pack2_sat(r[0], r[1]), p1 = pack2_sat(r[2], r[3]);
        const long long px = out.pixel(img, oy, x0 + j);
        *reinterpret_cast<uint32_t*>(out.lo(px) + c0) = __byte_perm(p0, p1, 0x6420);
        *reinterpret_cast<uint32_t*>(out.hi(px) + c0) = __byte_perm(p0, p1, 0x7531);
    }
}

// Input row iy, pixels x0-1 .. x0+kDwCols, four channels, joined back into
// int16 values; zero outside the image.
__device__ __forceinline__ void dw_load_row(const Act& in, int img, int iy, int x0, int c0,
                                            int32_t (&x)[kDwCols + 2][4]) {
    const bool row_ok = iy >= 0 && iy < in.h;
#pragma unroll
    for (int p = 0; p < kDwCols + 2; ++p) {
        const int xx = x0 - 1 + p;
        uint32_t lw = 0, hw = 0;
        if (row_ok && xx >= 0 && xx < in.w) {
            const long long px = in.pixel(img, iy, xx);
            lw = __ldg(reinterpret_cast<const uint32_t*>(in.lo(px) + c0));
            hw = __ldg(reinterpret_cast<const uint32_t*>(in.hi(px) + c0));
        }
        uint32_t q0, q1;  // channels (0, 1) and (2, 3) as int16 pairs
        join_bytes(lw, hw, q0, q1);
        x[p][0] = lo16(q0);
        x[p][1] = hi16(q0);
        x[p][2] = lo16(q1);
        x[p][3] = hi16(q1);
    }
}

__global__ void __launch_bounds__(kDwThreads, 2)
dwconv3x3_kernel(Act in, Act out, const int16_t* __restrict__ weight, const int16_t* __restrict__ bias, int ch_blocks,
                 int col_blocks, int strips) {
    int bid = blockIdx.x;
    const int cb = bid % ch_blocks;
    bid /= ch_blocks;
    const int xb = bid % col_blocks;
    bid /= col_blocks;
    const int sb = bid % strips;
    const int img = bid / strips;
    const int c0 = cb * 4 * kDwQuads + 4 * (threadIdx.x % kDwQuads);
    const int x0 = kDwCols * (xb * kDwColThreads + static_cast<int>(threadIdx.x / kDwQuads));
    if (c0 >= in.c || x0 >= in.w) return;
    const int y0 = sb * kDwRows, y1 = y0 + kDwRows < in.h ? y0 + kDwRows : in.h;
    int32_t w[3][3][4], b[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int t = 0; t < 9; ++t) w[t / 3][t % 3][c] = weight[(c0 + c) * 9 + t];
        b[c] = bias ? bias[c0 + c] : 0;
    }
    // output rows iy + 1, iy, iy - 1 take input row iy through weight rows 0, 1, 2
    DwAcc a0, a1, a2;
    dw_zero(a0);
    dw_zero(a1);
    dw_zero(a2);
    int32_t xv[kDwCols + 2][4];
    auto step = [&](DwAcc& next, DwAcc& mid, DwAcc& done, int iy) {
        dw_load_row(in, img, iy, x0, c0, xv);
        dw_add(next, xv, w[0]);
        dw_add(mid, xv, w[1]);
        dw_add(done, xv, w[2]);
        if (iy - 1 >= y0) dw_store(done, b, out, img, iy - 1, x0, c0);
        dw_zero(done);
    };
    for (int iy = y0 - 1; iy <= y1; iy += 3) {
        step(a0, a1, a2, iy);
        if (iy + 1 > y1) break;
        step(a2, a0, a1, iy + 1);
        if (iy + 2 > y1) break;
        step(a1, a2, a0, iy + 2);
    }
}

// ---- elementwise on dense int16 tensors (reference src/cuda/elementwise.cu) ----

__global__ void add_kernel(int16_t* out, const int16_t* a, const int16_t* b, const int16_t* c, const int16_t* d,
                           long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        int32_t s = static_cast<int32_t>(a[i]) + b[i];
        if (c) s += c[i];
        if (d) s += d[i];
        out[i] = sat16i(s);
    }
}

__global__ void mul_kernel(int16_t* out, const int16_t* x, const int16_t* scale, long long n, int c, int h, int w,
                           int sb, int sc, int sh, int sw) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int iw = static_cast<int>(i % w), ih = static_cast<int>((i / w) % h);
        const int ic = static_cast<int>((i / (static_cast<long long>(w) * h)) % c);
        const long long ib = i / (static_cast<long long>(w) * h * c);
        const long long off = (((sb == 1 ? 0 : ib) * sc + (sc == 1 ? 0 : ic)) * sh + (sh == 1 ? 0 : ih)) * sw +
                              (sw == 1 ? 0 : iw);
        out[i] = sat16(rna_div(static_cast<int64_t>(x[i]) * scale[off], kFeatureScale));
    }
}

template <class T>
__global__ void lut_kernel(T* out, const int16_t* x, const T* lut, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = lut[static_cast<int32_t>(x[i]) + 32768];
}

__global__ void bytes_kernel(int16_t* out, const uint8_t* x, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        out[i] = static_cast<int16_t>(rna_div((2 * static_cast<int32_t>(x[i]) - 255) * kFeatureScale, 510));
}

__global__ void wsilu4_kernel(int16_t* out, const int16_t* x, const int16_t* lut, long long n, int channels,
                              long long hw) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pos = i % hw;
        const long long ch = (i / hw) % channels, batch = i / (hw * channels);
        const long long first = (batch * channels * 4 + ch * 4) * hw + pos;
        int32_t sum = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) sum += lut[static_cast<int32_t>(x[first + k * hw]) + 32768];
        out[i] = sat16i(sum);
    }
}

// Fixed-point backward bilinear warp (config-2 kernel; this repository's spec,
// no reference counterpart).  One thread per output pixel and channel group;
// neighbour fetches stay inside the 2x2 footprint of the displaced position.
__global__ void warp_kernel(int16_t* __restrict__ out, const int16_t* __restrict__ feature,
                            const int16_t* __restrict__ flow, int n, int c, int h, int w) {
    const long long total = static_cast<long long>(n) * h * w;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(i % w);
        const int y = static_cast<int>((i / w) % h);
        const long long b = i / (static_cast<long long>(w) * h);
        const long long plane = static_cast<long long>(h) * w;
        const int fx = flow[(b * 2 + 0) * plane + static_cast<long long>(y) * w + x];
        const int fy = flow[(b * 2 + 1) * plane + static_cast<long long>(y) * w + x];
        int px = x * 512 + fx, py = y * 512 + fy;
        px = px < 0 ? 0 : (px > (w - 1) * 512 ? (w - 1) * 512 : px);
        py = py < 0 ? 0 : (py > (h - 1) * 512 ? (h - 1) * 512 : py);
        const int x0 = px >> 9, y0 = py >> 9;
        const int x1 = x0 + 1 < w ? x0 + 1 : w - 1, y1 = y0 + 1 < h ? y0 + 1 : h - 1;
        const int ax = px & 511, ay = py & 511;
        const int64_t wa = static_cast<int64_t>(512 - ax) * (512 - ay), wb = static_cast<int64_t>(512 - ax) * ay;
        const int64_t wc = static_cast<int64_t>(ax) * (512 - ay), wd = static_cast<int64_t>(ax) * ay;
        const long long o00 = static_cast<long long>(y0) * w + x0, o10 = static_cast<long long>(y1) * w + x0;
        const long long o01 = static_cast<long long>(y0) * w + x1, o11 = static_cast<long long>(y1) * w + x1;
        const int16_t* f = feature + b * c * plane;
        int16_t* o = out + b * c * plane + static_cast<long long>(y) * w + x;
        for (int ch = 0; ch < c; ++ch) {
            const int16_t* p = f + ch * plane;
            const int64_t s = wa * __ldg(p + o00) + wb * __ldg(p + o10) + wc * __ldg(p + o01) + wd * __ldg(p + o11);
            o[ch * plane] = sat16(rna_div(s, 1 << 18));
        }
    }
}

unsigned grid_for(long long n) {
    const long long b = (n + kBlock - 1) / kBlock;
    const long long cap = 148ll * 16;
    return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

cudaError_t nchw_to_split(const int16_t* x, int n, int c, int h, int w, int f, const Act& out, cudaStream_t s) {
    nchw_to_split_kernel<<<grid_for(static_cast<long long>(n) * c * h * w), kBlock, 0, s>>>(x, n, c, h, w, f, out);
    return cudaGetLastError();
}

cudaError_t split_to_nchw(const Act& in, int f, int16_t* out, cudaStream_t s) {
    split_to_nchw_kernel<<<grid_for(in.pixels() * in.c), kBlock, 0, s>>>(in, f, out);
    return cudaGetLastError();
}

cudaError_t conv_direct(int16_t* out, const int16_t* x, const int16_t* weight, const void* bias, int bias32, int n,
                        int ci, int co, int h, int w, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                        int groups, cudaStream_t s) {
    const long long count = static_cast<long long>(n) * co * oh * ow;
    conv_direct_kernel<<<grid_for(count), kBlock, 0, s>>>(out, x, weight, bias, bias32, count, ci, co, h, w, oh, ow, kh,
                                                          kw, sh, sw, ph, pw, groups);
    return cudaGetLastError();
}

cudaError_t dwconv3x3(const Act& in, const Act& out, const int16_t* weight, const int16_t* bias, cudaStream_t s) {
    if (in.c % 4 || in.c != out.c || in.h != out.h || in.w != out.w || in.n != out.n || in.pitch % 16 ||
        out.pitch % 16 || reinterpret_cast<uintptr_t>(in.base) % 16 || reinterpret_cast<uintptr_t>(out.base) % 16)
        return cudaErrorInvalidValue;
    const int ch_blocks = (in.c + 4 * kDwQuads - 1) / (4 * kDwQuads);
    const int col_blocks = (in.w + kDwCols * kDwColThreads - 1) / (kDwCols * kDwColThreads);
    const int strips = (in.h + kDwRows - 1) / kDwRows;
    const long long blocks = static_cast<long long>(ch_blocks) * col_blocks * strips * in.n;
    if (blocks > INT32_MAX) return cudaErrorInvalidValue;
    dwconv3x3_kernel<<<static_cast<unsigned>(blocks), kDwThreads, 0, s>>>(in, out, weight, bias, ch_blocks,
                                                                          col_blocks, strips);
    return cudaGetLastError();
}

cudaError_t ew_add(int16_t* out, const int16_t* a, const int16_t* b, const int16_t* c, const int16_t* d, long long n,
                   cudaStream_t s) {
    add_kernel<<<grid_for(n), kBlock, 0, s>>>(out, a, b, c, d, n);
    return cudaGetLastError();
}

cudaError_t ew_mul(int16_t* out, const int16_t* x, const int16_t* scale, const long long* xs, const long long* ss,
                   cudaStream_t s) {
    const long long n = xs[0] * xs[1] * xs[2] * xs[3];
    mul_kernel<<<grid_for(n), kBlock, 0, s>>>(out, x, scale, n, static_cast<int>(xs[1]), static_cast<int>(xs[2]),
                                              static_cast<int>(xs[3]), static_cast<int>(ss[0]),
                                              static_cast<int>(ss[1]), static_cast<int>(ss[2]),
                                              static_cast<int>(ss[3]));
    return cudaGetLastError();
}

cudaError_t ew_lut16(int16_t* out, const int16_t* x, const int16_t* lut, long long n, cudaStream_t s) {
    lut_kernel<int16_t><<<grid_for(n), kBlock, 0, s>>>(out, x, lut, n);
    return cudaGetLastError();
}

cudaError_t ew_lut8(uint8_t* out, const int16_t* x, const uint8_t* lut, long long n, cudaStream_t s) {
    lut_kernel<uint8_t><<<grid_for(n), kBlock, 0, s>>>(out, x, lut, n);
    return cudaGetLastError();
}

cudaError_t ew_bytes(int16_t* out, const uint8_t* x, long long n, cudaStream_t s) {
    bytes_kernel<<<grid_for(n), kBlock, 0, s>>>(out, x, n);
    return cudaGetLastError();
}

cudaError_t ew_wsilu4(int16_t* out, const int16_t* x, const int16_t* lut, int n, int c4, long long hw,
                      cudaStream_t s) {
    const long long total = static_cast<long long>(n) * (c4 / 4) * hw;
    wsilu4_kernel<<<grid_for(total), kBlock, 0, s>>>(out, x, lut, total, c4 / 4, hw);
    return cudaGetLastError();
}

cudaError_t warp_fixed(int16_t* out, const int16_t* feature, const int16_t* flow, int n, int c, int h, int w,
                       cudaStream_t s) {
    warp_kernel<<<grid_for(static_cast<long long>(n) * h * w), kBlock, 0, s>>>(out, feature, flow, n, c, h, w);
    return cudaGetLastError();
}

}  // namespace ufb
