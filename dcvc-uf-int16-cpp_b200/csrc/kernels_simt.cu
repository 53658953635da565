// Memory-bound INT16 kernels: layout conversion between
// the reference's NCHW tensors and split NHWC, the direct (grouped / strided /
// depthwise) convolution, the elementwise operators of the reference's CUDA
// extension (src/cuda/elementwise.cu:16-46).
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

}  // namespace ufb
