// Shared definitions of the B200 INT16 engine.
//
// Activation layout in HBM ("split NHWC"): every pixel owns a row of
// 2 * pitch bytes -- the low bytes (u8) of its `pitch` channels followed by the
// high bytes (s8).  An int16 value v is lo + 256 * hi with lo = v & 0xff and
// hi = v >> 8.  The planes feed tcgen05 kind::i8 directly (TMA loads the u8
// tile and the s8 tile of the same pixels), and a view may select a channel
// slice (c_off) or a spatial crop of a larger buffer, which is how channel
// concatenation and cropping cost no copies.
#pragma once

#include <cstdint>

namespace ufb {

// Arithmetic contract "uf-int16-q9-w13-acc64-rna-sat-v1"
// (reference include/uf/int16_ops.hpp:10-13).
constexpr int kFeatureScale = 512;
constexpr int kWeightScale = 8192;

__host__ __device__ __forceinline__ int16_t sat16(int64_t v) {
    return static_cast<int16_t>(v < -32768 ? -32768 : (v > 32767 ? 32767 : v));
}

__host__ __device__ __forceinline__ int16_t sat16i(int32_t v) {
    return static_cast<int16_t>(v < -32768 ? -32768 : (v > 32767 ? 32767 : v));
}

// Round to nearest, ties away from zero, for a positive power-of-two divisor
// 2^shift (reference src/cuda/conv.cu:9-13 and src/int16_ops.cpp:48-56).
__device__ __forceinline__ int64_t rna_shift(int64_t v, int shift) {
    const int64_t s = v >> 63;  // 0 or -1
    const int64_t a = (v ^ s) - s;
    const int64_t q = (a + (int64_t(1) << (shift - 1))) >> shift;
    return (q ^ s) - s;
}

// rna for a positive divisor (reference src/cuda/elementwise.cu:146).
__host__ __device__ __forceinline__ int64_t rna_div(int64_t v, int64_t d) {
    return v < 0 ? -((-v + d / 2) / d) : (v + d / 2) / d;
}

// Split-NHWC activation view.
struct Act {
    uint8_t* base;       // byte address of (image 0, row 0, col 0, lo plane, channel 0 of the view)
    int n, h, w, c;      // view extents
    int pitch;           // channels per pixel row of the underlying buffer (row = 2 * pitch bytes)
    int row_px;          // pixels between consecutive rows of the underlying buffer
    long long img_px;    // pixels between consecutive images of the underlying buffer

    __host__ __device__ long long pixel(int img, int y, int x) const {
        return img * img_px + static_cast<long long>(y) * row_px + x;
    }
    __host__ __device__ uint8_t* lo(long long px) const { return base + px * 2 * pitch; }
    __host__ __device__ uint8_t* hi(long long px) const { return base + px * 2 * pitch + pitch; }
    __host__ __device__ bool dense() const { return row_px == w && img_px == static_cast<long long>(h) * w; }
    __host__ __device__ long long pixels() const { return static_cast<long long>(n) * h * w; }
};

__host__ __device__ inline Act make_act(uint8_t* buffer, int n, int h, int w, int c, int pitch, int c_off = 0) {
    Act a;
    a.base = buffer + c_off;
    a.n = n;
    a.h = h;
    a.w = w;
    a.c = c;
    a.pitch = pitch;
    a.row_px = w;
    a.img_px = static_cast<long long>(h) * w;
    return a;
}

__device__ __forceinline__ int16_t join16(uint8_t lo, uint8_t hi) {
    return static_cast<int16_t>(static_cast<uint16_t>(lo) | (static_cast<uint16_t>(hi) << 8));
}

// Epilogue applied to every convolution output value, in reference order
// (src/layers.cpp:91-104 and the module wrappers at :132-184):
//   v = sat(rna(sum / 8192) + bias)
//   v = lut[v]                       when lut            (int16::lookup)
//   v = sat(v + res1)                when res1.base      (int16::add)
//   v = sat(v + res2)                when res2.base      (int16::add, shortcut)
//   v = sat(rna(v * q[c] / 512))     when mulq           (int16::multiply)
// or, in wsilu4 mode, out[c] = sat(sum_{k<4} lut[v[4c + k]]) (int16::wsilu4).
// shuffle2 scatters output channel 4c + 2i + j of pixel (y, x) to channel c of
// pixel (2y + i, 2x + j) (pixel_shuffle(2) of the subpel/up modules).
struct Epilogue {
    const void* bias;    // int16 or int32 per output channel, or null
    int bias32;          // 1 when bias is int32
    const int16_t* lut;  // 65536-entry table applied after the bias (or wsilu4 table)
    int lut_start;       // lut_n > 0: entries [lut_start, lut_start + lut_n) hold every value
    int lut_n;           //   that is not lut[lut_start] (v below) or v itself (v > lut_hi),
    int lut_hi;          //   so kernels may stage just that window in shared memory
    int wsilu4;          // 1: reduce groups of four channels through lut
    int shuffle2;        // 1: pixel-shuffle(2) store
    Act res1, res2;      // residual inputs in output coordinates (base == null: none)
    const int16_t* mulq; // per-channel Q9 multiplier applied last, or null
};

}  // namespace ufb
