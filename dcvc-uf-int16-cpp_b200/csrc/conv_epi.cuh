// Epilogue arithmetic of the tensor-core convolution (conv_tc.cu):
// recombination of the three byte-product accumulators, the bias, saturation,
// byte-plane packing and the fused elementwise steps.
#pragma once

#include <cstdint>

#include "uf_common.cuh"

namespace ufb {

// rna(S / 8192), ties away from zero, of S = L + 256 X + 65536 H, in 32-bit
// arithmetic (reductions of at most 8192 terms of |x w| <= 2^30, so
// |S| <= 2^43 and every intermediate fits in int32).  S + 4096 = 8192 (8H + (X >> 5)) + U with
// U = L + 256 (X & 31) + 4096, so T = 8H + (X >> 5) + (U >> 13) is
// floor((S + 4096) / 8192): round half up.  It differs from rounding half
// away from zero only at an exact tie (U % 8192 == 0) with S < 0, i.e. T <= 0,
// where the result is T - 1.
__device__ __forceinline__ int32_t recombine32(int32_t L, int32_t X, int32_t H) {
    const int32_t U = L + ((X & 31) << 8) + 4096;
    const int32_t T = H * 8 + (X >> 5) + (U >> 13);
    return T - static_cast<int32_t>(((U & 8191) == 0) & (T <= 0));
}

__device__ __forceinline__ int32_t clamp16(int32_t v) { return min(max(v, -32768), 32767); }

// Bias as staged in shared memory: clamped to +-(2^30 + 2^16).  With
// |rna(S / 8192)| <= 2^30 the sum cannot overflow int32
// and saturates to the same int16 as with the unclamped bias.
__host__ __device__ __forceinline__ int32_t stage_bias(long long b) {
    constexpr long long kMax = (1ll << 30) + (1ll << 16);
    return static_cast<int32_t>(b < -kMax ? -kMax : (b > kMax ? kMax : b));
}

// (sat16(lo) | sat16(hi) << 16): two saturating narrowings and the packing in
// one instruction (PTX cvt.pack.sat puts its first source in the upper half).
__device__ __forceinline__ uint32_t pack2_sat(int32_t lo, int32_t hi) {
    uint32_t d;
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(d) : "r"(hi), "r"(lo));
    return d;
}

__device__ __forceinline__ uint32_t pack2(int32_t a, int32_t b) {
    return __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x5410);
}

__device__ __forceinline__ int32_t lo16(uint32_t p) { return static_cast<int16_t>(p & 0xffffu); }
__device__ __forceinline__ int32_t hi16(uint32_t p) { return static_cast<int32_t>(p) >> 16; }

// 16 packed int16 values (8 words) -> 16 low bytes + 16 high bytes.
__device__ __forceinline__ void split_bytes(const uint32_t (&p)[8], uint4& lo, uint4& hi) {
    lo.x = __byte_perm(p[0], p[1], 0x6420);
    lo.y = __byte_perm(p[2], p[3], 0x6420);
    lo.z = __byte_perm(p[4], p[5], 0x6420);
    lo.w = __byte_perm(p[6], p[7], 0x6420);
    hi.x = __byte_perm(p[0], p[1], 0x7531);
    hi.y = __byte_perm(p[2], p[3], 0x7531);
    hi.z = __byte_perm(p[4], p[5], 0x7531);
    hi.w = __byte_perm(p[6], p[7], 0x7531);
}

// 4 low bytes + 4 high bytes -> 2 packed words of int16 pairs.
__device__ __forceinline__ void join_bytes(uint32_t lo, uint32_t hi, uint32_t& p0, uint32_t& p1) {
    p0 = __byte_perm(lo, hi, 0x5140);
    p1 = __byte_perm(lo, hi, 0x7362);
}

// lut[sat16(v + start)] - start through a window of differences
// d[i] = lut[start + i] - (start + i), i in [0, last], of a table that is
// lut[start] below start and the identity above start + last (or whose window
// reaches 32767); cap = 32767 - start.  The two clamps of v do the int16
// saturation: below the window d[0] + 0 = lut[start] - start, inside it
// d[v] + v, above it d[last] + v = v - start (capped at 32767 - start).
__device__ __forceinline__ int32_t lut_window(const int16_t* d, int last, int cap, int32_t v) {
    int32_t i, c;
    asm("min.relu.s32 %0, %1, %2;" : "=r"(i) : "r"(v), "r"(last));
    asm("min.relu.s32 %0, %1, %2;" : "=r"(c) : "r"(v), "r"(cap));
    return d[i] + c;
}

// Fused elementwise step applied by the epilogue (compile-time, so each
// kernel instantiation is short straight-line code).
enum EpiMode : int { kEpiPlain = 0, kEpiLut = 1, kEpiRes = 2, kEpiWsilu4 = 3, kEpiShuffle2 = 4 };

// v = sat(v + res1) [then sat(v + res2)] for 16 packed outputs p of one pixel,
// output channels cbase .. cbase + n_valid - 1 (src/layers.cpp:98-104).
__device__ __forceinline__ void add_residuals(const Epilogue& e, uint32_t (&p)[8], int cbase, int n_valid,
                                              long long rpx1, long long rpx2) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const Act& res = r == 0 ? e.res1 : e.res2;
        if (r == 1 && !res.base) break;
        const long long rp = r == 0 ? rpx1 : rpx2;
        uint4 rl, rh;
        if (n_valid >= 16) {
            rl = *reinterpret_cast<const uint4*>(res.lo(rp) + cbase);
            rh = *reinterpret_cast<const uint4*>(res.hi(rp) + cbase);
        } else {
            uint32_t wl[4] = {0, 0, 0, 0}, wh[4] = {0, 0, 0, 0};
            for (int j = 0; j < n_valid; ++j) {
                wl[j >> 2] |= static_cast<uint32_t>(res.lo(rp)[cbase + j]) << (8 * (j & 3));
                wh[j >> 2] |= static_cast<uint32_t>(res.hi(rp)[cbase + j]) << (8 * (j & 3));
            }
            rl = make_uint4(wl[0], wl[1], wl[2], wl[3]);
            rh = make_uint4(wh[0], wh[1], wh[2], wh[3]);
        }
        const uint32_t lw[4] = {rl.x, rl.y, rl.z, rl.w}, hw[4] = {rh.x, rh.y, rh.z, rh.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t q0, q1;
            join_bytes(lw[k], hw[k], q0, q1);
            p[2 * k] = pack2(clamp16(lo16(p[2 * k]) + lo16(q0)), clamp16(hi16(p[2 * k]) + hi16(q0)));
            p[2 * k + 1] = pack2(clamp16(lo16(p[2 * k + 1]) + lo16(q1)), clamp16(hi16(p[2 * k + 1]) + hi16(q1)));
        }
    }
}

}  // namespace ufb
