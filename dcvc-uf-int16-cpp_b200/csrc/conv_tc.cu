// INT16 convolution as an implicit GEMM on the sm_100a tensor cores.
//
// Replaces the reference's mma.sync kernel uf_mma_conv
// (src/cuda/int16_mma.cuh:40-109, dispatched from src/cuda/conv.cu:62-127) with
// the same exact arithmetic (src/cuda/conv.cu:9-13):
//     out = sat(rna(sum_k x_k * w_k / 8192) + bias)
//
// Operands are split into bytes, x = xl + 256 xh (xl u8, xh s8) and
// w = wl + 256 wh, and the products accumulate exactly in three s32 TMEM
// accumulators LL = sum xl wl, X = sum (xh wl + xl wh), HH = sum xh wh, which
// the epilogue recombines as LL + 256 X + 65536 HH.  Two weight splits:
//   unsigned (any weights): wl u8, wh s8 -- four N=128 MMAs per K step;
//   signed (w <= 32639):    wl s8, wh s8 -- the weight tile stacks its 128
//     low rows over its 128 high rows, so one N=256 MMA A_lo x [wl; wh]
//     yields [LL | xl wh] and one N=256 MMA A_hi x [wl; wh], written 128
//     columns further on, adds xh wl onto X and yields HH: two MMAs per step.
// For K <= 32768 every partial sum fits s32 (|X| <= 383 * 128 * K).
//
// GEMM orientation: M = 128 output pixels (TMEM lanes), N = 128 output
// channels per tile, K = taps x input channels.  Activations are split NHWC in
// HBM, so both operands are K-major and arrive by TMA as 128-byte swizzled
// tiles; 3x3 taps are spatially shifted TMA boxes over a 5-D tensor map whose
// zero fill is the convolution's zero padding.
//
// Persistent CTAs (one per SM) walk the output tiles.  Warp 0 issues TMA into a
// 3-stage ring that runs ahead across tiles, warp 1 owns TMEM and issues the
// MMAs, warps 2-9 run the epilogue in two phases: phase 1 reads the three
// accumulators, rounds, adds the bias and saturates into registers, then
// releases TMEM so the next tile's MMAs start; phase 2 applies the fused
// elementwise steps (LUT, residual adds, QP multiply, WSiLU4, pixel shuffle)
// and stores while those MMAs run.
#include "umma.cuh"
#include "uf_common.cuh"
#include "conv_tc.h"

#include <cuda_runtime.h>
#include <mutex>
#include <string>
#include <vector>

namespace ufb {

namespace {

constexpr int kBM = 128;                                    // output pixels per tile
constexpr int kBK = 128;                                    // input channels per K block
constexpr int kEpiWarps = 16;                               // four per TMEM lane quarter
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kABytes = kBM * kBK;                     // one activation plane tile
constexpr uint32_t kTmemCols = 512;

// Tile shape per output-channel width BN:
//   BN = 128: one accumulator set LL [0,128) X [128,256) HH [256,384), 3 x 64 KB ring
//   BN = 64:  two accumulator sets (at columns 0 and 256) so the epilogue of one
//             tile overlaps the MMAs of the next, 4 x 48 KB ring
template <int BN>
struct Tile {
    static constexpr uint32_t kBBytes = 2 * BN * kBK;       // stacked low / high weight rows
    static constexpr uint32_t kStageBytes = 2 * kABytes + kBBytes;
    static constexpr int kStages = BN == 128 ? 3 : 4;
    static constexpr int kBuffers = BN == 128 ? 1 : 2;
    static constexpr uint32_t kBufferStride = 256;          // TMEM columns between accumulator sets
    static constexpr size_t kRingBytes = size_t(kStages) * kStageBytes + 1024;
    static constexpr int kCols = BN / 4;                    // accumulator columns per epilogue warp
};

// Fused elementwise step applied by the epilogue (compile-time, so each
// instantiation is short straight-line code).
enum EpiMode : int { kEpiPlain = 0, kEpiLut = 1, kEpiRes = 2, kEpiWsilu4 = 3, kEpiShuffle2 = 4 };

struct ConvTcArgs {
    Act out;
    Epilogue epi;
    int co, ci, taps_h, taps_w, pad_h, pad_w, cpad;
    int oh, ow;
    int tile_w, tile_h, tiles_x, tiles_y;
    long long m_total;  // flat mode: output pixels
    int n_tiles, total_tiles;
    int signed_split;
    int wide;           // K >= 16384: int64 recombination
    int* status;
};

struct TileCoord {
    int img, y0, x0, co0;
    long long p0;
};

template <bool SPATIAL, int BN>
__device__ __forceinline__ TileCoord tile_coord(const ConvTcArgs& a, int tile) {
    TileCoord t{};
    const int m = tile / a.n_tiles;
    t.co0 = (tile - m * a.n_tiles) * BN;
    if (SPATIAL) {
        int r = m;
        const int tx = r % a.tiles_x;
        r /= a.tiles_x;
        const int ty = r % a.tiles_y;
        t.img = r / a.tiles_y;
        t.x0 = tx * a.tile_w;
        t.y0 = ty * a.tile_h;
    } else {
        t.p0 = static_cast<long long>(m) * kBM;
    }
    return t;
}

// rna(S / 8192) of S = L + 256 X + 65536 H without 64-bit arithmetic (valid
// for K < 16384, where 8 |H| < 2^31): S = 8192 T + Rl with 0 <= Rl < 8192, and
// round-half-away gives T + (Rl > 4096 || (Rl == 4096 && T >= 0)).
__device__ __forceinline__ int32_t recombine32(int32_t L, int32_t X, int32_t H) {
    const int32_t R = ((X & 31) << 8) + (L & 8191);
    const int32_t T = H * 8 + (X >> 5) + (L >> 13) + (R >> 13);
    const int32_t Rl = R & 8191;
    return T + ((Rl > 4096) | ((Rl == 4096) & (T >= 0)));
}

__device__ __forceinline__ int64_t recombine64(int32_t L, int32_t X, int32_t H) {
    return rna_shift(static_cast<int64_t>(L) + 256 * static_cast<int64_t>(X) + 65536 * static_cast<int64_t>(H), 13);
}

__device__ __forceinline__ int32_t clamp16(int32_t v) { return v < -32768 ? -32768 : (v > 32767 ? 32767 : v); }

__device__ __forceinline__ uint32_t pack2(int32_t a, int32_t b) {
    return (static_cast<uint32_t>(a) & 0xffffu) | (static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ int32_t lo16(uint32_t p) { return static_cast<int16_t>(p & 0xffffu); }
__device__ __forceinline__ int32_t hi16(uint32_t p) { return static_cast<int16_t>(p >> 16); }

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

// Phase 2 of 16 conv outputs (packed pairs p) of one pixel, output channels
// cbase .. cbase + 15, in the order of src/layers.cpp:91-104.
template <int MODE>
__device__ __forceinline__ void finish16(const ConvTcArgs& a, uint32_t (&p)[8], int cbase, int n_valid,
                                         long long opx, long long rpx1, long long rpx2, const Act& out) {
    const Epilogue& e = a.epi;
    if (MODE == kEpiLut) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            p[i] = pack2(__ldg(&e.lut[lo16(p[i]) + 32768]), __ldg(&e.lut[hi16(p[i]) + 32768]));
    }
    if (MODE == kEpiRes) {
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
                uint8_t bl[16], bh[16];
                for (int j = 0; j < 16; ++j) {
                    bl[j] = j < n_valid ? res.lo(rp)[cbase + j] : 0;
                    bh[j] = j < n_valid ? res.hi(rp)[cbase + j] : 0;
                }
                rl = *reinterpret_cast<const uint4*>(bl);
                rh = *reinterpret_cast<const uint4*>(bh);
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
    if (MODE == kEpiWsilu4) {
        // out[c] = sat(sum_{k<4} lut[v[4c + k]]): four output channels cbase / 4 ..
        int32_t r[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int32_t s = __ldg(&e.lut[lo16(p[2 * g]) + 32768]) + __ldg(&e.lut[hi16(p[2 * g]) + 32768]) +
                              __ldg(&e.lut[lo16(p[2 * g + 1]) + 32768]) + __ldg(&e.lut[hi16(p[2 * g + 1]) + 32768]);
            r[g] = clamp16(s);
        }
        const uint32_t w0 = pack2(r[0], r[1]), w1 = pack2(r[2], r[3]);
        uint8_t* dl = out.lo(opx) + (cbase >> 2);
        uint8_t* dh = out.hi(opx) + (cbase >> 2);
        if (n_valid >= 16) {
            *reinterpret_cast<uint32_t*>(dl) = __byte_perm(w0, w1, 0x6420);
            *reinterpret_cast<uint32_t*>(dh) = __byte_perm(w0, w1, 0x7531);
        } else {
            for (int g = 0; g < 4 && 4 * g < n_valid; ++g) {
                dl[g] = static_cast<uint8_t>(r[g] & 0xff);
                dh[g] = static_cast<uint8_t>((r[g] >> 8) & 0xff);
            }
        }
        return;
    }
    if (MODE == kEpiShuffle2) return;  // stored by the caller, which knows the four target pixels
    uint4 lo, hi;
    split_bytes(p, lo, hi);
    uint8_t* dl = out.lo(opx) + cbase;
    uint8_t* dh = out.hi(opx) + cbase;
    if (n_valid >= 16) {
        *reinterpret_cast<uint4*>(dl) = lo;
        *reinterpret_cast<uint4*>(dh) = hi;
    } else {
        const uint8_t* bl = reinterpret_cast<const uint8_t*>(&lo);
        const uint8_t* bh = reinterpret_cast<const uint8_t*>(&hi);
        for (int j = 0; j < n_valid; ++j) {
            dl[j] = bl[j];
            dh[j] = bh[j];
        }
    }
}

// pixel_shuffle(2) store: channel 4c + 2i + j of pixel (oy, ox) -> channel c
// of pixel (2 oy + i, 2 ox + j).
__device__ __forceinline__ void store_shuffle2(const Act& out, const uint32_t (&p)[8], int cbase, int n_valid,
                                               int img, int oy, int ox) {
    const int c0 = cbase >> 2;
    int32_t v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = lo16(p[i]);
        v[2 * i + 1] = hi16(p[i]);
    }
#pragma unroll
    for (int ij = 0; ij < 4; ++ij) {
        const long long opx = out.pixel(img, 2 * oy + (ij >> 1), 2 * ox + (ij & 1));
        uint8_t* dl = out.lo(opx) + c0;
        uint8_t* dh = out.hi(opx) + c0;
        if (n_valid >= 16) {
            const uint32_t w0 = pack2(v[ij], v[4 + ij]), w1 = pack2(v[8 + ij], v[12 + ij]);
            *reinterpret_cast<uint32_t*>(dl) = __byte_perm(w0, w1, 0x6420);
            *reinterpret_cast<uint32_t*>(dh) = __byte_perm(w0, w1, 0x7531);
        } else {
            for (int g = 0; g < 4 && 4 * g + ij < n_valid; ++g) {
                dl[g] = static_cast<uint8_t>(v[4 * g + ij] & 0xff);
                dh[g] = static_cast<uint8_t>((v[4 * g + ij] >> 8) & 0xff);
            }
        }
    }
}

template <bool SPATIAL, int MODE, int BN>
__global__ void __launch_bounds__(kThreads, 1)
conv_i16_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const ConvTcArgs args) {
    using T = Tile<BN>;
    constexpr int S = T::kStages;
    constexpr int NB = T::kBuffers;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int32_t* bias_s = reinterpret_cast<int32_t*>(smem + size_t(S) * T::kStageBytes);  // [n_tiles * BN]
    __shared__ __align__(8) uint64_t full_bar[S];
    __shared__ __align__(8) uint64_t empty_bar[S];
    __shared__ __align__(8) uint64_t tmem_full[NB];
    __shared__ __align__(8) uint64_t tmem_empty[NB];
    __shared__ uint32_t tmem_holder;
    __shared__ int consumed;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_per_tap = (args.ci + kBK - 1) / kBK;
    const int num_k = args.taps_h * args.taps_w * kb_per_tap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < NB; ++b) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], kEpiWarps);
        }
        consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    // the whole bias vector, zero padded to the tile grid, once per CTA
    for (int i = threadIdx.x; i < args.n_tiles * BN; i += kThreads) {
        int32_t b = 0;
        if (args.epi.bias && i < args.co)
            b = args.epi.bias32 ? static_cast<const int32_t*>(args.epi.bias)[i]
                                : static_cast<const int16_t*>(args.epi.bias)[i];
        bias_s[i] = b;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_holder;

    int issued = 0;
    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&mapA);
            prefetch_tmap(&mapB);
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x) {
                const TileCoord tc = tile_coord<SPATIAL, BN>(args, tile);
                for (int k = 0; k < num_k; ++k, ++it) {
                    const int s = it % S;
                    const uint32_t round = it / S;
                    if (it >= S && !mbar_wait(&empty_bar[s], (round - 1) & 1, args.status, 1)) {
                        ok = false;
                        break;
                    }
                    const int tap = k / kb_per_tap, cb = k - tap * kb_per_tap;
                    const int ky = tap / args.taps_w, kx = tap - ky * args.taps_w;
                    uint8_t* st = smem + size_t(s) * T::kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[s], T::kStageBytes);
                    const int c0 = cb * kBK;
                    if (SPATIAL) {
                        const int ix = tc.x0 + kx - args.pad_w, iy = tc.y0 + ky - args.pad_h;
                        tma_load_5d(st, &mapA, &full_bar[s], c0, 0, ix, iy, tc.img);
                        tma_load_5d(st + kABytes, &mapA, &full_bar[s], c0, 1, ix, iy, tc.img);
                    } else {
                        tma_load_3d(st, &mapA, &full_bar[s], c0, 0, static_cast<int>(tc.p0));
                        tma_load_3d(st + kABytes, &mapA, &full_bar[s], c0, 1, static_cast<int>(tc.p0));
                    }
                    tma_load_2d(st + 2 * kABytes, &mapB, &full_bar[s], tap * args.cpad + c0, (tc.co0 / BN) * 2 * BN);
                    issued = it + 1;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t i_uu = i8_idesc(kBM, BN, false, false);
            constexpr uint32_t i_su = i8_idesc(kBM, BN, true, false);
            constexpr uint32_t i_us = i8_idesc(kBM, BN, false, true);
            constexpr uint32_t i_ss = i8_idesc(kBM, BN, true, true);
            constexpr uint32_t i_us2 = i8_idesc(kBM, 2 * BN, false, true);
            constexpr uint32_t i_ss2 = i8_idesc(kBM, 2 * BN, true, true);
            int it = 0, ti = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x, ++ti) {
                const int buf = ti % NB, use = ti / NB;
                if (use > 0 && !mbar_wait(&tmem_empty[buf], (use - 1) & 1, args.status, 3)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_ll = tmem + buf * T::kBufferStride, d_x = d_ll + BN, d_hh = d_ll + 2 * BN;
                for (int k = 0; k < num_k; ++k, ++it) {
                    const int s = it % S;
                    const uint32_t round = it / S;
                    if (!mbar_wait(&full_bar[s], round & 1, args.status, 2)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_u32(smem + size_t(s) * T::kStageBytes);
                    const uint32_t a_lo = base, a_hi = base + kABytes, b_lo = base + 2 * kABytes,
                                   b_hi = b_lo + BN * kBK;
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk) {
                        const uint32_t o = kk * 32;
                        const bool first = k == 0 && kk == 0;
                        if (args.signed_split) {
                            mma_i8(d_ll, sw128_desc(a_lo + o), sw128_desc(b_lo + o), i_us2, first ? 0u : 1u);
                            if (first) {
                                mma_i8(d_x, sw128_desc(a_hi + o), sw128_desc(b_lo + o), i_ss, 1u);
                                mma_i8(d_hh, sw128_desc(a_hi + o), sw128_desc(b_hi + o), i_ss, 0u);
                            } else {
                                mma_i8(d_x, sw128_desc(a_hi + o), sw128_desc(b_lo + o), i_ss2, 1u);
                            }
                        } else {
                            const uint32_t acc = first ? 0u : 1u;
                            mma_i8(d_ll, sw128_desc(a_lo + o), sw128_desc(b_lo + o), i_uu, acc);
                            mma_i8(d_x, sw128_desc(a_hi + o), sw128_desc(b_lo + o), i_su, acc);
                            mma_i8(d_x, sw128_desc(a_lo + o), sw128_desc(b_hi + o), i_us, 1u);
                            mma_i8(d_hh, sw128_desc(a_hi + o), sw128_desc(b_hi + o), i_ss, acc);
                        }
                    }
                    mma_commit(&empty_bar[s]);
                }
                if (!ok) break;
                mma_commit(&tmem_full[buf]);
            }
            consumed = it;
        }
        __syncwarp();
    } else {
        constexpr int kC = T::kCols;                   // 32 (BN 128) or 16 (BN 64)
        const int quarter = warp & 3;
        const int cgroup = (warp - 2) >> 2;            // columns [kC * cgroup, kC * cgroup + kC)
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const Act& out = args.out;
        int ti = 0;
        for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x, ++ti) {
            const int buf = ti % NB, use = ti / NB;
            const TileCoord tc = tile_coord<SPATIAL, BN>(args, tile);
            bool valid;
            long long opx = 0, rpx1 = 0, rpx2 = 0;
            int oy = 0, ox = 0;
            if (SPATIAL) {
                const int ty = row / args.tile_w, tx = row - ty * args.tile_w;
                oy = tc.y0 + ty;
                ox = tc.x0 + tx;
                valid = oy < args.oh && ox < args.ow;
                if (MODE != kEpiShuffle2) opx = out.pixel(tc.img, oy, ox);
                if (MODE == kEpiRes) {
                    rpx1 = args.epi.res1.pixel(tc.img, oy, ox);
                    rpx2 = args.epi.res2.pixel(tc.img, oy, ox);
                }
            } else {
                opx = rpx1 = rpx2 = tc.p0 + row;
                valid = opx < args.m_total;
            }
            if (!mbar_wait(&tmem_full[buf], use & 1, args.status, 4)) break;
            tc_fence_after();
            const uint32_t acc_addr = lane_addr + buf * T::kBufferStride;
            // phase 1: accumulators -> sat(rna(sum / 8192) + bias), 16 columns at a time
            uint32_t packed[kC / 2];
#pragma unroll
            for (int c = 0; c < kC / 16; ++c) {
                const int col = cgroup * kC + c * 16;
                uint32_t ll[16], xx[16], hh[16];
                tmem_ld16(acc_addr + col, ll);
                tmem_ld16(acc_addr + BN + col, xx);
                tmem_ld16(acc_addr + 2 * BN + col, hh);
                const int4* bq = reinterpret_cast<const int4*>(bias_s + tc.co0 + col);
                const int4 b4[4] = {bq[0], bq[1], bq[2], bq[3]};
                const int32_t* bias = reinterpret_cast<const int32_t*>(b4);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    int32_t r[2];
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
                        const int32_t L = static_cast<int32_t>(ll[j + t]), X = static_cast<int32_t>(xx[j + t]),
                                      H = static_cast<int32_t>(hh[j + t]);
                        if (args.wide) {
                            const int64_t v = recombine64(L, X, H) + bias[j + t];
                            r[t] = v < -32768 ? -32768 : (v > 32767 ? 32767 : static_cast<int32_t>(v));
                        } else {
                            const int64_t v = static_cast<int64_t>(recombine32(L, X, H)) + bias[j + t];
                            r[t] = v < -32768 ? -32768 : (v > 32767 ? 32767 : static_cast<int32_t>(v));
                        }
                    }
                    packed[c * 8 + j / 2] = pack2(r[0], r[1]);
                }
            }
            // this accumulator set is free for the MMAs of the tile after next
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[buf]);
            // phase 2: fused elementwise steps and stores, overlapped with MMAs
            if (valid) {
#pragma unroll
                for (int c = 0; c < kC / 16; ++c) {
                    const int cbase = tc.co0 + cgroup * kC + c * 16;
                    if (cbase >= args.co) break;
                    const int n_valid = args.co - cbase < 16 ? args.co - cbase : 16;
                    uint32_t p8[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) p8[i] = packed[c * 8 + i];
                    if (MODE == kEpiShuffle2)
                        store_shuffle2(out, p8, cbase, n_valid, tc.img, oy, ox);
                    else
                        finish16<MODE>(args, p8, cbase, n_valid, opx, rpx1, rpx2, out);
                }
            }
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // abort path only: wait for TMA loads issued but never consumed, so no
        // copy into this CTA's shared memory outlives the CTA
        for (int k = consumed; k < issued; ++k) mbar_wait(&full_bar[k % S], (k / S) & 1, args.status, 5);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// [co_tiles][2][bn][kpad]: tile rows 0..bn-1 low bytes, bn..2bn-1 high bytes.
__global__ void prep_tc_weights_kernel(const int16_t* __restrict__ w, int co, int ci, int kh, int kw, int cpad,
                                       int kpad, int co_tiles, int bn, int signed_split, uint8_t* __restrict__ planes) {
    const long long total = static_cast<long long>(co_tiles) * 2 * bn * kpad;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(i % kpad);
        const long long rowg = i / kpad;  // tile * 2bn + r
        const int r = static_cast<int>(rowg % (2 * bn));
        const int tile = static_cast<int>(rowg / (2 * bn));
        const int plane = r / bn;
        const int o = tile * bn + (r - plane * bn);
        const int tap = k / cpad, c = k - tap * cpad;
        int32_t v = 0;
        if (o < co && c < ci) {
            const int ky = tap / kw, kx = tap - ky * kw;
            v = w[((static_cast<long long>(o) * ci + c) * kh + ky) * kw + kx];
        }
        int32_t lo, hi;
        if (signed_split) {
            lo = ((v + 128) & 255) - 128;
            hi = (v - lo) >> 8;
        } else {
            lo = v & 255;
            hi = v >> 8;
        }
        planes[i] = static_cast<uint8_t>((plane ? hi : lo) & 0xff);
    }
}

// ------------------------------------------------------------------ host ----

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    return fn;
}

bool encode(CUtensorMap* map, void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
            const cuuint32_t* box, std::string& err) {
    auto fn = encode_fn();
    if (!fn) {
        err = "cuTensorMapEncodeTiled is unavailable";
        return false;
    }
    cuuint32_t elem[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, base, dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        err = "cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r));
        return false;
    }
    return true;
}

std::mutex g_dev_mutex;
std::vector<int> g_sms;

int sm_count(int device) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (static_cast<size_t>(device) >= g_sms.size()) g_sms.resize(device + 1, 0);
    if (!g_sms[device]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) == cudaSuccess) g_sms[device] = n;
    }
    return g_sms[device] > 0 ? g_sms[device] : 148;
}

template <bool SPATIAL, int MODE, int BN>
cudaError_t launch_mode(const CUtensorMap& a, const CUtensorMap& b, const ConvTcArgs& args, cudaStream_t stream) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    const size_t smem = Tile<BN>::kRingBytes + size_t(args.n_tiles) * BN * sizeof(int32_t);
    // the attribute is per function and device; setting it each launch is cheap
    e = cudaFuncSetAttribute(conv_i16_tc_kernel<SPATIAL, MODE, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int sms = sm_count(device);
    const int grid = args.total_tiles < sms ? args.total_tiles : sms;
    conv_i16_tc_kernel<SPATIAL, MODE, BN><<<grid, kThreads, smem, stream>>>(a, b, args);
    return cudaGetLastError();
}

template <bool SPATIAL, int BN>
cudaError_t launch_bn(const CUtensorMap& a, const CUtensorMap& b, const ConvTcArgs& args, cudaStream_t stream) {
    const Epilogue& e = args.epi;
    if (e.shuffle2) return launch_mode<SPATIAL, kEpiShuffle2, BN>(a, b, args, stream);
    if (e.wsilu4) return launch_mode<SPATIAL, kEpiWsilu4, BN>(a, b, args, stream);
    if (e.lut) return launch_mode<SPATIAL, kEpiLut, BN>(a, b, args, stream);
    if (e.res1.base) return launch_mode<SPATIAL, kEpiRes, BN>(a, b, args, stream);
    return launch_mode<SPATIAL, kEpiPlain, BN>(a, b, args, stream);
}

template <bool SPATIAL>
cudaError_t launch(const CUtensorMap& a, const CUtensorMap& b, const ConvTcArgs& args, int bn, cudaStream_t stream) {
    return bn == 64 ? launch_bn<SPATIAL, 64>(a, b, args, stream) : launch_bn<SPATIAL, 128>(a, b, args, stream);
}

}  // namespace

size_t tc_weight_bytes(int co, int ci, int kh, int kw, int bn) {
    const int cpad = (ci + kBK - 1) / kBK * kBK;
    const int co_tiles = (co + bn - 1) / bn;
    return static_cast<size_t>(co_tiles) * 2 * bn * kh * kw * cpad;
}

int tc_choose_bn(int ci, int kh, int kw, bool signed_split) {
    // reductions of up to 512 are dominated by the per-tile epilogue: the
    // 64-wide tile double-buffers TMEM so the epilogue overlaps the MMAs; the
    // signed split keeps its MMAs 128 wide (full rate)
    return signed_split && static_cast<long long>(ci) * kh * kw <= 512 ? 64 : 128;
}

bool tc_signed_split_ok(const int16_t* weight_host, size_t count) {
    for (size_t i = 0; i < count; ++i)
        if (weight_host[i] > 32639) return false;
    return true;
}

bool tc_describe(TcWeights& w, int co, int ci, int kh, int kw, bool signed_split, int bn, uint8_t* planes,
                 std::string& err) {
    if (bn != 64 && bn != 128) {
        err = "tile width must be 64 or 128";
        return false;
    }
    w.bn = bn;
    w.co = co;
    w.ci = ci;
    w.kh = kh;
    w.kw = kw;
    w.cpad = (ci + kBK - 1) / kBK * kBK;
    w.kpad = kh * kw * w.cpad;
    w.co_tiles = (co + bn - 1) / bn;
    w.signed_split = signed_split;
    w.planes = planes;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w.kpad), static_cast<cuuint64_t>(w.co_tiles) * 2 * bn};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w.kpad)};
    const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(2 * bn)};
    return encode(&w.map, planes, 2, dims, strides, box, err);
}

bool tc_prepare(TcWeights& w, const int16_t* weight, int co, int ci, int kh, int kw, bool signed_split, int bn,
                uint8_t* planes, cudaStream_t s, std::string& err) {
    if (!tc_describe(w, co, ci, kh, kw, signed_split, bn, planes, err)) return false;
    const long long total = static_cast<long long>(w.co_tiles) * 2 * bn * w.kpad;
    const long long blocks = (total + 255) / 256;
    prep_tc_weights_kernel<<<static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(
        weight, co, ci, kh, kw, w.cpad, w.kpad, w.co_tiles, bn, signed_split ? 1 : 0, planes);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        err = std::string("weight preparation: ") + cudaGetErrorString(e);
        return false;
    }
    return true;
}

int conv_tc_run(const TcWeights& w, const Act& in, const Act& out, const Epilogue& epi, int pad_h, int pad_w,
                cudaStream_t stream, int* status, std::string& err) {
    const int oh = in.h + 2 * pad_h - w.kh + 1, ow = in.w + 2 * pad_w - w.kw + 1;
    if (oh <= 0 || ow <= 0) {
        err = "kernel exceeds input";
        return -1;
    }
    if (in.c != w.ci) {
        err = "input channels do not match weights";
        return -1;
    }
    if ((in.pitch % 16) || (reinterpret_cast<uintptr_t>(in.base) % 16) || (out.pitch % 16) ||
        (reinterpret_cast<uintptr_t>(out.base) % 16)) {
        err = "split activations need 16-byte aligned pitch and channel offset";
        return -1;
    }
    for (const Act* r : {&epi.res1, &epi.res2}) {
        if (r->base && ((r->pitch % 16) || (reinterpret_cast<uintptr_t>(r->base) % 16))) {
            err = "residual views need 16-byte aligned pitch and channel offset";
            return -1;
        }
    }
    const int modes = (epi.shuffle2 ? 1 : 0) + (epi.wsilu4 ? 1 : 0) + (epi.lut && !epi.wsilu4 ? 1 : 0) +
                      (epi.res1.base ? 1 : 0);
    if (modes > 1 || epi.mulq || (epi.res2.base && !epi.res1.base)) {
        err = "unsupported epilogue combination (one of lut, residual adds, wsilu4, pixel shuffle; no multiply)";
        return -1;
    }
    const size_t ring = w.bn == 64 ? Tile<64>::kRingBytes : Tile<128>::kRingBytes;
    if (w.co_tiles * w.bn * sizeof(int32_t) + ring > 227 * 1024) {
        err = "too many output channels for the staged bias";
        return -1;
    }
    const long long k_total = static_cast<long long>(w.kh) * w.kw * w.ci;
    if (k_total > 32768) {
        err = "reduction exceeds the exact s32 accumulator bound";
        return -1;
    }
    const bool flat = w.kh == 1 && w.kw == 1 && pad_h == 0 && pad_w == 0 && in.dense() && out.dense() &&
                      !epi.shuffle2 && (!epi.res1.base || epi.res1.dense()) && (!epi.res2.base || epi.res2.dense()) &&
                      in.pixels() < (1ll << 31);
    ConvTcArgs args{};
    args.out = out;
    args.epi = epi;
    args.co = w.co;
    args.ci = w.ci;
    args.taps_h = w.kh;
    args.taps_w = w.kw;
    args.pad_h = pad_h;
    args.pad_w = pad_w;
    args.cpad = w.cpad;
    args.oh = oh;
    args.ow = ow;
    args.signed_split = w.signed_split ? 1 : 0;
    args.wide = k_total >= 16384 ? 1 : 0;
    args.status = status;
    args.n_tiles = w.co_tiles;
    CUtensorMap amap;
    long long m_tiles;
    if (flat) {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(in.c), 2, static_cast<cuuint64_t>(in.pixels())};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(in.pitch), static_cast<cuuint64_t>(2 * in.pitch)};
        const cuuint32_t box[3] = {kBK, 1, kBM};
        if (!encode(&amap, in.base, 3, dims, strides, box, err)) return -1;
        args.m_total = in.pixels();
        m_tiles = (in.pixels() + kBM - 1) / kBM;
    } else {
        const int tw = ow >= 12 ? 16 : 8;
        const int th = kBM / tw;
        args.tile_w = tw;
        args.tile_h = th;
        args.tiles_x = (ow + tw - 1) / tw;
        args.tiles_y = (oh + th - 1) / th;
        const cuuint64_t dims[5] = {static_cast<cuuint64_t>(in.c), 2, static_cast<cuuint64_t>(in.w),
                                    static_cast<cuuint64_t>(in.h), static_cast<cuuint64_t>(in.n)};
        const cuuint64_t strides[4] = {static_cast<cuuint64_t>(in.pitch), static_cast<cuuint64_t>(2 * in.pitch),
                                       static_cast<cuuint64_t>(2 * in.pitch) * in.row_px,
                                       static_cast<cuuint64_t>(2 * in.pitch) * in.img_px};
        const cuuint32_t box[5] = {kBK, 1, static_cast<cuuint32_t>(tw), static_cast<cuuint32_t>(th), 1};
        if (!encode(&amap, in.base, 5, dims, strides, box, err)) return -1;
        m_tiles = static_cast<long long>(args.tiles_x) * args.tiles_y * in.n;
    }
    const long long total = m_tiles * w.co_tiles;
    if (total > INT32_MAX) {
        err = "too many output tiles";
        return -1;
    }
    args.total_tiles = static_cast<int>(total);
    const cudaError_t e =
        flat ? launch<false>(amap, w.map, args, w.bn, stream) : launch<true>(amap, w.map, args, w.bn, stream);
    if (e != cudaSuccess) {
        err = std::string("conv launch failed: ") + cudaGetErrorString(e);
        return -1;
    }
    return 0;
}

}  // namespace ufb
