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
// For K <= 8192 every partial sum fits s32 and the recombination runs in
// 32-bit arithmetic; longer reductions take the int64 SIMT path.
//
// GEMM orientation: M = 128 output pixels (TMEM lanes), N = 128 output
// channels per tile, K = taps x input channels.  Activations are split NHWC in
// HBM, so both operands are K-major and arrive by TMA as 128-byte swizzled
// tiles; 3x3 taps are spatially shifted TMA boxes over a 5-D tensor map whose
// zero fill is the convolution's zero padding.
//
// Persistent CTAs (one per SM) walk the output tiles.  Warp 0 issues TMA into a
// 3 x 64 KB ring that runs ahead across tiles (about 1.4 us of L2 round trip
// per stage needs that much in flight), warp 1 owns TMEM and issues the MMAs,
// warps 2-9 run the epilogue, two per TMEM lane quarter, 64 output channels
// each.  Consecutive tiles alternate between accumulator sets at TMEM columns
// [0, 384) and [128, 512): the next tile's set overlaps only two of the three
// slices of the current one, so the epilogue drains those two, releases TMEM
// and reads the third while the next tile's MMAs already run.  Each epilogue
// warp then recombines, adds the bias, saturates, applies the fused
// elementwise step and stores its 32 pixels x 64 channels through its own
// 2 KB shared-memory stage (64-byte swizzle, one byte plane at a time) with a
// TMA store, which writes whole lines: per-thread pixel-row stores reach only
// a third of the bandwidth.
#include "umma.cuh"
#include "conv_epi.cuh"
#include "conv_tc.h"

#include <cuda_runtime.h>
#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

namespace ufb {

namespace {

constexpr int kBM = 128;                                    // output pixels per tile
constexpr int kBN = 128;                                    // output channels per tile
constexpr int kBK = 128;                                    // input channels per K block
// Eight epilogue warps, two per TMEM lane quarter, 64 accumulator columns
// each: with ten warps per CTA (at most three per SM sub-partition) a thread
// may hold 168 registers, enough for two drained 64-column slices.
constexpr int kEpiWarps = 8;
constexpr int kFirstEpiWarp = 2;
constexpr int kThreads = (kFirstEpiWarp + kEpiWarps) * 32;  // 320
constexpr uint32_t kABytes = kBM * kBK;                     // one activation plane tile
constexpr uint32_t kBBytes = 2 * kBN * kBK;                 // stacked low / high weight rows
constexpr uint32_t kStageBytes = 2 * kABytes + kBBytes;     // 64 KB
constexpr int kStages = 3;
// Per epilogue warp: 32 pixels x 64 channels of one byte plane (2 KB), or of
// both planes in the residual mode (4 KB: the warp's residual tile arrives by
// TMA into the stage, which then holds both output planes).
constexpr int kWarpCols = kBN / (kEpiWarps / 4);              // output channels per epilogue warp
constexpr uint32_t kPlaneStage = 32 * kWarpCols;             // 32 pixels x kWarpCols channels, one plane
__host__ __device__ constexpr uint32_t warp_stage_bytes(int mode) { return mode == 2 ? 2 * kPlaneStage : kPlaneStage; }

// Position of 16-byte chunk h of stage row r: the 64-byte swizzle for 64-byte
// rows (chunk ^ ((r >> 1) & 3)) or the 32-byte swizzle for 32-byte rows
// (chunk ^ ((r >> 2) & 1)), so the eight lanes of a shared-memory phase hit
// distinct banks; the TMA maps use the matching swizzle mode.
__device__ __forceinline__ int stage_off(int r, int h) {
    return kWarpCols == 64 ? r * 64 + ((h ^ ((r >> 1) & 3)) << 4) : r * 32 + ((h ^ ((r >> 2) & 1)) << 4);
}
constexpr CUtensorMapSwizzle kStageSwizzle = kWarpCols == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
constexpr uint32_t kTmemCols = 512;                         // two staggered accumulator sets
constexpr size_t kSmemOptin = 227 * 1024;  // shared memory per CTA on sm_100 (static + dynamic)
constexpr size_t kSmemBudget = kSmemOptin - 256;  // host-side planning: static barriers stay below 256 B

// How an output tile is written.
enum StoreKind : int {
    kStoreTma = 0,      // both planes through the stage, 128-channel boxes
    kStoreThreadRows,   // wsilu4: each thread stores its pixel's 16 output channels per plane
    kStoreThreads,      // pixel shuffle: per-thread stores to four target pixels
};

struct ConvTcArgs {
    Act out;
    Epilogue epi;
    int co, ci, taps_h, taps_w, pad_h, pad_w, cpad;
    int stride;  // spatial mode: 1, or 2 (every second input pixel per tap, TMA element strides)
    int oh, ow;
    int tile_w, tile_h, tiles_x, tiles_y;
    long long m_total;  // flat mode: output pixels
    int n_tiles, total_tiles;
    int signed_split;
    int* status;
};

struct TileCoord {
    int img, y0, x0, co0;
    long long p0;
};

template <bool SPATIAL>
__device__ __forceinline__ TileCoord tile_coord(const ConvTcArgs& a, int tile) {
    TileCoord t{};
    const int m = tile / a.n_tiles;
    t.co0 = (tile - m * a.n_tiles) * kBN;
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

// v = sat(v + res) for 16 packed outputs of one pixel, the second residual of
// the fused epilogue (n_valid < 16 at a ragged channel tail; src/layers.cpp:98-104).
__device__ __forceinline__ void add_one_residual(const Act& res, uint32_t (&p)[8], int cbase, int n_valid,
                                                 long long rp) {
    uint32_t wl[4] = {0, 0, 0, 0}, wh[4] = {0, 0, 0, 0};
    const uint8_t* lo = res.lo(rp) + cbase;
    const uint8_t* hi = lo + res.pitch;
    if (n_valid == 16 && ((reinterpret_cast<uintptr_t>(lo) | reinterpret_cast<uintptr_t>(hi)) & 15) == 0) {
        // 16 channels of both planes in two 16-byte loads
        const uint4 l = *reinterpret_cast<const uint4*>(lo);
        const uint4 h = *reinterpret_cast<const uint4*>(hi);
        wl[0] = l.x, wl[1] = l.y, wl[2] = l.z, wl[3] = l.w;
        wh[0] = h.x, wh[1] = h.y, wh[2] = h.z, wh[3] = h.w;
    } else {
        // channel tails and views that are not 16-byte aligned: byte by byte
        // (unrolled, so the words stay in registers)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j < n_valid) {
                wl[j >> 2] |= static_cast<uint32_t>(lo[j]) << (8 * (j & 3));
                wh[j >> 2] |= static_cast<uint32_t>(hi[j]) << (8 * (j & 3));
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t q0, q1;
        join_bytes(wl[k], wh[k], q0, q1);
        p[2 * k] = pack2_sat(lo16(p[2 * k]) + lo16(q0), hi16(p[2 * k]) + hi16(q0));
        p[2 * k + 1] = pack2_sat(lo16(p[2 * k + 1]) + lo16(q1), hi16(p[2 * k + 1]) + hi16(q1));
    }
}

// L2 prefetch of both planes of a tile's second residual rows (the first
// arrives by TMA into the epilogue stages).
template <bool SPATIAL>
__device__ __forceinline__ void prefetch_residuals(const CUtensorMap* m2, const ConvTcArgs& a, int tile) {
    const TileCoord tc = tile_coord<SPATIAL>(a, tile);
#pragma unroll
    for (int plane = 0; plane < 2; ++plane) {
        if (SPATIAL)
            tma_prefetch_5d(m2, tc.co0, plane, tc.x0, tc.y0, tc.img);
        else
            tma_prefetch_3d(m2, tc.co0, plane, static_cast<int>(tc.p0));
    }
}

// Hands the drained accumulator columns back to the MMA warp.
__device__ __forceinline__ void release_tmem(uint64_t* bar, int lane) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

// TMA load of one epilogue warp's box (residual rows), completing on bar.
template <bool SPATIAL>
__device__ __forceinline__ void tma_load_quarter(const CUtensorMap* map, void* dst, uint64_t* bar, const ConvTcArgs& a,
                                                 const TileCoord& tc, int quarter, int c0, int plane) {
    if (SPATIAL)
        tma_load_5d(dst, map, bar, c0, plane, tc.x0, tc.y0 + quarter * 32 / a.tile_w, tc.img);
    else
        tma_load_3d(dst, map, bar, c0, plane, static_cast<int>(tc.p0) + quarter * 32);
}

// Bias loads from shared memory stay where the epilogue uses them (volatile):
// hoisted to the top of a tile they would hold 64 registers and cause spills.
__device__ __forceinline__ int4 load_bias4(const int32_t* b) {
    int4 v;
    asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(b)));
    return v;
}
__device__ __forceinline__ int4 load_bias4(const int16_t* b) {
    uint32_t x, y;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(x), "=r"(y) : "r"(smem_u32(b)));
    return make_int4(lo16(x), hi16(x), lo16(y), hi16(y));
}

// TMA store of one epilogue warp's box: the 32 pixels of TMEM lane quarter q
// (tile rows 32 q / tile_w ..) and channels c0 .. of one plane.
template <bool SPATIAL>
__device__ __forceinline__ void tma_store_quarter(const CUtensorMap* map, const void* src, const ConvTcArgs& a,
                                                  const TileCoord& tc, int quarter, int c0, int plane) {
    if (SPATIAL)
        tma_store_5d(map, src, c0, plane, tc.x0, tc.y0 + quarter * 32 / a.tile_w, tc.img);
    else
        tma_store_3d(map, src, c0, plane, static_cast<int>(tc.p0) + quarter * 32);
}

template <bool SPATIAL, int MODE, int SIGNED, bool NARROW>
__global__ void __launch_bounds__(kThreads, 1)
conv_i16_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapOut, const __grid_constant__ CUtensorMap mapRes1,
                   const __grid_constant__ CUtensorMap mapRes2, const ConvTcArgs args) {
    constexpr int STORE = MODE == kEpiShuffle2 ? kStoreThreads : (MODE == kEpiWsilu4 ? kStoreThreadRows : kStoreTma);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t kStage = warp_stage_bytes(MODE);
    // the residual mode stages its (int16) bias as int16 to fit the larger stages
    using BiasT = typename std::conditional<MODE == kEpiRes, int16_t, int32_t>::type;
    uint8_t* staging = smem + size_t(kStages) * kStageBytes;                           // 1024-aligned
    BiasT* bias_s = reinterpret_cast<BiasT*>(staging + kStage * kEpiWarps);             // [n_tiles * 128]
    int16_t* lut_s = reinterpret_cast<int16_t*>(bias_s + args.n_tiles * kBN);          // LUT window
    __shared__ __align__(8) uint64_t full_bar[kStages];
    __shared__ __align__(8) uint64_t empty_bar[kStages];
    __shared__ __align__(8) uint64_t tmem_full, tmem_empty;
    __shared__ __align__(8) uint64_t res_bar[MODE == kEpiRes ? kEpiWarps : 1];
    __shared__ uint32_t tmem_holder;
    __shared__ int consumed;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_per_tap = (args.ci + kBK - 1) / kBK;
    const int num_k = args.taps_h * args.taps_w * kb_per_tap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&tmem_full, 1);
        mbar_init(&tmem_empty, kEpiWarps);
        if (MODE == kEpiRes)
            for (int i = 0; i < kEpiWarps; ++i) mbar_init(&res_bar[i], 1);
        consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    // window start of the fused table step: the staged bias carries -lut_start
    const int lut_start = MODE == kEpiLut || MODE == kEpiWsilu4 ? args.epi.lut_start : 0;
    // the whole bias vector, zero padded to the tile grid, once per CTA
    for (int i = threadIdx.x; i < args.n_tiles * kBN; i += kThreads) {
        long long b = 0;
        if (args.epi.bias && i < args.co)
            b = args.epi.bias32 ? static_cast<const int32_t*>(args.epi.bias)[i]
                                : static_cast<const int16_t*>(args.epi.bias)[i];
        bias_s[i] = static_cast<BiasT>(MODE == kEpiRes ? b : stage_bias(b) - lut_start);
    }
    // table window as differences lut[v] - v (the host checked that they fit
    // int16); lut_window() turns them back into lut[sat16(v)]
    const int16_t* lut_d = lut_s;
    if (MODE == kEpiLut || MODE == kEpiWsilu4) {
        for (int i = threadIdx.x; i < args.epi.lut_n; i += kThreads)
            lut_s[i] = static_cast<int16_t>(args.epi.lut[lut_start + 32768 + i] - (lut_start + i));
    }
    const int lut_last = args.epi.lut_n - 1, lut_cap = 32767 - lut_start;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_holder;

    int issued = 0;
    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&mapA);
            prefetch_tmap(&mapB);
            int it = 0, s = 0, ti = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x, ++ti) {
                const TileCoord tc = tile_coord<SPATIAL>(args, tile);
                // weight rows of the tile: low-byte block at row w_row, high-byte block
                // 128 rows on; even tiles stack them high over low, odd tiles low over high
                const int w_row = (tc.co0 / kBN) * 2 * kBN;
                const int first_rows = (ti & 1) ? w_row : w_row + kBN;
                const int second_rows = (ti & 1) ? w_row + kBN : w_row;
                for (int k = 0; k < num_k; ++k, ++it) {
                    if (it >= kStages && !mbar_wait(&empty_bar[s], ((it / kStages) - 1) & 1, args.status, 1)) {
                        ok = false;
                        break;
                    }
                    const int tap = k / kb_per_tap, cb = k - tap * kb_per_tap;
                    const int ky = tap / args.taps_w, kx = tap - ky * args.taps_w;
                    uint8_t* st = smem + size_t(s) * kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
                    const int c0 = cb * kBK;
                    if (SPATIAL) {
                        const int ix = tc.x0 * args.stride + kx - args.pad_w;
                        const int iy = tc.y0 * args.stride + ky - args.pad_h;
                        tma_load_5d(st, &mapA, &full_bar[s], c0, 0, ix, iy, tc.img);
                        tma_load_5d(st + kABytes, &mapA, &full_bar[s], c0, 1, ix, iy, tc.img);
                    } else {
                        tma_load_3d(st, &mapA, &full_bar[s], c0, 0, static_cast<int>(tc.p0));
                        tma_load_3d(st + kABytes, &mapA, &full_bar[s], c0, 1, static_cast<int>(tc.p0));
                    }
                    tma_load_2d(st + 2 * kABytes, &mapB, &full_bar[s], tap * args.cpad + c0, first_rows);
                    tma_load_2d(st + 2 * kABytes + kBN * kBK, &mapB, &full_bar[s], tap * args.cpad + c0, second_rows);
                    issued = it + 1;
                    if (++s == kStages) s = 0;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t i_uu = i8_idesc(kBM, kBN, false, false);
            constexpr uint32_t i_su = i8_idesc(kBM, kBN, true, false);
            constexpr uint32_t i_us = i8_idesc(kBM, kBN, false, true);
            constexpr uint32_t i_ss = i8_idesc(kBM, kBN, true, true);
            constexpr uint32_t i_us2 = i8_idesc(kBM, 2 * kBN, false, true);
            constexpr uint32_t i_ss2 = i8_idesc(kBM, 2 * kBN, true, true);
            int it = 0, s = 0, ti = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < args.total_tiles; tile += gridDim.x, ++ti) {
                if (ti > 0 && !mbar_wait(&tmem_empty, (ti - 1) & 1, args.status, 3)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // Accumulator slots (columns): even tiles HH [0, 128), X [128, 256),
                // LL [256, 384); odd tiles LL [128, 256), X [256, 384), HH [384, 512).
                // Both sets keep LL and X in the two slots they share, HH in the
                // slot of their own, and the weight tile is stacked [wh; wl] for
                // even tiles and [wl; wh] for odd ones, so one N=256 MMA of the
                // low activation bytes always lands at column 128 and one of the
                // high bytes at column 0 (even) or 256 (odd).
                const bool even = (ti & 1) == 0;
                const uint32_t d_ll = tmem + (even ? 2 : 1) * kBN, d_x = tmem + (even ? 1 : 2) * kBN,
                               d_hh = tmem + (even ? 0 : 3) * kBN;
                const uint32_t d_lo2 = tmem + kBN, d_hi2 = tmem + (even ? 0 : 2) * kBN;
                for (int k = 0; k < num_k; ++k, ++it) {
                    if (!mbar_wait(&full_bar[s], (it / kStages) & 1, args.status, 2)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_u32(smem + size_t(s) * kStageBytes);
                    const uint32_t a_lo = base, a_hi = base + kABytes, b_first = base + 2 * kABytes,
                                   b_second = b_first + kBN * kBK;
                    const uint32_t b_lo = even ? b_second : b_first, b_hi = even ? b_first : b_second;
                    // descriptors are linear in the start address (its >> 4 in the low
                    // bits), so each K step adds 32 >> 4 = 2 to the block's base ones
                    const uint64_t q_alo = sw128_desc(a_lo), q_ahi = sw128_desc(a_hi), q_bf = sw128_desc(b_first),
                                   q_blo = sw128_desc(b_lo), q_bhi = sw128_desc(b_hi);
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk) {
                        const uint64_t o = 2 * kk;
                        const bool first = k == 0 && kk == 0;
                        if (SIGNED) {
                            mma_i8(d_lo2, q_alo + o, q_bf + o, i_us2, first ? 0u : 1u);
                            if (first) {
                                mma_i8(d_x, q_ahi + o, q_blo + o, i_ss, 1u);
                                mma_i8(d_hh, q_ahi + o, q_bhi + o, i_ss, 0u);
                            } else {
                                mma_i8(d_hi2, q_ahi + o, q_bf + o, i_ss2, 1u);
                            }
                        } else {
                            const uint32_t acc = first ? 0u : 1u;
                            mma_i8(d_ll, q_alo + o, q_blo + o, i_uu, acc);
                            mma_i8(d_x, q_ahi + o, q_blo + o, i_su, acc);
                            mma_i8(d_x, q_alo + o, q_bhi + o, i_us, 1u);
                            mma_i8(d_hh, q_ahi + o, q_bhi + o, i_ss, acc);
                        }
                    }
                    mma_commit(&empty_bar[s]);
                    if (++s == kStages) s = 0;
                }
                if (!ok) break;
                mma_commit(&tmem_full);
            }
            consumed = it;
        }
        __syncwarp();
    } else if (warp >= kFirstEpiWarp) {
        constexpr int kCols = kBN / (kEpiWarps / 4);  // accumulator columns (output channels) per thread
        constexpr int kWords = kCols / 2;              // packed int16 pairs per thread
        constexpr int kLd = kCols / 32;                // 32-column TMEM loads per slice
        const int quarter = warp & 3;
        const int cgroup = (warp - kFirstEpiWarp) >> 2;  // columns [kCols cgroup, kCols cgroup + kCols)
        const int row = quarter * 32 + lane;            // TMEM lane = pixel of the tile
        const uint32_t acc = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + cgroup * kCols;  // + set offset
        const bool issuer = warp == kFirstEpiWarp && lane == 0;  // residual prefetches
        const int ew = warp - kFirstEpiWarp;
        uint8_t* stage = staging + ew * kStage;  // this warp's own stage
        // Multipliers the compiler cannot see: products with them stay integer
        // multiply-adds on the FMA pipe instead of becoming shift-adds on the
        // ALU pipe, which the epilogue's compares, selects and shifts keep busy.
        int32_t c8 = 8, c256 = 256;
        asm volatile("" : "+r"(c8), "+r"(c256));
        int res_issued = 0, res_seen = 0;
        const Act& out = args.out;
        int ti = 0;
        if (MODE == kEpiRes && issuer && args.epi.res2.base && blockIdx.x < args.total_tiles)
            prefetch_residuals<SPATIAL>(&mapRes2, args, blockIdx.x);
        for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x, ++ti) {
            // residual rows of this CTA's next tile into L2 while this one finishes
            if (MODE == kEpiRes && issuer && args.epi.res2.base && tile + static_cast<int>(gridDim.x) < args.total_tiles)
                prefetch_residuals<SPATIAL>(&mapRes2, args, tile + gridDim.x);
            const TileCoord tc = tile_coord<SPATIAL>(args, tile);
            const int cbase = tc.co0 + cgroup * kCols;
            if (MODE == kEpiRes && lane == 0) {
                // this warp's 32 x 64 residual tile (both planes): in flight while the
                // MMAs finish and the accumulators are recombined, once the previous
                // tile's TMA store has read the stage (that store was left in flight
                // so the previous tile did not wait for it)
                bulk_wait_read();
                mbar_arrive_expect_tx(&res_bar[ew], 2 * kPlaneStage);
                tma_load_quarter<SPATIAL>(&mapRes1, stage, &res_bar[ew], args, tc, quarter, cbase, 0);
                tma_load_quarter<SPATIAL>(&mapRes1, stage + kPlaneStage, &res_bar[ew], args, tc, quarter, cbase, 1);
            }
            if (MODE == kEpiRes) ++res_issued;
            if (!mbar_wait(&tmem_full, ti & 1, args.status, 4)) break;
            tc_fence_after();
            uint32_t p[kWords];   // packed int16 pairs of the kCols outputs
            int32_t o4[kCols / 4];  // wsilu4: the kCols / 4 reduced outputs
            // LL and X sit in the two slots every accumulator set shares, HH in
            // the set's own slot (see the MMA warp)
            const bool even = (ti & 1) == 0;
            const uint32_t a_ll = acc + (even ? 2 : 1) * kBN, a_x = acc + (even ? 1 : 2) * kBN,
                           a_hh = acc + (even ? 0 : 3) * kBN;
            // Drain LL and X, then hand the shared slots back to the MMA warp.  NARROW: D = P = LL + 256 X (P + 4096 fits 32 bits
            // for this layer's weights), so S = 65536 HH + P.  Otherwise
            // D = (X >> 5) + (U >> 13) with U = LL + 256 (X & 31) + 4096 and a
            // tie bit U % 8192 == 0, so S + 4096 = 8192 (8 HH + D) + (U & 8191).
            // Both slots come in with one wait, so the MMA warp gets them back
            // after a single TMEM round trip.
            static_assert(kCols == 64, "drain loads 64 columns per slot");
            int32_t D[kCols];
            uint32_t ties[kLd];
            {
                uint32_t ll[kCols], xx[kCols];
                tmem_ld64(a_ll, ll);
                tmem_ld64(a_x, xx);
                tmem_wait_ld();
                release_tmem(&tmem_empty, lane);
#pragma unroll
                for (int i = 0; i < kLd; ++i) {
                    ties[i] = 0;
#pragma unroll
                    for (int t = 0; t < 32; ++t) {
                        const int32_t x = static_cast<int32_t>(xx[32 * i + t]);
                        const int32_t l = static_cast<int32_t>(ll[32 * i + t]);
                        if (NARROW) {
                            D[32 * i + t] = x * c256 + l;
                        } else {
                            const int32_t U = (x & 31) * c256 + (l + 4096);
                            D[32 * i + t] = (x >> 5) + (U >> 13);
                            ties[i] |= static_cast<uint32_t>((U & 8191) == 0) << t;
                        }
                    }
                }
            }
            // HH 16 columns at a time, the next 16 in flight while these are
            // finished: rna(S / 8192) = floor((S + 4096 - [S < 0]) / 8192) (half
            // away from zero); the general form takes T = floor((S + 4096) / 8192)
            // and, at an exact tie with S < 0 (T <= 0), T - 1.  Then the bias and
            // the fused table step.
            uint32_t hh_buf[2][16];
            tmem_ld16(a_hh, hh_buf[0]);
            tmem_wait_ld_regs(hh_buf[0]);
#pragma unroll
            for (int h = 0; h < kCols / 16; ++h) {
                if (h + 1 < kCols / 16) tmem_ld16(a_hh + 16 * (h + 1), hh_buf[(h + 1) & 1]);
                const uint32_t(&hh)[16] = hh_buf[h & 1];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int4 b = load_bias4(bias_s + cbase + 16 * h + 4 * q);
                    const int bb[4] = {b.x, b.y, b.z, b.w};
                    int32_t r[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const int j = 16 * h + 4 * q + t;
                        const int32_t H8 = static_cast<int32_t>(hh[4 * q + t]) * c8;
                        if (NARROW) {
                            // fl = floor(S / 8192) is negative exactly when S is, and
                            // rna(S / 8192) = 8 HH + floor((P + 4096 - [S < 0]) / 8192)
                            const int32_t fl = H8 + (D[j] >> 13);
                            r[t] = H8 + ((D[j] + 4096 + (fl >> 31)) >> 13) + bb[t];
                        } else {
                            const int32_t T = H8 + D[j];
                            const bool tie = (ties[j / 32] >> (j % 32)) & 1u;
                            r[t] = T - static_cast<int32_t>(tie & (T <= 0)) + bb[t];
                        }
                    }
                    if (MODE == kEpiLut || MODE == kEpiWsilu4) {
                        // table window: r is conv - window start (the staged bias
                        // carries the shift)
                        int32_t v[4];
#pragma unroll
                        for (int t = 0; t < 4; ++t) v[t] = lut_window(lut_d, lut_last, lut_cap, r[t]);
                        if (MODE == kEpiWsilu4) {
                            o4[4 * h + q] = v[0] + v[1] + v[2] + v[3] + 4 * lut_start;
                        } else {
                            p[8 * h + 2 * q] = pack2(v[0] + lut_start, v[1] + lut_start);
                            p[8 * h + 2 * q + 1] = pack2(v[2] + lut_start, v[3] + lut_start);
                        }
                    } else {
                        p[8 * h + 2 * q] = pack2_sat(r[0], r[1]);
                        p[8 * h + 2 * q + 1] = pack2_sat(r[2], r[3]);
                    }
                }
                if (h + 1 < kCols / 16) tmem_wait_ld_regs(hh_buf[(h + 1) & 1]);
            }
            const int n_valid = args.co - cbase < 0 ? 0 : (args.co - cbase < kCols ? args.co - cbase : kCols);
            bool valid;
            long long rpx1 = 0, rpx2 = 0;
            int oy = 0, ox = 0;
            if (SPATIAL) {
                const int ty = row / args.tile_w, tx = row - ty * args.tile_w;
                oy = tc.y0 + ty;
                ox = tc.x0 + tx;
                valid = oy < args.oh && ox < args.ow;
                if (MODE == kEpiRes) {
                    rpx1 = args.epi.res1.pixel(tc.img, oy, ox);
                    rpx2 = args.epi.res2.pixel(tc.img, oy, ox);
                }
            } else {
                rpx1 = rpx2 = tc.p0 + row;
                valid = rpx1 < args.m_total;
            }
            if (STORE == kStoreThreads) {
                if (valid) {
#pragma unroll
                    for (int h = 0; h < kCols / 16; ++h) {
                        if (16 * h >= n_valid) break;
                        uint32_t p8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) p8[i] = p[8 * h + i];
                        store_shuffle2(out, p8, cbase + 16 * h, n_valid - 16 * h < 16 ? n_valid - 16 * h : 16,
                                       tc.img, oy, ox);
                    }
                }
                continue;
            }
            // fused residual step (residual rows outside the image read nothing)
            if (MODE == kEpiRes) {
                // first residual from the stage (64-byte swizzle, like the output)
                ++res_seen;
                if (!mbar_wait(&res_bar[ew], ti & 1, args.status, 7)) break;
#pragma unroll
                for (int h = 0; h < kCols / 16; ++h) {
                    const int off = stage_off(lane, h);
                    const uint4 rl = *reinterpret_cast<const uint4*>(stage + off);
                    const uint4 rh = *reinterpret_cast<const uint4*>(stage + kPlaneStage + off);
                    const uint32_t lw[4] = {rl.x, rl.y, rl.z, rl.w}, hw[4] = {rh.x, rh.y, rh.z, rh.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint32_t q0, q1;
                        join_bytes(lw[k], hw[k], q0, q1);
                        uint32_t& a0 = p[8 * h + 2 * k];
                        uint32_t& a1 = p[8 * h + 2 * k + 1];
                        a0 = pack2_sat(lo16(a0) + lo16(q0), hi16(a0) + hi16(q0));
                        a1 = pack2_sat(lo16(a1) + lo16(q1), hi16(a1) + hi16(q1));
                    }
                }
                __syncwarp();  // every lane has read the stage before it takes the output
                // second residual (the up / down blocks' shortcut): per-thread loads
                if (args.epi.res2.base && valid) {
#pragma unroll
                    for (int h = 0; h < kCols / 16; ++h) {
                        if (16 * h >= n_valid) break;
                        uint32_t p8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) p8[i] = p[8 * h + i];
                        add_one_residual(args.epi.res2, p8, cbase + 16 * h,
                                         n_valid - 16 * h < 16 ? n_valid - 16 * h : 16, rpx2);
#pragma unroll
                        for (int i = 0; i < 8; ++i) p[8 * h + i] = p8[i];
                    }
                }
            }
            if (STORE == kStoreTma && MODE == kEpiRes) {
                // both output planes into the 4 KB stage, one wait for the reads
#pragma unroll
                for (int h = 0; h < kCols / 16; ++h) {
                    uint32_t p8[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) p8[i] = p[8 * h + i];
                    uint4 lo, hi;
                    split_bytes(p8, lo, hi);
                    const int off = stage_off(lane, h);
                    *reinterpret_cast<uint4*>(stage + off) = lo;
                    *reinterpret_cast<uint4*>(stage + kPlaneStage + off) = hi;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_quarter<SPATIAL>(&mapOut, stage, args, tc, quarter, cbase, 0);
                    tma_store_quarter<SPATIAL>(&mapOut, stage + kPlaneStage, args, tc, quarter, cbase, 1);
                    bulk_commit();  // read by the next tile's residual load (bulk_wait_read there)
                }
            } else if (STORE == kStoreTma) {
                // each warp stores its own 32 pixels x 64 channels, one byte plane
                // at a time, through its 2 KB stage in the 64-byte swizzle
                // (16-byte chunk c of row r at position c ^ ((r >> 1) & 3)), so
                // the eight lanes of a shared-memory phase hit distinct banks
#pragma unroll
                for (int plane = 0; plane < 2; ++plane) {
                    // the stage is free once the previous store out of it (the other
                    // plane, or the previous tile's second plane, left in flight) is read
                    if (lane == 0) bulk_wait_read();
                    __syncwarp();
#pragma unroll
                    for (int h = 0; h < kCols / 16; ++h) {
                        uint32_t p8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) p8[i] = p[8 * h + i];
                        uint4 lo, hi;
                        split_bytes(p8, lo, hi);
                        *reinterpret_cast<uint4*>(stage + stage_off(lane, h)) = plane ? hi : lo;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_quarter<SPATIAL>(&mapOut, stage, args, tc, quarter, cbase, plane);
                        bulk_commit();
                    }
                }
            } else {
                // wsilu4: each thread holds kCols / 4 = 16 output channels of its
                // pixel, stored as one 16-byte word per plane (the two column
                // groups of a pixel fill its 32-byte sector together)
                static_assert(kCols / 4 == 16, "wsilu4 stores 16 channels per thread");
                uint32_t lw[4], hw[4];
#pragma unroll
                for (int h = 0; h < kCols / 16; ++h) {
                    const uint32_t w0 = pack2_sat(o4[4 * h], o4[4 * h + 1]), w1 = pack2_sat(o4[4 * h + 2], o4[4 * h + 3]);
                    lw[h] = __byte_perm(w0, w1, 0x6420);
                    hw[h] = __byte_perm(w0, w1, 0x7531);
                }
                const int oc = cbase / 4;
                const int n_out = args.out.c - oc < 16 ? args.out.c - oc : 16;
                if (valid && n_out > 0) {
                    const long long opx = SPATIAL ? out.pixel(tc.img, oy, ox) : rpx1;
                    if (n_out == 16) {
                        *reinterpret_cast<uint4*>(out.lo(opx) + oc) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                        *reinterpret_cast<uint4*>(out.hi(opx) + oc) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    } else {
                        // channel tail (unrolled, so the words stay in registers)
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (j < n_out) {
                                out.lo(opx)[oc + j] = static_cast<uint8_t>(lw[j >> 2] >> (8 * (j & 3)));
                                out.hi(opx)[oc + j] = static_cast<uint8_t>(hw[j >> 2] >> (8 * (j & 3)));
                            }
                        }
                    }
                }
            }
        }
        // abort path only: a residual load issued for a tile that was not finished
        if (MODE == kEpiRes && res_issued > res_seen) mbar_wait(&res_bar[ew], (res_issued - 1) & 1, args.status, 8);
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // abort path only: wait for TMA loads issued but never consumed, so no
        // copy into this CTA's shared memory outlives the CTA
        for (int k = consumed; k < issued; ++k) mbar_wait(&full_bar[k % kStages], (k / kStages) & 1, args.status, 5);
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
            const cuuint32_t* box, std::string& err, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B,
            const cuuint32_t* element_strides = nullptr) {
    auto fn = encode_fn();
    if (!fn) {
        err = "cuTensorMapEncodeTiled is unavailable";
        return false;
    }
    cuuint32_t elem[5] = {1, 1, 1, 1, 1};
    if (element_strides)
        for (int i = 0; i < rank; ++i) elem[i] = element_strides[i];
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, base, dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        err = "cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r));
        return false;
    }
    return true;
}

std::atomic<int> g_max_ctas{0};
std::atomic<bool> g_narrow{true};

int current_device() {
    int device = 0;
    return cudaGetDevice(&device) == cudaSuccess ? device : 0;
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

struct ConvMaps {
    CUtensorMap a, b, out, res1, res2;
};

template <bool SPATIAL, int MODE, int SIGNED, bool NARROW>
cudaError_t launch_mode(const ConvMaps& m, const ConvTcArgs& args, size_t smem, int sms, cudaStream_t stream) {
    auto kernel = conv_i16_tc_kernel<SPATIAL, MODE, SIGNED, NARROW>;
    // The attribute is per function and device and shared by every thread that
    // launches the kernel, so it is always the kernel's full allowance (a
    // per-launch value could be lowered by another thread between its set and
    // this launch).
    static const int allowance = [&] {
        cudaFuncAttributes attr{};
        return cudaFuncGetAttributes(&attr, kernel) == cudaSuccess
                   ? static_cast<int>(kSmemOptin) - static_cast<int>(attr.sharedSizeBytes)
                   : 0;
    }();
    if (smem > static_cast<size_t>(allowance)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, allowance);
    if (e != cudaSuccess) return e;
    int grid = args.total_tiles < sms ? args.total_tiles : sms;
    const int cap = g_max_ctas.load(std::memory_order_relaxed);
    if (cap > 0 && grid > cap) grid = cap;
    kernel<<<grid, kThreads, smem, stream>>>(m.a, m.b, m.out, m.res1, m.res2, args);
    return cudaGetLastError();
}

template <bool SPATIAL, int SIGNED, bool NARROW>
cudaError_t launch_signed(const ConvMaps& m, const ConvTcArgs& args, size_t smem, int sms, cudaStream_t stream) {
    const Epilogue& e = args.epi;
    if (e.shuffle2) return launch_mode<SPATIAL, kEpiShuffle2, SIGNED, NARROW>(m, args, smem, sms, stream);
    if (e.wsilu4) return launch_mode<SPATIAL, kEpiWsilu4, SIGNED, NARROW>(m, args, smem, sms, stream);
    if (e.lut) return launch_mode<SPATIAL, kEpiLut, SIGNED, NARROW>(m, args, smem, sms, stream);
    if (e.res1.base) return launch_mode<SPATIAL, kEpiRes, SIGNED, NARROW>(m, args, smem, sms, stream);
    return launch_mode<SPATIAL, kEpiPlain, SIGNED, NARROW>(m, args, smem, sms, stream);
}

template <bool SPATIAL>
cudaError_t launch(const ConvMaps& m, const ConvTcArgs& args, bool narrow, size_t smem, int sms,
                   cudaStream_t stream) {
    if (narrow)
        return args.signed_split ? launch_signed<SPATIAL, 1, true>(m, args, smem, sms, stream)
                                 : launch_signed<SPATIAL, 0, true>(m, args, smem, sms, stream);
    return args.signed_split ? launch_signed<SPATIAL, 1, false>(m, args, smem, sms, stream)
                             : launch_signed<SPATIAL, 0, false>(m, args, smem, sms, stream);
}

// Tensor map of a split-NHWC view in tile order: flat {c, plane, pixels} (box
// of tw * th pixels) or spatial {c, plane, w, h, n} (box tw x th), box of
// `box_c` channels of one plane.  stride 2 (spatial only): the box spans
// 2 tw x 2 th pixels traversed with element stride 2, so it brings the tw x th
// input pixels a stride-2 convolution tap reads for a tw x th output tile.
bool act_map(CUtensorMap* map, const Act& v, bool flat, int tw, int th, cuuint32_t box_c,
             CUtensorMapSwizzle swizzle, std::string& err, int stride = 1) {
    if (flat) {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(v.c), 2, static_cast<cuuint64_t>(v.pixels())};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(v.pitch), static_cast<cuuint64_t>(2 * v.pitch)};
        const cuuint32_t box[3] = {box_c, 1, static_cast<cuuint32_t>(tw * th)};
        return encode(map, v.base, 3, dims, strides, box, err, swizzle);
    }
    const cuuint64_t dims[5] = {static_cast<cuuint64_t>(v.c), 2, static_cast<cuuint64_t>(v.w),
                                static_cast<cuuint64_t>(v.h), static_cast<cuuint64_t>(v.n)};
    const cuuint64_t strides[4] = {static_cast<cuuint64_t>(v.pitch), static_cast<cuuint64_t>(2 * v.pitch),
                                   static_cast<cuuint64_t>(2 * v.pitch) * v.row_px,
                                   static_cast<cuuint64_t>(2 * v.pitch) * v.img_px};
    const cuuint32_t box[5] = {box_c, 1, static_cast<cuuint32_t>(tw * stride), static_cast<cuuint32_t>(th * stride), 1};
    const cuuint32_t elem[5] = {1, 1, static_cast<cuuint32_t>(stride), static_cast<cuuint32_t>(stride), 1};
    return encode(map, v.base, 5, dims, strides, box, err, swizzle, elem);
}

}  // namespace

void tc_set_max_ctas(int n) { g_max_ctas.store(n > 0 ? n : 0, std::memory_order_relaxed); }
int tc_max_ctas() { return g_max_ctas.load(std::memory_order_relaxed); }

void tc_set_narrow(bool enable) { g_narrow.store(enable, std::memory_order_relaxed); }

bool tc_narrow_enabled() { return g_narrow.load(std::memory_order_relaxed); }

bool tc_narrow_ok(const int16_t* weight_host, int co, int ci, int kh, int kw, bool signed_split) {
    const long long k = static_cast<long long>(ci) * kh * kw;
    for (int o = 0; o < co; ++o) {
        // |LL + 256 X| = |sum_k wl x + 256 wh xl| <= sum_k 32768 |wl| + 65280 |wh|
        long long bound = 4096;
        for (long long i = 0; i < k; ++i) {
            const int32_t v = weight_host[o * k + i];
            const int32_t lo = signed_split ? ((v + 128) & 255) - 128 : (v & 255);
            const int32_t hi = (v - lo) >> 8;
            bound += 32768ll * (lo < 0 ? -lo : lo) + 65280ll * (hi < 0 ? -hi : hi);
        }
        if (bound > INT32_MAX) return false;
    }
    return true;
}

bool tc_encode_map(CUtensorMap* map, void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, std::string& err, CUtensorMapSwizzle swizzle) {
    return encode(map, base, rank, dims, strides, box, err, swizzle);
}

// Dynamic shared memory of a launch without its table window: alignment slack,
// the operand ring, the epilogue warps' stages and the staged bias vector.
size_t conv_smem_bytes(const TcWeights& w, bool res_mode) {
    return 1024 + size_t(kStages) * kStageBytes + size_t(warp_stage_bytes(res_mode ? 2 : 0)) * kEpiWarps +
           size_t(w.co_tiles) * kBN * (res_mode ? 2 : 4);
}

bool tc_table_window_fits(const TcWeights& w, int lut_n, bool res_mode) {
    return lut_n > 0 && conv_smem_bytes(w, res_mode) + (static_cast<size_t>(lut_n) * 2 + 15) / 16 * 16 <= kSmemBudget;
}

size_t tc_weight_bytes(int co, int ci, int kh, int kw, int bn) {
    const int cpad = (ci + kBK - 1) / kBK * kBK;
    const int co_tiles = (co + bn - 1) / bn;
    return static_cast<size_t>(co_tiles) * 2 * bn * kh * kw * cpad;
}

int tc_choose_bn(int, int, int, bool) { return kBN; }

void tc_lut_window(const int16_t* table, int& start, int& n, int& hi) {
    int first_nonzero = 32768, last_moved = -32769;
    for (int v = -32768; v <= 32767; ++v) {
        if (table[v + 32768] != 0 && first_nonzero == 32768) first_nonzero = v;
        if (table[v + 32768] != v) last_moved = v;
    }
    start = first_nonzero > -32768 ? first_nonzero - 1 : -32768;  // lut[start] == 0 unless start == -32768
    hi = last_moved;
    const int end = last_moved < 32767 ? last_moved + 1 : 32767;   // inclusive
    n = end >= start && end - start + 1 <= 8192 ? end - start + 1 : 0;
    for (int i = 0; i < n; ++i) {
        const int d = table[start + i + 32768] - (start + i);
        if (d < -32768 || d > 32767) n = 0;
    }
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
    const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(bn)};
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
                cudaStream_t stream, int* status, std::string& err, int stride) {
    if (stride != 1 && stride != 2) {
        err = "tensor-core convolutions take stride 1 or 2";
        return -1;
    }
    if (in.h + 2 * pad_h < w.kh || in.w + 2 * pad_w < w.kw) {
        err = "kernel exceeds input";
        return -1;
    }
    const int oh = (in.h + 2 * pad_h - w.kh) / stride + 1, ow = (in.w + 2 * pad_w - w.kw) / stride + 1;
    if (stride != 1 && (epi.shuffle2 || epi.wsilu4 || epi.lut || epi.res1.base)) {
        err = "strided convolutions take no fused epilogue step";
        return -1;
    }
    if (in.c != w.ci) {
        err = "input channels do not match weights";
        return -1;
    }
    if (w.bn != kBN) {
        err = "weights must be prepared in 128-wide tiles";
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
    if (epi.wsilu4 && (w.co % 4 || out.c != w.co / 4)) {
        err = "wsilu4 output must have a quarter of the convolution's channels";
        return -1;
    }
    const bool res_mode = epi.res1.base && !epi.shuffle2 && !epi.wsilu4 && !epi.lut;
    if (res_mode && epi.bias && epi.bias32) {
        err = "fused residual adds take an int16 bias";
        return -1;
    }
    if ((epi.lut || epi.wsilu4) && epi.bias && epi.bias32) {
        err = "fused table steps take an int16 bias";
        return -1;
    }
    const size_t base_smem = conv_smem_bytes(w, res_mode);
    if (base_smem > kSmemBudget) {
        err = "too many output channels for the staged bias";
        return -1;
    }
    const long long k_total = static_cast<long long>(w.kh) * w.kw * w.ci;
    if (k_total > kTcMaxReduction) {
        err = "reduction longer than the tensor-core path's 32-bit recombination bound";
        return -1;
    }
    if (k_total == kTcMaxReduction && epi.bias && epi.bias32) {
        // |rna(S / 8192)| reaches 2^30 only here; with an int32 bias staged at
        // up to 2^30 + 2^16 the 32-bit sum could wrap
        err = "a reduction of 8192 terms takes an int16 bias on the tensor-core path";
        return -1;
    }
    const bool flat = stride == 1 && w.kh == 1 && w.kw == 1 && pad_h == 0 && pad_w == 0 && in.dense() && out.dense() &&
                      !epi.shuffle2 && (!epi.res1.base || epi.res1.dense()) && (!epi.res2.base || epi.res2.dense()) &&
                      in.pixels() < (1ll << 31);
    ConvTcArgs args{};
    args.out = out;
    args.epi = epi;
    // the table window rides in shared memory after the bias
    const size_t lut_bytes = (epi.lut || epi.wsilu4) ? (static_cast<size_t>(epi.lut_n) * 2 + 15) / 16 * 16 : 0;
    if ((epi.lut || epi.wsilu4) && !tc_table_window_fits(w, epi.lut_n, res_mode)) {
        err = "fused table steps need a table window that fits shared memory";
        return -1;
    }
    const size_t smem = base_smem + lut_bytes;
    args.co = w.co;
    args.ci = w.ci;
    args.taps_h = w.kh;
    args.taps_w = w.kw;
    args.pad_h = pad_h;
    args.pad_w = pad_w;
    args.cpad = w.cpad;
    args.stride = stride;
    args.oh = oh;
    args.ow = ow;
    args.signed_split = w.signed_split ? 1 : 0;
    args.status = status;
    args.n_tiles = w.co_tiles;
    // output box: 128 channels of one plane (128-byte swizzle), or 32 channels
    // (wsilu4, unswizzled); the map's extent is the view's, so tails are clipped
    ConvMaps maps{};
    maps.b = w.map;
    long long m_tiles;
    int tw = 16, th = kBM / 16;  // flat mode: only tw * th = 128 matters
    if (flat) {
        args.m_total = in.pixels();
        m_tiles = (in.pixels() + kBM - 1) / kBM;
    } else {
        tw = ow >= 12 ? 16 : 8;
        th = kBM / tw;
        args.tile_w = tw;
        args.tile_h = th;
        args.tiles_x = (ow + tw - 1) / tw;
        args.tiles_y = (oh + th - 1) / th;
        m_tiles = static_cast<long long>(args.tiles_x) * args.tiles_y * in.n;
    }
    // the activation box is the tile's input window (shifted per tap in spatial mode)
    if (!act_map(&maps.a, in, flat, tw, th, kBK, CU_TENSOR_MAP_SWIZZLE_128B, err, stride)) return -1;
    // output box: one epilogue warp's 32 pixels, 64 channels (64-byte swizzle);
    // the map's extent is the view's, so tails are clipped
    if (!epi.shuffle2 && !epi.wsilu4) {
        if (!act_map(&maps.out, out, flat, tw, 32 / tw, kWarpCols, kStageSwizzle, err)) return -1;
    } else {
        maps.out = maps.a;  // unused: pixel-shuffled and wsilu4 tiles are stored by the threads
    }
    maps.res1 = maps.res2 = maps.a;  // unused unless residuals are fused
    // first residual: loaded per epilogue warp like the output box; second: L2 prefetch per tile
    if (epi.res1.base && !act_map(&maps.res1, epi.res1, flat, tw, 32 / tw, kWarpCols, kStageSwizzle, err))
        return -1;
    if (epi.res2.base && !act_map(&maps.res2, epi.res2, flat, tw, th, kBN, CU_TENSOR_MAP_SWIZZLE_NONE, err))
        return -1;
    const long long total = m_tiles * w.co_tiles;
    if (total > INT32_MAX) {
        err = "too many output tiles";
        return -1;
    }
    args.total_tiles = static_cast<int>(total);
    const int sms = sm_count(current_device());
    const bool narrow = w.narrow && g_narrow.load(std::memory_order_relaxed);
    const cudaError_t e = flat ? launch<false>(maps, args, narrow, smem, sms, stream)
                               : launch<true>(maps, args, narrow, smem, sms, stream);
    if (e != cudaSuccess) {
        err = std::string("conv launch failed: ") + cudaGetErrorString(e);
        return -1;
    }
    return 0;
}

}  // namespace ufb
