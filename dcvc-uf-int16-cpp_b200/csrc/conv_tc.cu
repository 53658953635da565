// INT16 convolution as an implicit GEMM on the sm_100a tensor cores.
//
// Replaces the reference's mma.sync kernel uf_mma_conv
// (src/cuda/int16_mma.cuh:40-109, dispatched from src/cuda/conv.cu:62-127) with
// the same exact arithmetic (src/cuda/conv.cu:9-13):
//     out = sat(rna(sum_k x_k * w_k / 8192) + bias)
// Each int16 operand is split into an unsigned low byte and a signed high byte,
// v = lo + 256 * hi.  Four tcgen05 kind::i8 products per K block
//     LL = xlo*wlo (u8*u8),  X = xhi*wlo (s8*u8) + xlo*whi (u8*s8),  HH = xhi*whi (s8*s8)
// accumulate exactly in three s32 TMEM accumulators (for K <= 32768:
// |X| <= 65280 K < 2^31, LL <= 65025 K < 2^31) and the epilogue recombines
// LL + 256 X + 65536 HH in int64.
//
// GEMM orientation: M = 128 output pixels (TMEM lanes), N = BN output
// channels (TMEM columns), K = taps x input channels.  Activations are split
// NHWC in HBM, so both operands are K-major and arrive by TMA as 128-byte
// swizzled tiles: one u8 and one s8 tile per operand per K block of 128
// channels.  3x3 taps are spatially shifted TMA boxes over a 5-D tensor map;
// the zero fill of out-of-range coordinates is the convolution's zero padding.
//
// Warp roles (320 threads): warp 0 issues TMA, warp 1 owns TMEM and issues
// the MMAs, warps 2-9 run the epilogue (two warps per TMEM lane quarter, each
// taking half of the accumulator columns).
#include "umma.cuh"
#include "uf_common.cuh"
#include "conv_tc.h"

#include <cuda_runtime.h>
#include <cstdio>
#include <mutex>
#include <string>

namespace ufb {

constexpr int kBM = 128;   // output pixels per tile
constexpr int kBK = 128;   // input channels (bytes per plane row) per K block
constexpr int kThreads = 320;

struct ConvTcArgs {
    Act out;
    Epilogue epi;
    int co, ci;
    int taps_h, taps_w, pad_h, pad_w;
    int cpad;              // channels per tap in the weight matrix (multiple of kBK)
    int n, oh, ow;         // output geometry before any pixel shuffle
    int tile_w, tile_h, tiles_x, tiles_y;
    long long m_total;     // flat mode: output pixels
    Act res1, res2;
    int* status;
};

template <int BN>
struct TcConfig {
    static constexpr int kStages = BN == 128 ? 3 : 4;
    static constexpr uint32_t kABytes = kBM * kBK;
    static constexpr uint32_t kBBytes = BN * kBK;
    static constexpr uint32_t kStageBytes = 2 * kABytes + 2 * kBBytes;
    static constexpr uint32_t kTmemCols = 3 * BN <= 256 ? 256 : 512;
    static constexpr size_t kSmem = size_t(kStages) * kStageBytes + 1024;
};

__device__ __forceinline__ int16_t epilogue_value(int64_t sum, int co, const ConvTcArgs& a) {
    int64_t v = rna_shift(sum, 13);
    if (a.epi.bias) {
        v += a.epi.bias32 ? static_cast<const int32_t*>(a.epi.bias)[co] : static_cast<const int16_t*>(a.epi.bias)[co];
    }
    return sat16(v);
}

// Applies the epilogue to 16 accumulator columns of one pixel row and stores
// them (split NHWC, 16-byte vector stores when the whole chunk is in range).
__device__ __forceinline__ void store_chunk(const ConvTcArgs& args, const uint32_t (&ll)[16], const uint32_t (&xx)[16],
                                            const uint32_t (&hh)[16], int cbase, int img, int oy, int ox,
                                            long long px, bool spatial) {
    const Epilogue& e = args.epi;
    int16_t v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int64_t sum = static_cast<int64_t>(static_cast<int32_t>(ll[j])) +
                            256 * static_cast<int64_t>(static_cast<int32_t>(xx[j])) +
                            65536 * static_cast<int64_t>(static_cast<int32_t>(hh[j]));
        v[j] = cbase + j < args.co ? epilogue_value(sum, cbase + j, args) : int16_t(0);
    }
    const bool full = cbase + 16 <= args.co;
    if (e.wsilu4) {
        // four output channels cbase / 4 .. cbase / 4 + 3
        uint8_t lo[4], hi[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            int32_t s = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) s += __ldg(&e.lut[static_cast<int32_t>(v[4 * g + t]) + 32768]);
            const int16_t r = sat16i(s);
            lo[g] = static_cast<uint8_t>(r & 0xff);
            hi[g] = static_cast<uint8_t>((r >> 8) & 0xff);
        }
        const long long opx = spatial ? args.out.pixel(img, oy, ox) : px;
        const int oc = cbase >> 2;
        uint8_t* dl = args.out.lo(opx) + oc;
        uint8_t* dh = args.out.hi(opx) + oc;
        if (full) {
            *reinterpret_cast<uint32_t*>(dl) = *reinterpret_cast<const uint32_t*>(lo);
            *reinterpret_cast<uint32_t*>(dh) = *reinterpret_cast<const uint32_t*>(hi);
        } else {
            for (int g = 0; g < 4 && 4 * g + cbase < args.co; ++g) {
                dl[g] = lo[g];
                dh[g] = hi[g];
            }
        }
        return;
    }
    if (e.shuffle2) {
        // channel 4c + 2i + j of pixel (oy, ox) -> channel c of pixel (2oy + i, 2ox + j)
        const int c0 = cbase >> 2;
#pragma unroll
        for (int ij = 0; ij < 4; ++ij) {
            const long long opx = args.out.pixel(img, 2 * oy + (ij >> 1), 2 * ox + (ij & 1));
            uint8_t* dl = args.out.lo(opx) + c0;
            uint8_t* dh = args.out.hi(opx) + c0;
            for (int g = 0; g < 4; ++g) {
                if (cbase + 4 * g + ij >= args.co) break;
                const int16_t r = v[4 * g + ij];
                dl[g] = static_cast<uint8_t>(r & 0xff);
                dh[g] = static_cast<uint8_t>((r >> 8) & 0xff);
            }
        }
        return;
    }
    if (e.lut) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __ldg(&e.lut[static_cast<int32_t>(v[j]) + 32768]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const Act& res = r == 0 ? args.res1 : args.res2;
        if (!res.base) continue;
        const long long rpx = spatial ? res.pixel(img, oy, ox) : px;
        const uint8_t* rl = res.lo(rpx) + cbase;
        const uint8_t* rh = res.hi(rpx) + cbase;
        uint8_t bl[16], bh[16];
        if (full) {
            *reinterpret_cast<uint4*>(bl) = *reinterpret_cast<const uint4*>(rl);
            *reinterpret_cast<uint4*>(bh) = *reinterpret_cast<const uint4*>(rh);
        } else {
            for (int j = 0; j < 16; ++j) {
                bl[j] = cbase + j < args.co ? rl[j] : 0;
                bh[j] = cbase + j < args.co ? rh[j] : 0;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = sat16i(static_cast<int32_t>(v[j]) + join16(bl[j], bh[j]));
    }
    if (e.mulq) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int32_t q = cbase + j < args.co ? __ldg(&e.mulq[cbase + j]) : 0;
            v[j] = sat16(rna_shift(static_cast<int64_t>(v[j]) * q, 9));
        }
    }
    uint8_t ol[16], oh8[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        ol[j] = static_cast<uint8_t>(v[j] & 0xff);
        oh8[j] = static_cast<uint8_t>((v[j] >> 8) & 0xff);
    }
    const long long opx = spatial ? args.out.pixel(img, oy, ox) : px;
    uint8_t* dl = args.out.lo(opx) + cbase;
    uint8_t* dh = args.out.hi(opx) + cbase;
    if (full) {
        *reinterpret_cast<uint4*>(dl) = *reinterpret_cast<const uint4*>(ol);
        *reinterpret_cast<uint4*>(dh) = *reinterpret_cast<const uint4*>(oh8);
    } else {
        for (int j = 0; j < 16 && cbase + j < args.co; ++j) {
            dl[j] = ol[j];
            dh[j] = oh8[j];
        }
    }
}

template <int BN, bool SPATIAL>
__global__ void __launch_bounds__(kThreads, 1)
conv_i16_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const ConvTcArgs args) {
    using Cfg = TcConfig<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full_bar[S];
    __shared__ __align__(8) uint64_t empty_bar[S];
    __shared__ __align__(8) uint64_t accum_bar;
    __shared__ uint32_t tmem_holder;
    __shared__ int consumed;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int co0 = blockIdx.y * BN;

    int img = 0, y0 = 0, x0 = 0;
    long long p0 = 0;
    if (SPATIAL) {
        int t = blockIdx.x;
        const int tx = t % args.tiles_x;
        t /= args.tiles_x;
        const int ty = t % args.tiles_y;
        img = t / args.tiles_y;
        x0 = tx * args.tile_w;
        y0 = ty * args.tile_h;
    } else {
        p0 = static_cast<long long>(blockIdx.x) * kBM;
    }
    const int kb_per_tap = (args.ci + kBK - 1) / kBK;
    const int num_k = args.taps_h * args.taps_w * kb_per_tap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&accum_bar, 1);
        consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_holder, Cfg::kTmemCols);
        tmem_relinquish();
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
            for (int k = 0; k < num_k; ++k) {
                const int s = k % S;
                const uint32_t round = k / S;
                if (k >= S && !mbar_wait(&empty_bar[s], (round - 1) & 1, args.status, 1)) break;
                const int tap = k / kb_per_tap, cb = k - tap * kb_per_tap;
                const int ky = tap / args.taps_w, kx = tap - ky * args.taps_w;
                uint8_t* st = smem + size_t(s) * Cfg::kStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], Cfg::kStageBytes);
                const int c0 = cb * kBK;
                if (SPATIAL) {
                    const int ix = x0 + kx - args.pad_w, iy = y0 + ky - args.pad_h;
                    tma_load_5d(st, &mapA, &full_bar[s], c0, 0, ix, iy, img);
                    tma_load_5d(st + Cfg::kABytes, &mapA, &full_bar[s], c0, 1, ix, iy, img);
                } else {
                    tma_load_3d(st, &mapA, &full_bar[s], c0, 0, static_cast<int>(p0));
                    tma_load_3d(st + Cfg::kABytes, &mapA, &full_bar[s], c0, 1, static_cast<int>(p0));
                }
                const int kw = tap * args.cpad + c0;
                tma_load_3d(st + 2 * Cfg::kABytes, &mapB, &full_bar[s], kw, co0, 0);
                tma_load_3d(st + 2 * Cfg::kABytes + Cfg::kBBytes, &mapB, &full_bar[s], kw, co0, 1);
                issued = k + 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t i_uu = i8_idesc(kBM, BN, false, false);
            constexpr uint32_t i_su = i8_idesc(kBM, BN, true, false);
            constexpr uint32_t i_us = i8_idesc(kBM, BN, false, true);
            constexpr uint32_t i_ss = i8_idesc(kBM, BN, true, true);
            const uint32_t d_ll = tmem, d_x = tmem + BN, d_hh = tmem + 2 * BN;
            int k = 0;
            for (; k < num_k; ++k) {
                const int s = k % S;
                const uint32_t round = k / S;
                if (!mbar_wait(&full_bar[s], round & 1, args.status, 2)) break;
                tc_fence_after();
                const uint32_t base = smem_u32(smem + size_t(s) * Cfg::kStageBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 32; ++kk) {
                    const uint64_t a_lo = sw128_desc(base + kk * 32);
                    const uint64_t a_hi = sw128_desc(base + Cfg::kABytes + kk * 32);
                    const uint64_t b_lo = sw128_desc(base + 2 * Cfg::kABytes + kk * 32);
                    const uint64_t b_hi = sw128_desc(base + 2 * Cfg::kABytes + Cfg::kBBytes + kk * 32);
                    const uint32_t acc = (k > 0 || kk > 0) ? 1u : 0u;
                    mma_i8(d_ll, a_lo, b_lo, i_uu, acc);
                    mma_i8(d_x, a_hi, b_lo, i_su, acc);
                    mma_i8(d_x, a_lo, b_hi, i_us, 1u);
                    mma_i8(d_hh, a_hi, b_hi, i_ss, acc);
                }
                mma_commit(&empty_bar[s]);
            }
            consumed = k;
            mma_commit(&accum_bar);
        }
        __syncwarp();
    } else {
        const bool ready = mbar_wait(&accum_bar, 0, args.status, 3);
        tc_fence_after();
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        bool valid;
        long long px;
        int oy = 0, ox = 0;
        if (SPATIAL) {
            const int ty = row / args.tile_w, tx = row - ty * args.tile_w;
            oy = y0 + ty;
            ox = x0 + tx;
            valid = oy < args.oh && ox < args.ow;
            px = 0;
        } else {
            px = p0 + row;
            valid = px < args.m_total;
        }
        valid = valid && ready;
        constexpr int kHalfCols = BN / 2;
        for (int col = half * kHalfCols; col < (half + 1) * kHalfCols; col += 16) {
            uint32_t ll[16], xx[16], hh[16];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + col;
            tmem_ld16(taddr, ll);
            tmem_ld16(taddr + BN, xx);
            tmem_ld16(taddr + 2 * BN, hh);
            tmem_wait_ld();
            const int cbase = co0 + col;
            if (valid && cbase < args.co) store_chunk(args, ll, xx, hh, cbase, img, oy, ox, px, SPATIAL);
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // Drain TMA loads that were issued but never consumed (abort path only),
        // so no copy into this CTA's shared memory outlives the CTA.
        for (int k = consumed; k < issued; ++k) {
            mbar_wait(&full_bar[k % S], (k / S) & 1, args.status, 4);
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// ------------------------------------------------------------------ host ----

namespace {

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

template <int BN, bool SPATIAL>
cudaError_t launch(const CUtensorMap& a, const CUtensorMap& b, const ConvTcArgs& args, dim3 grid,
                   cudaStream_t stream) {
    using Cfg = TcConfig<BN>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(conv_i16_tc_kernel<BN, SPATIAL>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(Cfg::kSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    conv_i16_tc_kernel<BN, SPATIAL><<<grid, kThreads, Cfg::kSmem, stream>>>(a, b, args);
    return cudaGetLastError();
}

}  // namespace

bool tc_weight_map(const TcWeights& w, int bn, CUtensorMap* map, std::string& err) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(w.kpad), static_cast<cuuint64_t>(w.co), 2};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(w.kpad),
                                   static_cast<cuuint64_t>(w.kpad) * static_cast<cuuint64_t>(w.co)};
    const cuuint32_t box[3] = {kBK, static_cast<cuuint32_t>(bn), 1};
    return encode(map, w.planes, 3, dims, strides, box, err);
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
    if (epi.shuffle2 && (epi.lut || epi.wsilu4 || epi.res1.base || epi.res2.base || epi.mulq)) {
        err = "pixel-shuffle store supports the plain epilogue only";
        return -1;
    }
    if (static_cast<long long>(w.kh) * w.kw * w.ci > 32768) {
        err = "reduction exceeds the exact s32 accumulator bound";
        return -1;
    }
    const bool flat = w.kh == 1 && w.kw == 1 && pad_h == 0 && pad_w == 0 && in.dense() && out.dense() &&
                      !epi.shuffle2 && (!epi.res1.base || epi.res1.dense()) && (!epi.res2.base || epi.res2.dense()) &&
                      in.pixels() < (1ll << 31);
    ConvTcArgs args{};
    args.out = out;
    args.epi = epi;
    args.res1 = epi.res1;
    args.res2 = epi.res2;
    args.co = w.co;
    args.ci = w.ci;
    args.taps_h = w.kh;
    args.taps_w = w.kw;
    args.pad_h = pad_h;
    args.pad_w = pad_w;
    args.cpad = w.cpad;
    args.n = in.n;
    args.oh = oh;
    args.ow = ow;
    args.status = status;

    const int bn = w.co <= 64 ? 64 : 128;
    const CUtensorMap* bmap = bn == 128 ? &w.map128 : &w.map64;
    CUtensorMap amap;
    dim3 grid;
    if (flat) {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(in.c), 2, static_cast<cuuint64_t>(in.pixels())};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(in.pitch), static_cast<cuuint64_t>(2 * in.pitch)};
        const cuuint32_t box[3] = {kBK, 1, kBM};
        if (!encode(&amap, in.base, 3, dims, strides, box, err)) return -1;
        args.m_total = in.pixels();
        grid = dim3(static_cast<unsigned>((in.pixels() + kBM - 1) / kBM), (w.co + bn - 1) / bn, 1);
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
        grid = dim3(static_cast<unsigned>(args.tiles_x * args.tiles_y * in.n), (w.co + bn - 1) / bn, 1);
    }
    cudaError_t e;
    if (bn == 128)
        e = flat ? launch<128, false>(amap, *bmap, args, grid, stream) : launch<128, true>(amap, *bmap, args, grid, stream);
    else
        e = flat ? launch<64, false>(amap, *bmap, args, grid, stream) : launch<64, true>(amap, *bmap, args, grid, stream);
    if (e != cudaSuccess) {
        err = std::string("conv launch failed: ") + cudaGetErrorString(e);
        return -1;
    }
    return 0;
}

}  // namespace ufb
