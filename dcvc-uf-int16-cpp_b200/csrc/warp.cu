// Fixed-point backward bilinear warp (ufb_warp).  The
// reference's only warp is the float DCVC-FM kernel (src/dcvc_fm_motion.cu:
// 29-76, not on the UF HT-L path); this is the integer restatement of its
// semantics that oracle/uf_oracle.c:ufo_warp specifies: sample position =
// pixel + flow (int16 Q9, channel 0 = x, 1 = y), clamped to the border,
// x0 = floor, x1 = min(x0 + 1, W - 1), 9-bit fractions, Q18 products,
// rna(sum / 2^18) (always inside the int16 range: the weights sum to 2^18).
//
// Layout: NCHW int16 feature planes, as the float kernel takes them.  A CTA
// owns a 64 x 16 output tile and a slab of 8 channels.  From the tile's flow it
// finds the source window every bilinear footprint of the tile falls in (its
// bounding box), and TMA brings that window for two channels at a time into a
// two-stage shared-memory ring (boxes of 128 px x 8 rows x 2 planes, only as
// many row blocks as the window needs); the gathers then read shared memory,
// and each thread writes its two horizontally adjacent outputs per row as one
// 32-bit store, so every output row leaves the SM as whole coalesced lines.
// A CTA whose window does not fit the ring (flow spread above ~60 px inside
// one tile), or a tensor that TMA cannot describe (W not a multiple of 8,
// unaligned base, odd channel count), gathers straight from global memory
// with the same arithmetic.
#include "kernels.h"
#include "umma.cuh"

#include <climits>
#include <mutex>
#include <string>
#include <type_traits>

namespace ufb {

namespace {

constexpr int kTW = 64, kTH = 16;              // output tile
constexpr int kThreads = 256;                  // 8 warps x (2 rows x 64 px)
constexpr int kSlab = 8;                       // channels per CTA
constexpr int kCG = 2;                         // channels per TMA stage
constexpr int kStages = 2;
constexpr int kBoxW = 128;                     // window width limit (px)
constexpr int kRowBlk = 8;                     // rows per TMA box
constexpr int kMaxRows = 64;                   // window height limit
constexpr int kBlkElems = kCG * kRowBlk * kBoxW;               // one box: 2048 int16
constexpr int kStageElems = (kMaxRows / kRowBlk) * kBlkElems;  // 16384 int16 = 32 KB
constexpr int kSmemBytes = kStages * kStageElems * 2;
constexpr int kWarpTimeoutCode = 11;

// rna(sum / 2^18) of the Q18 bilinear sum s = wa v00 + wb v10 + wc v01 + wd v11
// (weights (512 - ax)(512 - ay), (512 - ax) ay, ax (512 - ay), ax ay; they sum
// to 2^18, so |s| < 2^33 and the result is inside the int16 range).  The sum
// needs 35 bits: four 32 x 32 -> 64-bit multiply-adds form it exactly, and
// rna(s / 2^18) = floor((s + 2^17 - [s < 0]) / 2^18) is one 64-bit add and one
// funnel shift.
__device__ __forceinline__ int32_t bilerp_q18(int32_t v00, int32_t v01, int32_t v10, int32_t v11, int32_t wa,
                                              int32_t wb, int32_t wc, int32_t wd) {
    const int64_t s = static_cast<int64_t>(wa) * v00 + static_cast<int64_t>(wb) * v10 +
                      static_cast<int64_t>(wc) * v01 + static_cast<int64_t>(wd) * v11;
    const int32_t neg = static_cast<int32_t>(s >> 32) >> 31;
    return static_cast<int32_t>((s + ((1 << 17) + neg)) >> 18);
}

__device__ __forceinline__ uint32_t pack_pair(int32_t a, int32_t b) {
    return (static_cast<uint32_t>(a) & 0xffffu) | (static_cast<uint32_t>(b) << 16);
}

// Sign-extending 16-bit shared-memory load at addr + OFF (an immediate).
template <int OFF>
__device__ __forceinline__ int32_t lds_s16(uint32_t addr) {
    int32_t v;
    asm volatile("ld.shared.s16 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(OFF) : "memory");
    return v;
}

__device__ __forceinline__ void store_pair(int16_t* row, int x, int w, bool pair_ok, bool v0, bool v1, int32_t a,
                                           int32_t b) {
    if (pair_ok && v0 && v1) {
        *reinterpret_cast<uint32_t*>(row + x) = pack_pair(a, b);
    } else {
        if (v0) row[x] = static_cast<int16_t>(a);
        if (v1) row[x + 1] = static_cast<int16_t>(b);
    }
}

__global__ void __launch_bounds__(kThreads, 3)
    warp_tile_kernel(const __grid_constant__ CUtensorMap map, int map_ok, const int16_t* __restrict__ feature,
                     const int16_t* __restrict__ flow, int16_t* __restrict__ out, int c, int h, int w, int slabs,
                     int pair_ok, int* status) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    int16_t* ring = reinterpret_cast<int16_t*>(smem_raw);
    __shared__ __align__(8) uint64_t full[kStages];
    __shared__ int window[4];

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int b = blockIdx.z / slabs, slab = blockIdx.z - b * slabs;
    const int c0 = slab * kSlab;
    const int cn = min(kSlab, c - c0);
    const int tx0 = blockIdx.x * kTW, ty0 = blockIdx.y * kTH;
    const long long plane = static_cast<long long>(h) * w;
    const int xs = tx0 + 2 * lane;

    if (tid == 0) {
        window[0] = INT_MAX;
        window[1] = -1;
        window[2] = INT_MAX;
        window[3] = -1;
    }
    // per pixel: p = row (0, 1) * 2 + column (0, 1)
    int x0[4], x1[4], y0[4], y1[4], wa[4], wb[4], wc[4], wd[4];
    bool valid[4];
    int mnx = INT_MAX, mxx = -1, mny = INT_MAX, mxy = -1;
    const int16_t* fl = flow + static_cast<long long>(b) * 2 * plane;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int x = xs + (p & 1), y = ty0 + 2 * wid + (p >> 1);
        valid[p] = x < w && y < h;
        x0[p] = x1[p] = y0[p] = y1[p] = wa[p] = wb[p] = wc[p] = wd[p] = 0;
        if (valid[p]) {
            const long long i = static_cast<long long>(y) * w + x;
            int px = x * 512 + static_cast<int>(__ldg(fl + i));
            int py = y * 512 + static_cast<int>(__ldg(fl + plane + i));
            px = px < 0 ? 0 : (px > (w - 1) * 512 ? (w - 1) * 512 : px);
            py = py < 0 ? 0 : (py > (h - 1) * 512 ? (h - 1) * 512 : py);
            x0[p] = px >> 9;
            y0[p] = py >> 9;
            x1[p] = min(x0[p] + 1, w - 1);
            y1[p] = min(y0[p] + 1, h - 1);
            const int ax = px & 511, ay = py & 511;
            wa[p] = (512 - ax) * (512 - ay);
            wb[p] = (512 - ax) * ay;
            wc[p] = ax * (512 - ay);
            wd[p] = ax * ay;
            mnx = min(mnx, x0[p]);
            mxx = max(mxx, x1[p]);
            mny = min(mny, y0[p]);
            mxy = max(mxy, y1[p]);
        }
    }
    __syncthreads();
    mnx = __reduce_min_sync(0xffffffffu, mnx);
    mxx = __reduce_max_sync(0xffffffffu, mxx);
    mny = __reduce_min_sync(0xffffffffu, mny);
    mxy = __reduce_max_sync(0xffffffffu, mxy);
    if (lane == 0) {
        atomicMin(&window[0], mnx);
        atomicMax(&window[1], mxx);
        atomicMin(&window[2], mny);
        atomicMax(&window[3], mxy);
    }
    __syncthreads();
    const int wx0 = window[0] & ~7;  // TMA: x * 2 bytes on a 16-byte boundary
    const int wy0 = window[2];
    const int ww = window[1] - wx0 + 1, wh = window[3] - wy0 + 1;
    const bool use_tma = map_ok && ww <= kBoxW && wh <= kMaxRows;

    const long long out_base = (static_cast<long long>(b) * c + c0) * plane;
    int16_t* orow0 = out + out_base + static_cast<long long>(ty0 + 2 * wid) * w;
    int16_t* orow1 = orow0 + w;

    if (!use_tma) {
        const int16_t* f = feature + out_base;
        for (int ch = 0; ch < cn; ++ch) {
            const int16_t* fp = f + ch * plane;
            int32_t r[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                r[p] = 0;
                if (valid[p]) {
                    const int16_t* a = fp + static_cast<long long>(y0[p]) * w;
                    const int16_t* bb = fp + static_cast<long long>(y1[p]) * w;
                    r[p] = bilerp_q18(__ldg(a + x0[p]), __ldg(a + x1[p]), __ldg(bb + x0[p]), __ldg(bb + x1[p]),
                                      wa[p], wb[p], wc[p], wd[p]);
                }
            }
            store_pair(orow0 + ch * plane, xs, w, pair_ok, valid[0], valid[1], r[0], r[1]);
            store_pair(orow1 + ch * plane, xs, w, pair_ok, valid[2], valid[3], r[2], r[3]);
        }
        return;
    }

    // shared-memory byte offsets of the four footprint samples inside a stage,
    // layout [row block][channel][8 rows][128 px]; the stage and channel parts
    // of an address are compile-time immediates of the loads below
    uint32_t a00[4], a01[4], a10[4], a11[4];
    const uint32_t ring_s = smem_u32(ring);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const int r0 = y0[p] - wy0, r1 = y1[p] - wy0, xx = x0[p] - wx0, dx = x1[p] - x0[p];
        const uint32_t o0 = 2u * ((r0 >> 3) * kBlkElems + (r0 & 7) * kBoxW + xx);
        const uint32_t o1 = 2u * ((r1 >> 3) * kBlkElems + (r1 & 7) * kBoxW + xx);
        a00[p] = valid[p] ? ring_s + o0 : ring_s;
        a01[p] = valid[p] ? ring_s + o0 + 2u * dx : ring_s;
        a10[p] = valid[p] ? ring_s + o1 : ring_s;
        a11[p] = valid[p] ? ring_s + o1 + 2u * dx : ring_s;
    }
    const int blocks = (wh + kRowBlk - 1) / kRowBlk;
    const uint32_t stage_bytes = static_cast<uint32_t>(blocks) * kBlkElems * 2;
    const int stages = cn / kCG;
    const int plane0 = b * c + c0;
    // interior tiles with paired stores need no per-pixel checks
    const bool full_tile = pair_ok && tx0 + kTW <= w && ty0 + kTH <= h;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
        prefetch_tmap(&map);
    }
    __syncthreads();
    auto issue = [&](int s) {
        int16_t* dst = ring + (s % kStages) * kStageElems;
        uint64_t* bar = &full[s % kStages];
        mbar_arrive_expect_tx(bar, stage_bytes);
        for (int r = 0; r < blocks; ++r)
            tma_load_3d(dst + r * kBlkElems, &map, bar, wx0 * 2, wy0 + r * kRowBlk, plane0 + s * kCG);
    };
    int issued = 0;
    if (tid == 0)
        for (; issued < min(kStages, stages); ++issued) issue(issued);
    bool alive = true;
    int16_t* o_row0 = orow0 + xs;
    int16_t* o_row1 = orow1 + xs;
    // one stage: kCG channels from ring buffer BUF
    auto consume = [&](auto buf_tag, int s) {
        constexpr int BUF = decltype(buf_tag)::value;
        if (alive) alive = mbar_wait(&full[BUF], (s / kStages) & 1, status, kWarpTimeoutCode);
        if (alive) {
#pragma unroll
            for (int cc = 0; cc < kCG; ++cc) {
                constexpr int kBufBytes = BUF * kStageElems * 2;
                int32_t r[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    int32_t v00, v01, v10, v11;
                    if (cc == 0) {
                        v00 = lds_s16<kBufBytes>(a00[p]);
                        v01 = lds_s16<kBufBytes>(a01[p]);
                        v10 = lds_s16<kBufBytes>(a10[p]);
                        v11 = lds_s16<kBufBytes>(a11[p]);
                    } else {
                        v00 = lds_s16<kBufBytes + kRowBlk * kBoxW * 2>(a00[p]);
                        v01 = lds_s16<kBufBytes + kRowBlk * kBoxW * 2>(a01[p]);
                        v10 = lds_s16<kBufBytes + kRowBlk * kBoxW * 2>(a10[p]);
                        v11 = lds_s16<kBufBytes + kRowBlk * kBoxW * 2>(a11[p]);
                    }
                    r[p] = bilerp_q18(v00, v01, v10, v11, wa[p], wb[p], wc[p], wd[p]);
                }
                if (full_tile) {
                    *reinterpret_cast<uint32_t*>(o_row0) = pack_pair(r[0], r[1]);
                    *reinterpret_cast<uint32_t*>(o_row1) = pack_pair(r[2], r[3]);
                } else {
                    store_pair(o_row0 - xs, xs, w, pair_ok, valid[0], valid[1], r[0], r[1]);
                    store_pair(o_row1 - xs, xs, w, pair_ok, valid[2], valid[3], r[2], r[3]);
                }
                o_row0 += plane;
                o_row1 += plane;
            }
        }
        __syncthreads();  // every thread is done with this stage's buffer
        if (tid == 0 && alive && issued < stages) issue(issued++);
    };
    static_assert(kStages == 2, "the stage loop alternates between two ring buffers");
    for (int s = 0; s < stages; s += 2) {
        consume(std::integral_constant<int, 0>{}, s);
        if (s + 1 < stages) consume(std::integral_constant<int, 1>{}, s + 1);
    }
    // after a timeout, let this CTA's own copies in flight land (bounded)
    // before its shared memory is released
    if (tid == 0 && !alive) {
        for (int s = 0; s < issued; ++s) mbar_wait(&full[s % kStages], (s / kStages) & 1, status, kWarpTimeoutCode);
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn warp_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

cudaError_t warp_fixed(int16_t* out, const int16_t* feature, const int16_t* flow, int n, int c, int h, int w,
                       int* status, cudaStream_t s) {
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(warp_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    });
    if (attr_err != cudaSuccess) return attr_err;
    // TMA describes the planes as bytes: rows of w * 2 bytes (a multiple of 16),
    // planes of h * w * 2, a 16-byte aligned base, boxes of 2 whole planes.
    CUtensorMap map{};
    int map_ok = 0;
    if (w % 8 == 0 && c % kCG == 0 && reinterpret_cast<uintptr_t>(feature) % 16 == 0) {
        if (auto fn = warp_encode_fn()) {
            const cuuint64_t dims[3] = {static_cast<cuuint64_t>(w) * 2, static_cast<cuuint64_t>(h),
                                        static_cast<cuuint64_t>(n) * c};
            const cuuint64_t strides[2] = {static_cast<cuuint64_t>(w) * 2, static_cast<cuuint64_t>(h) * w * 2};
            const cuuint32_t box[3] = {kBoxW * 2, kRowBlk, kCG};
            const cuuint32_t elem[3] = {1, 1, 1};
            map_ok = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int16_t*>(feature), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
    }
    const int slabs = (c + kSlab - 1) / kSlab;
    const dim3 grid((w + kTW - 1) / kTW, (h + kTH - 1) / kTH, n * slabs);
    const int pair_ok = w % 2 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0;
    warp_tile_kernel<<<grid, kThreads, kSmemBytes, s>>>(map, map_ok, feature, flow, out, c, h, w, slabs, pair_ok,
                                                        status);
    return cudaGetLastError();
}

}  // namespace ufb
