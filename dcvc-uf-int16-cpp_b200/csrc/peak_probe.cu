// Dense tcgen05 kind::i8 throughput probe: the int8 tensor-pipe peak that the
// convolution roofline is measured against (no published or driver-measured
// int8 figure exists for this part).  One CTA per SM issues back-to-back
// M=128, N=256, K=32 u8 x u8 MMAs from resident shared-memory tiles into one
// TMEM accumulator; no global memory traffic.  The caller times the launch.
#include "uf_b200.h"
#include "capi_util.h"
#include "umma.cuh"

using namespace ufb;

namespace {

__global__ void __launch_bounds__(128, 1) i8_peak_kernel(int iters, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_holder;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < (128 + 256) * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0x01010101u, 0, 0x02020202u, 0);
    if (threadIdx.x == 0) {
        mbar_init(&done_bar, 1);
        fence_mbar_init();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 0) {
        tmem_alloc(&tmem_holder, 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_holder;
    if (warp == 0) {
        if (lane == 0) {
            constexpr uint32_t idesc = i8_idesc(128, 256, false, false);
            const uint32_t a = smem_u32(smem), b = smem_u32(smem + 128 * 128);
            for (int i = 0; i < iters; ++i) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_i8(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), idesc, (i | kk) ? 1u : 0u);
            }
            mma_commit(&done_bar);
            mbar_wait(&done_bar, 0, status, 5);
        }
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace

extern "C" int ufb_probe_i8_peak(int iters, int ctas, void* stream, int64_t* int8_ops) {
    clear_error();
    if (iters <= 0 || ctas <= 0) return err(UFB_EINVAL, "iters and ctas must be positive");
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return last_code();
    int* status = device_status(device);
    if (!status) return last_code();
    // 120 KB keeps one probe CTA per SM
    const int smem = 120 * 1024;
    if (!cuda_ok(cudaFuncSetAttribute(i8_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "smem attribute"))
        return last_code();
    i8_peak_kernel<<<ctas, 128, smem, static_cast<cudaStream_t>(stream)>>>(iters, status);
    if (!cuda_ok(cudaGetLastError(), "peak probe launch")) return last_code();
    if (int8_ops) *int8_ops = static_cast<int64_t>(ctas) * iters * 4 * 128 * 256 * 32 * 2;
    return UFB_OK;
}
