// Host launchers of the memory-bound kernels (kernels_simt.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "uf_common.cuh"

namespace ufb {

cudaError_t nchw_to_split(const int16_t* x, int n, int c, int h, int w, int f, const Act& out, cudaStream_t s);
cudaError_t split_to_nchw(const Act& in, int f, int16_t* out, cudaStream_t s);
cudaError_t conv_direct(int16_t* out, const int16_t* x, const int16_t* weight, const void* bias, int bias32, int n,
                        int ci, int co, int h, int w, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                        int groups, cudaStream_t s);
// Depthwise 3x3, stride 1, padding 1 on split views (dwconv.cu); a bounded
// wait that gives up records a code in *status (9: a window load, 11: a
// buffer release, 10: the drain of a load in flight on the way out).
// narrow: the layer passed dw_narrow_ok, so every sum runs in one int32.
cudaError_t dwconv3x3(const Act& in, const Act& out, const int16_t* weight, const int16_t* bias, int* status,
                      cudaStream_t s, bool narrow = false);
// True when, for every channel c of the int16 [channels, 1, 3, 3] weights and
// int16 bias (host data, bias may be null), 32768 sum_k |w| + 4096 +
// 8192 |bias| fits int32: then S + 4096 + 8192 bias does for every input.
bool dw_narrow_ok(const int16_t* weight_host, const int16_t* bias_host, int channels);
cudaError_t ew_add(int16_t* out, const int16_t* a, const int16_t* b, const int16_t* c, const int16_t* d, long long n,
                   cudaStream_t s);
cudaError_t ew_mul(int16_t* out, const int16_t* x, const int16_t* scale, const long long* xs, const long long* ss,
                   cudaStream_t s);
cudaError_t ew_lut16(int16_t* out, const int16_t* x, const int16_t* lut, long long n, cudaStream_t s);
cudaError_t ew_lut8(uint8_t* out, const int16_t* x, const uint8_t* lut, long long n, cudaStream_t s);
cudaError_t ew_bytes(int16_t* out, const uint8_t* x, long long n, cudaStream_t s);
cudaError_t ew_wsilu4(int16_t* out, const int16_t* x, const int16_t* lut, int n, int c4, long long hw,
                      cudaStream_t s);
// Fixed-point backward bilinear warp (warp.cu); a bounded wait that gives up
// records code 11 in *status.
cudaError_t warp_fixed(int16_t* out, const int16_t* feature, const int16_t* flow, int n, int c, int h, int w,
                       int* status, cudaStream_t s);

}  // namespace ufb
