// Host launchers of the model-level kernels (engine_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "uf_common.cuh"

namespace ufb {

cudaError_t copy_channels(const Act& src, const Act& dst, cudaStream_t s);
cudaError_t fill_zero(const Act& dst, cudaStream_t s);
cudaError_t symbols_to_split(const int8_t* sym, const Act& out, cudaStream_t s);
cudaError_t split_to_symbols(const Act& in, int8_t* sym, cudaStream_t s);
cudaError_t mul_unshuffle2(const Act& in, const int16_t* q, const Act& out, cudaStream_t s);
cudaError_t mul_channels(const Act& in, const int16_t* q, const Act& out, cudaStream_t s);
cudaError_t yhat(const Act& restored, const Act& qraw, const Act& out, cudaStream_t s);
// out = lut[in] (groups 1) or the wsilu4 reduction of groups of 4 channels (groups 4)
cudaError_t lut_split(const Act& in, const int16_t* lut, int groups, const Act& out, cudaStream_t s);

int prior_blocks_per_stream(int channels, int h, int w);
// count + per-stream scan: block_counts becomes per-block offsets, totals[n]
cudaError_t prior_scan(int channels, int h, int w, int n, int part, const Act& scales, int thr, int* block_counts,
                       int* totals, cudaStream_t s);
cudaError_t prior_indexes(int channels, int h, int w, int n, int part, const Act& scales, int thr,
                          const int* offsets, const uint8_t* scale_index, uint8_t* indexes, long long cap,
                          cudaStream_t s);
cudaError_t prior_restore(int channels, int h, int w, int n, int part, const Act& scales, const Act& means, int thr,
                          const int* offsets, const int8_t* symbols, long long cap, const Act& restored,
                          cudaStream_t s);
cudaError_t prior_encode(int channels, int h, int w, int n, int part, const Act& scales, const Act& means,
                         const Act& yenc, int thr, const int* offsets, const uint8_t* scale_index, int16_t* packed,
                         long long cap, const Act& restored, cudaStream_t s);
cudaError_t raw_frame(const Act& head, int height, int width, uint8_t* out, long long frame_bytes, cudaStream_t s);
cudaError_t bytes_to_split(const uint8_t* x, int n, int c, int h, int w, int f, const Act& out, cudaStream_t s);

cudaError_t reciprocal_q(const Act& qraw, const Act& out, cudaStream_t s);
cudaError_t mul_elementwise(const Act& x, const Act& q, const Act& out, cudaStream_t s);
cudaError_t pad_replicate(const Act& src, const Act& dst, cudaStream_t s);
cudaError_t bytes_to_split_padded(const uint8_t* x, int n, int c, int h, int w, int hp, int wp, int f, const Act& out,
                                  cudaStream_t s);

}  // namespace ufb
