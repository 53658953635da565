// Host interface of the tcgen05 INT16 convolution (conv_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <string>

#include "uf_common.cuh"

namespace ufb {

// Longest reduction (taps x input channels) the tensor-core kernel takes: its
// epilogue recombines the byte-product accumulators in 32-bit arithmetic.
// Longer reductions run on the int64 SIMT path.
constexpr long long kTcMaxReduction = 8192;

// Device-resident convolution weights prepared for the tensor-core kernel.
// Layout: [co_tiles][2][bn][kpad] bytes -- per tile of bn (128) output
// channels, bn rows of the weights' low bytes followed by bn rows of their high bytes,
// k = (ky * kw + kx) * cpad + c, zero rows / columns as padding.
//   unsigned split (any weights):   w = lo + 256 hi, lo u8 = w & 0xff, hi s8 = w >> 8
//   signed split (w <= 32639):      w = lo + 256 hi, lo s8 in [-128, 127], hi s8
// The signed split lets one MMA over the stacked 256 rows produce two partial
// products (see conv_tc.cu), halving the MMA count.
struct TcWeights {
    uint8_t* planes = nullptr;
    int co = 0, ci = 0, kh = 0, kw = 0, cpad = 0, kpad = 0, co_tiles = 0, bn = 128;
    bool signed_split = false;
    // LL + 256 X + 4096 fits int32 for every input (tc_narrow_ok): the epilogue
    // then recombines with one multiply-add less per output and no 5-bit split
    bool narrow = false;
    CUtensorMap map{};  // TMA map over the [co_tiles * 2bn][kpad] byte matrix, bn-row box (one byte block)
};

// Bytes needed for the prepared planes of a [co, ci, kh, kw] convolution.
size_t tc_weight_bytes(int co, int ci, int kh, int kw, int bn);

// Tile width used for a layer (the kernel runs 128-wide output tiles).
int tc_choose_bn(int ci, int kh, int kw, bool signed_split);

// Describe already prepared planes (fields + TMA map; no device work).
bool tc_describe(TcWeights& w, int co, int ci, int kh, int kw, bool signed_split, int bn, uint8_t* planes,
                 std::string& err);

// tc_describe plus the preparation of int16 weights already on the device
// into `planes` (tc_weight_bytes bytes), launched on stream s.
bool tc_prepare(TcWeights& w, const int16_t* weight, int co, int ci, int kh, int kw, bool signed_split, int bn,
                uint8_t* planes, cudaStream_t s, std::string& err);

// Shared-memory window of a 65536-entry lookup table (host data, index
// v + 32768): lut[v] == 0 for every v < start + 1, lut[v] == v for every
// v > hi, and entries [start, start + n) cover the rest (n == 0: no window;
// kernels then read the global table).  Kernels stage the window as the
// differences lut[v] - v, so n is 0 as well when one of them leaves int16.
void tc_lut_window(const int16_t* table, int& start, int& n, int& hi);

// True when a fused table step (LUT or wsilu4 epilogue) of a layer with these
// weights can stage a table window of lut_n entries in shared memory (res_mode:
// the residual epilogue's larger stages; table steps use the others).
bool tc_table_window_fits(const TcWeights& w, int lut_n, bool res_mode = false);

// True when every weight allows the signed split (host data).
bool tc_signed_split_ok(const int16_t* weight_host, size_t count);

// cuTensorMapEncodeTiled for a byte tensor (128-byte swizzle unless given).
bool tc_encode_map(CUtensorMap* map, void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, std::string& err,
                   CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// Caps the persistent grids of the tensor-core and depthwise convolutions at n
// CTAs (0: no cap).  A testing aid: with few CTAs every CTA walks many tiles,
// which exercises both TMEM accumulator sets and every reuse of the depthwise
// window buffers.
void tc_set_max_ctas(int n);
int tc_max_ctas();

// True when, for every output channel o of these int16 [co, ci, kh, kw] weights
// (host data) in the given byte split, sum_k 32768 |wl| + 65280 |wh| + 4096 fits
// int32: then LL + 256 X + 4096 = sum_k wl x + 256 wh xl + 4096 fits int32 for
// every int16 input, and TcWeights::narrow may be set.
bool tc_narrow_ok(const int16_t* weight_host, int co, int ci, int kh, int kw, bool signed_split);

// Process-wide switch for the narrow recombination (default on); off runs every
// layer through the general one.  A testing aid: both give identical outputs.
void tc_set_narrow(bool enable);
bool tc_narrow_enabled();

// out = epilogue(conv(in, w)), zero padding (pad_h, pad_w), stride 1 or 2
// (strided: plain epilogue only).  Both views must have 16-byte aligned pitch
// and base.  Asynchronous on `stream`; pipeline timeouts are reported through
// *status.
int conv_tc_run(const TcWeights& w, const Act& in, const Act& out, const Epilogue& epi, int pad_h, int pad_w,
                cudaStream_t stream, int* status, std::string& err, int stride = 1);

}  // namespace ufb
