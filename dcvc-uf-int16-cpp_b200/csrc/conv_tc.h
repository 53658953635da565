// Host interface of the tcgen05 INT16 convolution (conv_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <string>

#include "uf_common.cuh"

namespace ufb {

// Device-resident convolution weights prepared for the tensor-core kernel:
// two planes [2][co][kpad] bytes -- plane 0 holds the low bytes (u8), plane 1
// the high bytes (s8) -- with k = (ky * kw + kx) * cpad + c and zero padding
// for c >= ci.  cpad = ci rounded up to 128, kpad = kh * kw * cpad.
struct TcWeights {
    uint8_t* planes = nullptr;
    int co = 0, ci = 0, kh = 0, kw = 0, cpad = 0, kpad = 0;
    CUtensorMap map128{};  // TMA map with a 128-row box
    CUtensorMap map64{};   // TMA map with a 64-row box
};

bool tc_weight_map(const TcWeights& w, int bn, CUtensorMap* map, std::string& err);

// out = epilogue(conv(in, w)), stride 1, zero padding (pad_h, pad_w).
// Both views must have 16-byte aligned pitch and base.  Asynchronous on
// `stream`; pipeline timeouts are reported through *status.
int conv_tc_run(const TcWeights& w, const Act& in, const Act& out, const Epilogue& epi, int pad_h, int pad_w,
                cudaStream_t stream, int* status, std::string& err);

}  // namespace ufb
