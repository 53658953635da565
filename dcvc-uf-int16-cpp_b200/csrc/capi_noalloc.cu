// ufb_conv2d_noalloc: the uf_conv replacement for callers that must not
// allocate GPU memory while they process (see include/uf_b200.h).
//
// ufb_conv2d needs three scratch buffers per call -- the input in split NHWC,
// the weights as tensor-core planes and the output in split NHWC -- and takes
// them from cudaMallocAsync.  This variant carves them out of one fixed,
// file-scope device array instead, sized kNoAllocScratchBytes.  The array is
// part of the library image: every GPU that loads the library holds it until
// the process exits.
#include "uf_b200.h"

#include "capi_util.h"
#include "conv_tc.h"
#include "kernels.h"

#include <mutex>
#include <string>
#include <vector>

using namespace ufb;

namespace {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(UFB_NOALLOC_SCRATCH_BYTES);

// Shared by every call on a device; holds the last call's contents.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mutex;
std::vector<uint8_t*> g_device_ptr;  // per device ordinal, null until resolved

// Host code may not use g_noalloc_scratch as an address (it names the host
// shadow of the symbol).  Resolve the device address once per device, with
// that device current.
uint8_t* scratch_for_current_device() {
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (static_cast<size_t>(device) >= g_device_ptr.size()) g_device_ptr.resize(device + 1, nullptr);
    if (!g_device_ptr[device]) {
        void* p = nullptr;
        if (!cuda_ok(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)")) return nullptr;
        g_device_ptr[device] = static_cast<uint8_t*>(p);
    }
    return g_device_ptr[device];
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int ufb_conv2d_noalloc(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co,
                                  int kh, int kw, const void* bias, int bias_bits, int sh, int sw, int ph, int pw,
                                  int groups, int16_t* out, void* stream) {
    clear_error();
    if (!bias) bias_bits = 0;
    int oh = 0, ow = 0;
    // the same argument checks as ufb_conv2d
    if (!check_conv(x, n, ci, h, w, weight, co, kh, kw, bias_bits, sh, sw, ph, pw, groups, out, oh, ow))
        return last_code();
    auto s = static_cast<cudaStream_t>(stream);
    // first call on this device: resolve the scratch array's device address
    uint8_t* base = scratch_for_current_device();
    if (!base) return last_code();

    // (a full 8192-term reduction with an int32 bias could wrap the 32-bit epilogue sum)
    const long long k_total = static_cast<long long>(ci) * kh * kw;
    const bool tensor_core = groups == 1 && sh == 1 && sw == 1 &&
                             (k_total < kTcMaxReduction || (k_total == kTcMaxReduction && bias_bits != 32));
    if (!tensor_core) {
        // the direct int64 kernel reads NCHW in place and needs no scratch
        return cuda_ok(conv_direct(out, x, weight, bias_bits ? bias : nullptr, bias_bits == 32, n, ci, co, h, w, oh,
                                   ow, kh, kw, sh, sw, ph, pw, groups, s),
                       "direct convolution")
                   ? UFB_OK
                   : last_code();
    }
    const int cip = round_up(ci, 16), cop = round_up(co, 16);
    const size_t x_bytes = align256(static_cast<size_t>(n) * h * w * 2 * cip);
    const size_t w_bytes = align256(tc_weight_bytes(co, ci, kh, kw, 128));
    const size_t o_bytes = align256(static_cast<size_t>(n) * oh * ow * 2 * cop);
    if (x_bytes + w_bytes + o_bytes > kNoAllocScratchBytes)
        return err(UFB_ERANGE, "convolution needs " + std::to_string(x_bytes + w_bytes + o_bytes) +
                                   " scratch bytes; ufb_conv2d_noalloc is limited to " +
                                   std::to_string(kNoAllocScratchBytes) + " (UFB_NOALLOC_SCRATCH_BYTES)");
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return last_code();
    // the pipeline-timeout status word is a device variable too (no allocation)
    int* status = device_status(device);
    if (!status) return last_code();
    // Nothing in the scratch must start at zero: the layout conversion and the
    // weight preparation overwrite every byte the convolution reads (channels
    // past ci are outside the TMA tensor extent and read as zero), and the
    // epilogue writes every output byte that is converted back.
    TcWeights tw;
    std::string msg;
    // unsigned byte split: valid for any weights, needs no host inspection
    if (!tc_prepare(tw, weight, co, ci, kh, kw, false, 128, base + x_bytes, s, msg)) return err(UFB_ECUDA, msg);
    const Act in = make_act(base, n, h, w, ci, cip);
    const Act ov = make_act(base + x_bytes + w_bytes, n, oh, ow, co, cop);
    if (!cuda_ok(nchw_to_split(x, n, ci, h, w, 1, in, s), "input layout")) return last_code();
    Epilogue epi{};
    epi.bias = bias_bits ? bias : nullptr;
    epi.bias32 = bias_bits == 32;
    if (conv_tc_run(tw, in, ov, epi, ph, pw, s, status, msg) != 0) return err(UFB_ECUDA, msg);
    if (!cuda_ok(split_to_nchw(ov, 1, out, s), "output layout")) return last_code();
    return UFB_OK;
}
