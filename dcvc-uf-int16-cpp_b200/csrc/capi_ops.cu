// Operator-level C ABI (include/uf_b200.h): the B200 replacements of the
// reference's CUDA extension functions uf_conv / uf_conv_generic /
// uf_conv_baseline / uf_add / uf_mul / uf_lut / uf_bytes / uf_wsilu4
// (include/uf/cuda_ops.hpp:10-23).  Argument checks follow the reference's
// TORCH_CHECKs in src/cuda/conv.cu:65-83 and src/cuda/elementwise.cu:49-98.
#include "uf_b200.h"

#include "capi_util.h"
#include "conv_tc.h"
#include "kernels.h"

#include <climits>
#include <cstdint>
#include <string>

using namespace ufb;

namespace {

int conv_direct_path(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                     const void* bias, int bias_bits, int sh, int sw, int ph, int pw, int groups, int oh, int ow,
                     int16_t* out, cudaStream_t s) {
    return cuda_ok(conv_direct(out, x, weight, bias_bits ? bias : nullptr, bias_bits == 32, n, ci, co, h, w, oh, ow,
                               kh, kw, sh, sw, ph, pw, groups, s),
                   "direct convolution")
               ? UFB_OK
               : last_code();
}

int conv_tc_path(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                 const void* bias, int bias_bits, int stride, int ph, int pw, int oh, int ow, int16_t* out,
                 cudaStream_t s) {
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return last_code();
    const int cip = round_up(ci, 16), cop = round_up(co, 16);
    StreamBuffer xs(static_cast<size_t>(n) * h * w * 2 * cip, s);
    StreamBuffer wp(tc_weight_bytes(co, ci, kh, kw, 128), s);
    StreamBuffer os(static_cast<size_t>(n) * oh * ow * 2 * cop, s);
    if (!xs.ok() || !wp.ok() || !os.ok()) return err(UFB_ECUDA, "cudaMallocAsync failed for convolution scratch");
    int* status = device_status(device);
    if (!status) return last_code();
    TcWeights tw;
    std::string msg;
    // unsigned byte split: valid for any weights, needs no host inspection
    if (!tc_prepare(tw, weight, co, ci, kh, kw, false, 128, wp.get<uint8_t>(), s, msg)) return err(UFB_ECUDA, msg);
    const Act in = make_act(xs.get<uint8_t>(), n, h, w, ci, cip);
    const Act ov = make_act(os.get<uint8_t>(), n, oh, ow, co, cop);
    if (!cuda_ok(nchw_to_split(x, n, ci, h, w, 1, in, s), "input layout")) return last_code();
    Epilogue epi{};
    epi.bias = bias_bits ? bias : nullptr;
    epi.bias32 = bias_bits == 32;
    if (conv_tc_run(tw, in, ov, epi, ph, pw, s, status, msg, stride) != 0) return err(UFB_ECUDA, msg);
    if (!cuda_ok(split_to_nchw(ov, 1, out, s), "output layout")) return last_code();
    return UFB_OK;
}

// Depthwise 3x3 (stride 1, padding 1): the split-layout depthwise kernel the
// engine uses for DepthConvBlock dc.2, between two layout conversions.
int conv_depthwise_path(const int16_t* x, int n, int c, int h, int w, const int16_t* weight, const void* bias,
                        int16_t* out, cudaStream_t s) {
    const int cp = round_up(c, 16);
    StreamBuffer xs(static_cast<size_t>(n) * h * w * 2 * cp, s);
    StreamBuffer os(static_cast<size_t>(n) * h * w * 2 * cp, s);
    if (!xs.ok() || !os.ok()) return err(UFB_ECUDA, "cudaMallocAsync failed for convolution scratch");
    const Act in = make_act(xs.get<uint8_t>(), n, h, w, c, cp);
    const Act ov = make_act(os.get<uint8_t>(), n, h, w, c, cp);
    if (!cuda_ok(nchw_to_split(x, n, c, h, w, 1, in, s), "input layout")) return last_code();
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "current device")) return last_code();
    int* status = device_status(device);
    if (!status) return last_code();
    if (!cuda_ok(dwconv3x3(in, ov, weight, static_cast<const int16_t*>(bias), status, s), "depthwise convolution"))
        return last_code();
    if (!cuda_ok(split_to_nchw(ov, 1, out, s), "output layout")) return last_code();
    return UFB_OK;
}

int conv_dispatch(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                  const void* bias, int bias_bits, int sh, int sw, int ph, int pw, int groups, int16_t* out,
                  void* stream, bool allow_tc, bool allow_direct) {
    clear_error();
    if (!bias) bias_bits = 0;
    int oh = 0, ow = 0;
    if (!check_conv(x, n, ci, h, w, weight, co, kh, kw, bias_bits, sh, sw, ph, pw, groups, out, oh, ow))
        return last_code();
    auto s = static_cast<cudaStream_t>(stream);
    if (allow_tc && groups == ci && ci == co && ci % 4 == 0 && kh == 3 && kw == 3 && sh == 1 && sw == 1 && ph == 1 &&
        pw == 1 && bias_bits != 32)
        return conv_depthwise_path(x, n, ci, h, w, weight, bias_bits ? bias : nullptr, out, s);
    // stride 1, or stride 2 in both directions (TMA element strides)
    // (a full 8192-term reduction with an int32 bias could wrap the 32-bit epilogue sum)
    const long long k_total = static_cast<long long>(ci) * kh * kw;
    const bool tc_ok = allow_tc && groups == 1 && sh == sw && (sh == 1 || sh == 2) &&
                       (k_total < kTcMaxReduction || (k_total == kTcMaxReduction && bias_bits != 32));
    if (tc_ok)
        return conv_tc_path(x, n, ci, h, w, weight, co, kh, kw, bias, bias_bits, sh, ph, pw, oh, ow, out, s);
    if (!allow_direct && !allow_tc) return err(UFB_EINVAL, "no convolution path");
    return conv_direct_path(x, n, ci, h, w, weight, co, kh, kw, bias, bias_bits, sh, sw, ph, pw, groups, oh, ow, out,
                            s);
}

}  // namespace

extern "C" {

int ufb_version(void) { return 100; }

int ufb_set_conv_max_ctas(int n) {
    clear_error();
    if (n < 0) return err(UFB_EINVAL, "CTA cap must be >= 0");
    tc_set_max_ctas(n);
    return UFB_OK;
}

int ufb_set_conv_narrow(int enable) {
    clear_error();
    if (enable != 0 && enable != 1) return err(UFB_EINVAL, "narrow switch must be 0 or 1");
    tc_set_narrow(enable != 0);
    return UFB_OK;
}

const char* ufb_last_error(void) { return last_message(); }

int ufb_device_status(int device) {
    clear_error();
    int* st = device_status(device);
    if (!st) return last_code();
    int prev = 0;
    if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice") || !cuda_ok(cudaDeviceSynchronize(), "synchronize") ||
        !cuda_ok(cudaMemcpy(&prev, st, sizeof(int), cudaMemcpyDeviceToHost), "status read") ||
        !cuda_ok(cudaMemset(st, 0, sizeof(int)), "status clear"))
        return last_code();
    return prev;
}

int ufb_conv2d(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
               const void* bias, int bias_bits, int sh, int sw, int ph, int pw, int groups, int16_t* out,
               void* stream) {
    return conv_dispatch(x, n, ci, h, w, weight, co, kh, kw, bias, bias_bits, sh, sw, ph, pw, groups, out, stream,
                         true, true);
}

int ufb_conv2d_generic(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                       const void* bias, int bias_bits, int sh, int sw, int ph, int pw, int groups, int16_t* out,
                       void* stream) {
    return conv_dispatch(x, n, ci, h, w, weight, co, kh, kw, bias, bias_bits, sh, sw, ph, pw, groups, out, stream,
                         false, true);
}

int ufb_conv2d_baseline(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh,
                        int kw, const void* bias, int bias_bits, int sh, int sw, int ph, int pw, int groups,
                        int16_t* out, void* stream) {
    return conv_dispatch(x, n, ci, h, w, weight, co, kh, kw, bias, bias_bits, sh, sw, ph, pw, groups, out, stream,
                         true, true);
}

int ufb_add(int count, const int16_t* const* values, int64_t numel, int16_t* out, void* stream) {
    clear_error();
    if (count < 2 || count > 4) return err(UFB_EINVAL, "add supports 2 to 4 tensors");
    if (!values || !out || numel <= 0 || numel > INT32_MAX) return err(UFB_EINVAL, "unsupported tensor size");
    for (int i = 0; i < count; ++i)
        if (!values[i]) return err(UFB_EINVAL, "add operand is null");
    return cuda_ok(ew_add(out, values[0], values[1], count > 2 ? values[2] : nullptr, count > 3 ? values[3] : nullptr,
                          numel, static_cast<cudaStream_t>(stream)),
                   "add")
               ? UFB_OK
               : last_code();
}

int ufb_mul(const int16_t* x, const int64_t* xs, const int16_t* scale, const int64_t* ss, int16_t* out,
            void* stream) {
    clear_error();
    if (!x || !xs || !scale || !ss || !out) return err(UFB_EINVAL, "multiply requires matching CUDA 4D tensors");
    long long xl[4], sl[4];
    long long numel = 1, snumel = 1;
    for (int d = 0; d < 4; ++d) {
        xl[d] = xs[d];
        sl[d] = ss[d];
        if (sl[d] != 1 && sl[d] != xl[d]) return err(UFB_EINVAL, "invalid broadcast");
        numel *= xl[d];
        snumel *= sl[d];
    }
    if (numel <= 0 || numel > INT32_MAX || snumel <= 0) return err(UFB_EINVAL, "unsupported tensor size");
    return cuda_ok(ew_mul(out, x, scale, xl, sl, static_cast<cudaStream_t>(stream)), "multiply") ? UFB_OK
                                                                                                : last_code();
}

int ufb_lut(const int16_t* x, int64_t numel, const void* table, int table_bits, void* out, void* stream) {
    clear_error();
    if (!x || !table || !out || numel <= 0 || numel > INT32_MAX) return err(UFB_EINVAL, "unsupported tensor size");
    auto s = static_cast<cudaStream_t>(stream);
    if (table_bits == 16)
        return cuda_ok(ew_lut16(static_cast<int16_t*>(out), x, static_cast<const int16_t*>(table), numel, s), "lut")
                   ? UFB_OK
                   : last_code();
    if (table_bits == 8)
        return cuda_ok(ew_lut8(static_cast<uint8_t*>(out), x, static_cast<const uint8_t*>(table), numel, s), "lut")
                   ? UFB_OK
                   : last_code();
    return err(UFB_EINVAL, "invalid table dtype");
}

int ufb_bytes(const uint8_t* x, int64_t numel, int16_t* out, void* stream) {
    clear_error();
    if (!x || !out || numel <= 0 || numel > INT32_MAX) return err(UFB_EINVAL, "CUDA bytes required");
    return cuda_ok(ew_bytes(out, x, numel, static_cast<cudaStream_t>(stream)), "bytes") ? UFB_OK : last_code();
}

int ufb_wsilu4(const int16_t* x, int n, int c4, int h, int w, const int16_t* table, int16_t* out, void* stream) {
    clear_error();
    if (!x || !table || !out || n <= 0 || c4 <= 0 || h <= 0 || w <= 0 || c4 % 4)
        return err(UFB_EINVAL, "invalid WSiLU4 inputs");
    if (static_cast<long long>(n) * c4 * h * w > INT32_MAX) return err(UFB_EINVAL, "unsupported tensor size");
    return cuda_ok(ew_wsilu4(out, x, table, n, c4, static_cast<long long>(h) * w, static_cast<cudaStream_t>(stream)),
                   "wsilu4")
               ? UFB_OK
               : last_code();
}

int ufb_warp(const int16_t* feature, const int16_t* flow, int n, int c, int h, int w, int16_t* out, void* stream) {
    clear_error();
    if (!feature || !flow || !out || n <= 0 || c <= 0 || h <= 0 || w <= 0)
        return err(UFB_EINVAL, "invalid warp dimensions");
    if (static_cast<long long>(n) * c * h * w > INT32_MAX || static_cast<long long>(w) * 512 > INT32_MAX / 2 ||
        static_cast<long long>(h) * 512 > INT32_MAX / 2)
        return err(UFB_ERANGE, "warp tensor exceeds indexing bounds");
    if (static_cast<long long>(n) * ((c + 7) / 8) > 65535) return err(UFB_ERANGE, "warp batch exceeds grid bounds");
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return last_code();
    int* status = device_status(device);
    if (!status) return last_code();
    return cuda_ok(warp_fixed(out, feature, flow, n, c, h, w, status, static_cast<cudaStream_t>(stream)), "warp")
               ? UFB_OK
               : last_code();
}

int ufb_to_split(const int16_t* x, int n, int c, int h, int w, int factor, uint8_t* out, int pitch, void* stream) {
    clear_error();
    if (!x || !out || n <= 0 || c <= 0 || h <= 0 || w <= 0 || factor <= 0 || h % factor || w % factor)
        return err(UFB_EINVAL, "invalid split conversion geometry");
    if (pitch % 16 || pitch < c * factor * factor || reinterpret_cast<uintptr_t>(out) % 16)
        return err(UFB_EINVAL, "split pitch must be a multiple of 16 covering every channel");
    const Act a = make_act(out, n, h / factor, w / factor, c * factor * factor, pitch);
    return cuda_ok(nchw_to_split(x, n, c, h, w, factor, a, static_cast<cudaStream_t>(stream)), "to split")
               ? UFB_OK
               : last_code();
}

int ufb_from_split(const uint8_t* x, int n, int c, int h, int w, int pitch, int factor, int16_t* out,
                   void* stream) {
    clear_error();
    if (!x || !out || n <= 0 || c <= 0 || h <= 0 || w <= 0 || factor <= 0 || c % (factor * factor))
        return err(UFB_EINVAL, "invalid split conversion geometry");
    if (pitch % 16 || pitch < c || reinterpret_cast<uintptr_t>(x) % 16)
        return err(UFB_EINVAL, "split pitch must be a multiple of 16 covering every channel");
    const Act a = make_act(const_cast<uint8_t*>(x), n, h, w, c, pitch);
    return cuda_ok(split_to_nchw(a, factor, out, static_cast<cudaStream_t>(stream)), "from split") ? UFB_OK
                                                                                                   : last_code();
}

int64_t ufb_weight_bytes(int co, int ci, int kh, int kw) {
    if (co <= 0 || ci <= 0 || kh <= 0 || kw <= 0) return 0;
    return static_cast<int64_t>(tc_weight_bytes(co, ci, kh, kw, 128));
}

int ufb_prepare_weights(const int16_t* weight, int co, int ci, int kh, int kw, uint8_t* planes, void* stream) {
    clear_error();
    if (!weight || !planes || co <= 0 || ci <= 0 || kh <= 0 || kw <= 0) return err(UFB_EINVAL, "invalid weights");
    TcWeights tw;
    std::string msg;
    if (!tc_prepare(tw, weight, co, ci, kh, kw, false, 128, planes, static_cast<cudaStream_t>(stream), msg))
        return err(UFB_ECUDA, msg);
    return UFB_OK;
}

int ufb_conv2d_split(const uint8_t* x, int n, int ci, int h, int w, int x_pitch, const uint8_t* planes, int co,
                     int kh, int kw, const void* bias, int bias_bits, int pad_h, int pad_w, uint8_t* out,
                     int out_pitch, void* stream) {
    clear_error();
    if (!bias) bias_bits = 0;
    int oh = 0, ow = 0;
    // geometry checks of the NCHW entry point (x only needs to be non-null)
    if (!check_conv(reinterpret_cast<const int16_t*>(x), n, ci, h, w, reinterpret_cast<const int16_t*>(planes), co,
                    kh, kw, bias_bits, 1, 1, pad_h, pad_w, 1, reinterpret_cast<int16_t*>(out), oh, ow))
        return last_code();
    if (static_cast<long long>(ci) * kh * kw > kTcMaxReduction) return err(UFB_ERANGE, "reduction exceeds 8192");
    int device = 0;
    if (!cuda_ok(cudaGetDevice(&device), "cudaGetDevice")) return last_code();
    int* status = device_status(device);
    if (!status) return last_code();
    TcWeights tw;
    std::string msg;
    if (!tc_describe(tw, co, ci, kh, kw, false, 128, const_cast<uint8_t*>(planes), msg)) return err(UFB_ECUDA, msg);
    const Act in = make_act(const_cast<uint8_t*>(x), n, h, w, ci, x_pitch);
    const Act ov = make_act(out, n, oh, ow, co, out_pitch);
    Epilogue epi{};
    epi.bias = bias_bits ? bias : nullptr;
    epi.bias32 = bias_bits == 32;
    if (conv_tc_run(tw, in, ov, epi, pad_h, pad_w, static_cast<cudaStream_t>(stream), status, msg))
        return err(UFB_EINVAL, msg);
    return UFB_OK;
}

}  // extern "C"
