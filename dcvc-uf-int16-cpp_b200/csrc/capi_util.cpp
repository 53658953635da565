#include "capi_util.h"

#include "uf_b200.h"

#include <climits>
#include <cstdint>

namespace ufb {

namespace {
thread_local std::string g_message;
thread_local int g_code = 0;
}  // namespace

void clear_error() {
    g_message.clear();
    g_code = 0;
}

bool fail(int code, const std::string& message) {
    g_code = code;
    g_message = message;
    return false;
}

int last_code() { return g_code ? g_code : UFB_ECUDA; }

const char* last_message() { return g_message.c_str(); }

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    return fail(UFB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool check_conv(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                int bias_bits, int sh, int sw, int ph, int pw, int groups, const int16_t* out, int& oh, int& ow) {
    if (!x || !weight || !out) return fail(UFB_EINVAL, "convolution tensors must be non-null");
    if (sh <= 0 || sw <= 0 || ph < 0 || pw < 0 || groups <= 0) return fail(UFB_EINVAL, "invalid convolution geometry");
    if (ci <= 0 || co <= 0 || kh <= 0 || kw <= 0 || n <= 0 || h <= 0 || w <= 0)
        return fail(UFB_EINVAL, "empty convolution");
    if (ci % groups || co % groups) return fail(UFB_EINVAL, "invalid groups");
    if (bias_bits != 16 && bias_bits != 32 && bias_bits != 0) return fail(UFB_EINVAL, "bias_bits must be 16 or 32");
    const long long padded_h = static_cast<long long>(h) + 2ll * ph, padded_w = static_cast<long long>(w) + 2ll * pw;
    if (padded_h < kh || padded_w < kw) return fail(UFB_EINVAL, "kernel exceeds input");
    if (static_cast<long long>(ci / groups) * kh * kw >= (INT64_MAX / 1073741824LL) - 1)
        return fail(UFB_ERANGE, "dot product overflow");
    const long long ohl = (padded_h - kh) / sh + 1, owl = (padded_w - kw) / sw + 1;
    const long long planes = static_cast<long long>(n) * co;
    if (planes > INT32_MAX || ohl > INT32_MAX / planes || owl > INT32_MAX / (planes * ohl) ||
        static_cast<long long>(n) * ci * h * w > INT32_MAX)
        return fail(UFB_ERANGE, "convolution output exceeds indexing bounds");
    oh = static_cast<int>(ohl);
    ow = static_cast<int>(owl);
    return true;
}

}  // namespace ufb
