// SHA-256 helpers and the prepared-model identity (declarations in digest.h).
#include "digest.h"

#include <openssl/evp.h>

#include <algorithm>
#include <stdexcept>

namespace ufb {

Sha256::Sha256() : ctx_(EVP_MD_CTX_new()) {
    if (!ctx_ || EVP_DigestInit_ex(static_cast<EVP_MD_CTX*>(ctx_), EVP_sha256(), nullptr) != 1)
        throw std::runtime_error("OpenSSL SHA-256 initialization failed");
}

Sha256::~Sha256() { EVP_MD_CTX_free(static_cast<EVP_MD_CTX*>(ctx_)); }

void Sha256::update(const void* data, size_t n) {
    if (n && EVP_DigestUpdate(static_cast<EVP_MD_CTX*>(ctx_), data, n) != 1)
        throw std::runtime_error("OpenSSL SHA-256 update failed");
}

std::array<uint8_t, 32> Sha256::finish() {
    std::array<uint8_t, 32> out{};
    unsigned int len = 0;
    auto* ctx = static_cast<EVP_MD_CTX*>(ctx_);
    if (EVP_DigestFinal_ex(ctx, out.data(), &len) != 1 || len != 32 ||
        EVP_DigestInit_ex(ctx, EVP_sha256(), nullptr) != 1)
        throw std::runtime_error("OpenSSL SHA-256 finalization failed");
    return out;
}

std::string to_hex(const uint8_t* bytes, size_t n) {
    static const char* kDigits = "0123456789abcdef";
    std::string s(2 * n, '0');
    for (size_t i = 0; i < n; ++i) {
        s[2 * i] = kDigits[bytes[i] >> 4];
        s[2 * i + 1] = kDigits[bytes[i] & 15];
    }
    return s;
}

namespace {

void hex_escape(std::string& out, uint32_t v) {
    static const char* kDigits = "0123456789abcdef";
    out += "\\u";
    for (int d = 3; d >= 0; --d) out.push_back(kDigits[(v >> (4 * d)) & 15]);
}

// Next code point of strict UTF-8 (no overlong forms, no surrogates).
uint32_t next_code_point(const std::string& s, size_t& i) {
    const auto byte = [&](size_t k) { return static_cast<uint8_t>(s[k]); };
    const uint8_t b0 = byte(i);
    if (b0 < 0x80) {
        ++i;
        return b0;
    }
    int extra;
    uint32_t cp, min;
    if ((b0 & 0xe0) == 0xc0) extra = 1, cp = b0 & 0x1f, min = 0x80;
    else if ((b0 & 0xf0) == 0xe0) extra = 2, cp = b0 & 0x0f, min = 0x800;
    else if ((b0 & 0xf8) == 0xf0) extra = 3, cp = b0 & 0x07, min = 0x10000;
    else throw std::invalid_argument("tensor name is not valid UTF-8");
    if (i + extra >= s.size()) throw std::invalid_argument("tensor name is not valid UTF-8");
    for (int k = 1; k <= extra; ++k) {
        const uint8_t b = byte(i + k);
        if ((b & 0xc0) != 0x80) throw std::invalid_argument("tensor name is not valid UTF-8");
        cp = cp << 6 | (b & 0x3f);
    }
    if (cp < min || cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff))
        throw std::invalid_argument("tensor name is not valid UTF-8");
    i += extra + 1;
    return cp;
}

const char* torch_dtype_name(int code) {
    switch (code) {
    case 0: return "torch.int16";
    case 1: return "torch.uint8";
    case 2: return "torch.int32";
    case 3: return "torch.int8";
    case 4: return "torch.int64";
    default: throw std::invalid_argument("prepared tensor has an unsupported dtype");
    }
}

size_t dtype_size(int code) { return code == 0 ? 2 : code == 2 ? 4 : code == 4 ? 8 : 1; }

}  // namespace

std::string json_ascii_string(const std::string& s) {
    std::string out = "\"";
    for (size_t i = 0; i < s.size();) {
        const uint32_t cp = next_code_point(s, i);
        if (cp == '"' || cp == '\\') {
            out.push_back('\\');
            out.push_back(static_cast<char>(cp));
        } else if (cp == '\b') out += "\\b";
        else if (cp == '\f') out += "\\f";
        else if (cp == '\n') out += "\\n";
        else if (cp == '\r') out += "\\r";
        else if (cp == '\t') out += "\\t";
        else if (cp < 0x20 || cp >= 0x7f) {
            if (cp <= 0xffff) hex_escape(out, cp);
            else {
                const uint32_t v = cp - 0x10000;
                hex_escape(out, 0xd800 + (v >> 10));
                hex_escape(out, 0xdc00 + (v & 0x3ff));
            }
        } else out.push_back(static_cast<char>(cp));
    }
    out.push_back('"');
    return out;
}

std::string prepared_identity(const std::string& format, const std::string& arithmetic, const std::string& variant,
                              const std::string& source_sha256, std::vector<IdentityTensor> tensors) {
    std::sort(tensors.begin(), tensors.end(),
              [](const IdentityTensor& a, const IdentityTensor& b) { return a.name < b.name; });
    for (size_t i = 1; i < tensors.size(); ++i)
        if (tensors[i].name == tensors[i - 1].name) throw std::invalid_argument("duplicate prepared tensor name");
    Sha256 h;
    h.update("{\"arithmetic\":" + json_ascii_string(arithmetic) + ",\"format\":" + json_ascii_string(format) +
             ",\"source_sha256\":" + json_ascii_string(source_sha256) + ",\"variant\":" + json_ascii_string(variant) +
             "}");
    for (const IdentityTensor& t : tensors) {
        std::string d = "[" + json_ascii_string(t.name) + ",\"" + torch_dtype_name(t.dtype) + "\",[";
        size_t n = 1;
        for (size_t k = 0; k < t.shape.size(); ++k) {
            if (t.shape[k] < 0) throw std::invalid_argument("prepared tensor has a negative extent");
            if (k) d.push_back(',');
            d += std::to_string(t.shape[k]);
            n *= static_cast<size_t>(t.shape[k]);
        }
        d += "]]";
        h.update(d);
        if (n && !t.data) throw std::invalid_argument("prepared tensor has no data");
        h.update(t.data, n * dtype_size(t.dtype));  // little-endian host bytes
    }
    const auto digest = h.finish();
    return to_hex(digest.data(), digest.size());
}

}  // namespace ufb
