// SHA-256 digests of the UF pipeline: the decoded-YUV checksum of a stream
// (IntegerCodec::decode_stream_impl, src/integer_codec.cpp:426-488) and the
// identity of a prepared model (content_hash, src/prepared.cpp:64-105).
// Hashing is OpenSSL's EVP SHA-256, as in the reference.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ufb {

class Sha256 {
public:
    Sha256();
    ~Sha256();
    Sha256(const Sha256&) = delete;
    Sha256& operator=(const Sha256&) = delete;
    void update(const void* data, size_t n);
    void update(const std::string& s) { update(s.data(), s.size()); }
    std::array<uint8_t, 32> finish();  // the object can be reused after finish

private:
    void* ctx_;
};

std::string to_hex(const uint8_t* bytes, size_t n);

// One tensor of a prepared model as the identity hashes it: name, dtype code
// (0 int16, 1 uint8, 2 int32, 3 int8, 4 int64), shape and little-endian data.
struct IdentityTensor {
    std::string name;
    int dtype;
    std::vector<int64_t> shape;
    const void* data;
};

// prepared_identity (src/prepared.cpp:64-105, 114-116): SHA-256 over the
// compact sorted-key ASCII JSON {"arithmetic","format","source_sha256",
// "variant"}, then for every tensor in byte order of its name the compact JSON
// [name, "torch.<dtype>", shape] followed by the tensor's bytes.  Returns
// 64 lowercase hex digits.  Names must be valid UTF-8.
std::string prepared_identity(const std::string& format, const std::string& arithmetic, const std::string& variant,
                              const std::string& source_sha256, std::vector<IdentityTensor> tensors);

// Python json.dumps(s, ensure_ascii=True) of one string (quotes included).
std::string json_ascii_string(const std::string& s);

}  // namespace ufb
