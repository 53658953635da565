// UF16 video bitstream container (the reference's uf::read_* / write_* /
// scan_bitstream, src/bitstream.cpp:173-360, include/uf/bitstream.hpp:20-107).
//
// Wire layout:
//   preamble  "UF16" 01 00 00 00, image identity (32 bytes), video identity
//             (32 bytes); absent for an FP16 stream (its first byte is a NAL
//             header, whose type nibble is at most 2, never 'U').
//   NAL unit  one header byte: type << 4 | sps_id (type 0 SPS, 1 I, 2 P).
//   SPS       height, width as adaptive integers.
//   packet    qp byte, flags byte (entropy_parallel << 1 | reset), payload
//             length as an adaptive integer, payload bytes.
//   adaptive  v < 2^7: 1 byte v; v < 2^14: 0x80 | v >> 8, v & 0xff;
//             v < 2^30: 0xc0 | v >> 24 then three bytes, big endian.
//
// Parsing works on a byte span in memory; payloads are returned as views into
// it.  Every malformed or truncated input throws StreamError with the
// reference's message; invalid writer arguments throw std::invalid_argument
// or std::out_of_range.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <vector>

namespace ufb {
namespace uf16 {

enum class Nal : uint8_t { sps = 0, intra = 1, predicted = 2 };

using Identity = std::array<uint8_t, 32>;

struct Preamble {
    bool integer = false;
    Identity image_identity{};
    Identity video_identity{};
};

struct Sps {
    uint8_t id = 0;
    uint32_t width = 0;
    uint32_t height = 0;
};

struct Packet {
    Nal type = Nal::intra;
    uint8_t sps_id = 0;
    uint8_t qp = 0;
    uint8_t entropy_parallel = 0;
    bool reset = false;
    const uint8_t* payload = nullptr;  // view into the parsed span
    size_t length = 0;
};

struct Scan {
    Preamble preamble;
    Sps dimensions;
    uint64_t packets = 0;
    uint64_t intra_packets = 0;
    uint64_t predicted_packets = 0;
    uint64_t maximum_frames = 0;
};

// Sequential reader over one bitstream held in memory.
class Reader {
public:
    Reader(const uint8_t* data, size_t size) : data_(data), size_(size) {}
    size_t position() const { return pos_; }
    void seek(size_t pos) { pos_ = pos < size_ ? pos : size_; }

    Preamble preamble();                               // read_preamble
    // read_optional_header: false at the clean end of the stream
    bool header(Nal& type, uint8_t& sps_id);
    Sps sps(uint8_t id);                               // read_sps
    Packet packet(Nal type, uint8_t sps_id);           // read_packet
    uint32_t uint_adaptive();                          // read_uint_adaptive

private:
    uint8_t byte();
    const uint8_t* take(size_t n, const char* message);
    const uint8_t* data_;
    size_t size_;
    size_t pos_ = 0;
};

// Appends to a byte vector; each call returns the bytes it wrote (the
// reference's writers return the same counts).
class Writer {
public:
    explicit Writer(std::vector<uint8_t>& out) : out_(out) {}
    size_t preamble(const Preamble& p);                // write_preamble (0 for FP16)
    size_t sps(const Sps& s);                          // write_sps
    size_t packet(const Packet& p);                    // write_packet
    size_t uint_adaptive(uint32_t v);                  // write_uint_adaptive

private:
    std::vector<uint8_t>& out_;
};

// scan_bitstream: validates the NAL sequence of a whole stream without
// decoding payloads. variant "ld" (P packets of 1 frame), "hts" or "htl" (8).
Scan scan(const uint8_t* data, size_t size, const std::string& variant, std::optional<uint64_t> expected_frames);

// Identity bytes from the 64-digit lowercase hex identity of a prepared model.
Identity identity_from_hex(const std::string& hex);
std::string identity_to_hex(const Identity& id);

}  // namespace uf16
}  // namespace ufb
