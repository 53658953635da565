// UF16 bitstream container: parsing and writing in memory (layout in
// uf16_stream.h; behaviour of the reference's src/bitstream.cpp:173-360).
#include "uf16_stream.h"

#include "rans.h"  // StreamError

#include <cstring>
#include <stdexcept>

namespace ufb {
namespace uf16 {

namespace {

constexpr uint8_t kMagic[8] = {'U', 'F', '1', '6', 1, 0, 0, 0};

}  // namespace

uint8_t Reader::byte() {
    if (pos_ >= size_) throw StreamError("Truncated UF bitstream");
    return data_[pos_++];
}

const uint8_t* Reader::take(size_t n, const char* message) {
    if (size_ - pos_ < n) throw StreamError(message);
    const uint8_t* p = data_ + pos_;
    pos_ += n;
    return p;
}

// read_preamble (src/bitstream.cpp:221-245): a stream whose first byte is not
// 'U' is an FP16 stream and nothing is consumed.
Preamble Reader::preamble() {
    Preamble p;
    if (pos_ >= size_ || data_[pos_] != 'U') return p;
    const uint8_t* sig = take(4, "Truncated UF bitstream payload");
    if (std::memcmp(sig, kMagic, 4) != 0) throw StreamError("Unsupported UF preamble signature");
    const uint8_t* ver = take(4, "Truncated UF bitstream payload");
    if (std::memcmp(ver, kMagic + 4, 4) != 0) throw StreamError("Unsupported UF16 preamble version");
    p.integer = true;
    std::memcpy(p.image_identity.data(), take(32, "Truncated UF bitstream payload"), 32);
    std::memcpy(p.video_identity.data(), take(32, "Truncated UF bitstream payload"), 32);
    return p;
}

// read_optional_header (src/bitstream.cpp:181-189).
bool Reader::header(Nal& type, uint8_t& sps_id) {
    if (pos_ >= size_) return false;
    const uint8_t h = data_[pos_++];
    if ((h >> 4) > 2) throw StreamError("Unsupported UF NAL type");
    type = static_cast<Nal>(h >> 4);
    sps_id = h & 0x0f;
    return true;
}

// read_uint_adaptive (src/bitstream.cpp:197-205): the two top bits of the
// first byte select 1, 2 or 4 bytes.
uint32_t Reader::uint_adaptive() {
    const uint32_t b0 = byte();
    if (!(b0 & 0x80u)) return b0;
    const uint32_t b1 = byte();
    if (!(b0 & 0x40u)) return (b0 & 0x3fu) << 8 | b1;
    const uint32_t b2 = byte();
    const uint32_t b3 = byte();
    return (b0 & 0x3fu) << 24 | b1 << 16 | b2 << 8 | b3;
}

// read_sps (src/bitstream.cpp:258-264): height first, then width.
Sps Reader::sps(uint8_t id) {
    Sps s;
    s.id = id;
    s.height = uint_adaptive();
    s.width = uint_adaptive();
    if (!s.width || !s.height) throw StreamError("Invalid UF dimensions");
    return s;
}

// read_packet (src/bitstream.cpp:276-290).
Packet Reader::packet(Nal type, uint8_t sps_id) {
    if (type != Nal::intra && type != Nal::predicted) throw std::invalid_argument("Expected an I or P packet");
    Packet p;
    p.type = type;
    p.sps_id = sps_id;
    p.qp = byte();
    const uint8_t flags = byte();
    p.entropy_parallel = flags >> 1;
    p.reset = (flags & 1u) != 0;
    p.length = uint_adaptive();
    p.payload = take(p.length, "Truncated UF bitstream payload");
    return p;
}

size_t Writer::uint_adaptive(uint32_t v) {
    if (v < (1u << 7)) {
        out_.push_back(static_cast<uint8_t>(v));
        return 1;
    }
    if (v < (1u << 14)) {
        out_.push_back(static_cast<uint8_t>(0x80u | v >> 8));
        out_.push_back(static_cast<uint8_t>(v));
        return 2;
    }
    if (v < (1u << 30)) {
        out_.push_back(static_cast<uint8_t>(0xc0u | v >> 24));
        out_.push_back(static_cast<uint8_t>(v >> 16));
        out_.push_back(static_cast<uint8_t>(v >> 8));
        out_.push_back(static_cast<uint8_t>(v));
        return 4;
    }
    throw std::out_of_range("UF adaptive integer exceeds 30 bits");
}

// write_preamble (src/bitstream.cpp:247-256): nothing for an FP16 stream.
size_t Writer::preamble(const Preamble& p) {
    if (!p.integer) return 0;
    out_.insert(out_.end(), kMagic, kMagic + 8);
    out_.insert(out_.end(), p.image_identity.begin(), p.image_identity.end());
    out_.insert(out_.end(), p.video_identity.begin(), p.video_identity.end());
    return 72;
}

// write_sps (src/bitstream.cpp:266-274): the header byte of an SPS is its id.
size_t Writer::sps(const Sps& s) {
    if (s.id >= 16 || !s.width || !s.height) throw std::invalid_argument("Invalid UF SPS");
    // validate both integers before appending anything
    if (s.height >= (1u << 30) || s.width >= (1u << 30)) throw std::out_of_range("UF adaptive integer exceeds 30 bits");
    out_.push_back(s.id);
    const size_t h = uint_adaptive(s.height);
    return 1 + h + uint_adaptive(s.width);
}

// write_packet (src/bitstream.cpp:292-306).
size_t Writer::packet(const Packet& p) {
    if (p.sps_id >= 16 || p.entropy_parallel >= 128 || (p.type != Nal::intra && p.type != Nal::predicted) ||
        p.length >= (size_t{1} << 30) || (p.length && !p.payload))
        throw std::invalid_argument("Invalid UF packet");
    out_.push_back(static_cast<uint8_t>(static_cast<uint8_t>(p.type) << 4 | p.sps_id));
    out_.push_back(p.qp);
    out_.push_back(static_cast<uint8_t>(p.entropy_parallel << 1 | (p.reset ? 1 : 0)));
    const size_t n = uint_adaptive(static_cast<uint32_t>(p.length));
    if (p.length) out_.insert(out_.end(), p.payload, p.payload + p.length);
    return 3 + n + p.length;
}

// scan_bitstream (src/bitstream.cpp:315-358).
Scan scan(const uint8_t* data, size_t size, const std::string& variant, std::optional<uint64_t> expected_frames) {
    if (variant != "ld" && variant != "hts" && variant != "htl")
        throw std::invalid_argument("UF model variant must be ld, hts or htl");
    Reader r(data, size);
    Scan out;
    out.preamble = r.preamble();
    std::array<std::optional<Sps>, 16> table{};
    const uint64_t chunk = variant == "ld" ? 1 : 8;
    bool first = true;
    Nal type;
    uint8_t id;
    while (r.header(type, id)) {
        if (type == Nal::sps) {
            table[id] = r.sps(id);
            continue;
        }
        if (!table[id]) throw StreamError("UF packet uses an unknown SPS");
        if (first && type != Nal::intra) throw StreamError("UF bitstream must start with an I packet");
        first = false;
        const Sps& s = *table[id];
        if (out.packets && (out.dimensions.width != s.width || out.dimensions.height != s.height))
            throw StreamError("UF dimensions changed within the stream");
        out.dimensions = s;
        if (expected_frames && out.maximum_frames >= *expected_frames) throw StreamError("Unexpected extra UF packet");
        const Packet p = r.packet(type, id);
        if (!p.entropy_parallel) throw StreamError("Invalid UF entropy parallelism");
        ++out.packets;
        if (type == Nal::intra) ++out.intra_packets;
        else ++out.predicted_packets;
        out.maximum_frames += type == Nal::intra ? 1 : chunk;
    }
    if (!out.packets) throw StreamError("UF bitstream has no coded frames");
    if (expected_frames && out.maximum_frames < *expected_frames) throw StreamError("UF bitstream has too few coded frames");
    return out;
}

// hex_identity (src/integer_codec.cpp:53-66).
Identity identity_from_hex(const std::string& hex) {
    if (hex.size() != 64) throw std::invalid_argument("Invalid UF prepared identity");
    auto digit = [](char c) -> int {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        throw std::invalid_argument("Invalid UF prepared identity hex");
    };
    Identity id{};
    for (size_t i = 0; i < id.size(); ++i) id[i] = static_cast<uint8_t>(digit(hex[2 * i]) * 16 + digit(hex[2 * i + 1]));
    return id;
}

std::string identity_to_hex(const Identity& id) {
    static const char* kDigits = "0123456789abcdef";
    std::string s(64, '0');
    for (size_t i = 0; i < id.size(); ++i) {
        s[2 * i] = kDigits[id[i] >> 4];
        s[2 * i + 1] = kDigits[id[i] & 15];
    }
    return s;
}

}  // namespace uf16
}  // namespace ufb
