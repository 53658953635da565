// Host single-lane rANS coder for the UF INT16 bitstream.
//
// Wire format of the reference's uf::EntropyEncoder / EntropyDecoder
// (src/entropy.cpp:11-247, after Microsoft DCVC-UF py_rans): 32-bit state with
// lower bound 2^23, 16-bit probability scale, byte-wise renormalisation, and an
// escape symbol whose excess is sent as 2-bit bypass digits.  Symbols are int8
// mapped to v = 2|s| - (s > 0).  Y rows are chosen per symbol by a CDF index,
// Z rows by (qp * channels + c).  Encode order: Y parts in reverse, then Z;
// the flushed stream is the final state (little endian) followed by the
// emitted bytes in reverse.  Decode runs Z first, then Y parts forward.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <vector>

namespace ufb {

class RansTables {
public:
    // flat: rows x width int32 CDFs, lengths: entries used per row
    // (src/entropy.cpp:22-48 validates the same properties).
    void set(const int32_t* flat, int rows, int width, const int32_t* lengths);
    int rows() const { return static_cast<int>(max_.size()); }
    const uint32_t* row(int r) const { return cdf_.data() + static_cast<size_t>(r) * width_; }
    int maximum(int r) const { return max_[r]; }
    // Symbol search: index i with cdf[i] <= v < cdf[i + 1].
    int find(int r, uint32_t v) const;

private:
    std::vector<uint32_t> cdf_;   // rows x width
    std::vector<int> max_;        // escape index (length - 2) per row
    std::vector<uint8_t> guess_;  // rows x 256: first candidate index per (v >> 8)
    int width_ = 0;
};

class RansEncoder {
public:
    void reset();
    // packed values (symbol << 8) | index, coded last to first (src/entropy.cpp:173-183)
    void encode_y(const RansTables& t, const int16_t* packed, size_t n);
    // symbols in NHWC order, row = offset + i % channels (src/entropy.cpp:185-193)
    void encode_z(const RansTables& t, const int8_t* symbols, size_t n, int offset, int channels);
    std::vector<uint8_t> flush();

private:
    void put(uint32_t start, uint32_t freq);
    void put_bypass(uint32_t v);
    void encode_one(const RansTables& t, int row, int symbol);
    uint32_t state_ = 1u << 23;
    std::vector<uint8_t> out_;
};

class RansDecoder {
public:
    void set_stream(const uint8_t* data, size_t n);
    void decode_z(const RansTables& t, size_t count, int offset, int channels, int8_t* out);
    void decode_y(const RansTables& t, const uint8_t* indexes, size_t n, int8_t* out);

private:
    uint8_t next();
    uint32_t get_bypass();
    int8_t decode_one(const RansTables& t, int row);
    const uint8_t* data_ = nullptr;
    size_t size_ = 0, pos_ = 0;
    uint32_t state_ = 0;
};

// Error thrown for corrupt or truncated streams (maps to UFB_ESTREAM).
struct StreamError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

}  // namespace ufb
