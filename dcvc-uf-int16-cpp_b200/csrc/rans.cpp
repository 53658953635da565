#include "rans.h"

#include <algorithm>
#include <cstdlib>
#include <string>

namespace ufb {

namespace {
constexpr uint32_t kScaleBits = 16;
constexpr uint32_t kLower = 1u << 23;
constexpr uint32_t kProbMask = (1u << kScaleBits) - 1u;
constexpr uint32_t kBypassBits = 2;
constexpr uint32_t kMaxBypass = (1u << kBypassBits) - 1u;
}  // namespace

void RansTables::set(const int32_t* flat, int rows, int width, const int32_t* lengths) {
    if (rows <= 0 || width <= 0) throw std::invalid_argument("UF CDF table shape is invalid");
    width_ = width;
    cdf_.assign(static_cast<size_t>(rows) * width, 0);
    max_.assign(rows, 0);
    guess_.assign(static_cast<size_t>(rows) * 256, 0);
    for (int r = 0; r < rows; ++r) {
        const int len = lengths[r];
        if (len < 2 || len > width || len - 2 > 127) throw std::invalid_argument("UF CDF row length is invalid");
        const int32_t* row = flat + static_cast<size_t>(r) * width;
        if (row[0] != 0 || row[len - 1] != (1 << kScaleBits))
            throw std::invalid_argument("UF CDF does not span 16-bit probability space");
        for (int j = 1; j < len; ++j)
            if (row[j] <= row[j - 1]) throw std::invalid_argument("UF CDF is not increasing");
        uint32_t* dst = cdf_.data() + static_cast<size_t>(r) * width;
        for (int j = 0; j < len; ++j) dst[j] = static_cast<uint32_t>(row[j]);
        // entries past the row length stay unused; mark them unreachable
        for (int j = len; j < width; ++j) dst[j] = 0xFFFFFFFFu;
        max_[r] = len - 2;
        // guess[b] = last index i (< len - 1) with cdf[i] <= b * 256
        int i = 0;
        for (int b = 0; b < 256; ++b) {
            const uint32_t v = static_cast<uint32_t>(b) << 8;
            while (i + 1 < len - 1 && dst[i + 1] <= v) ++i;
            guess_[static_cast<size_t>(r) * 256 + b] = static_cast<uint8_t>(i);
        }
    }
}

int RansTables::find(int r, uint32_t v) const {
    const uint32_t* row = this->row(r);
    int i = guess_[static_cast<size_t>(r) * 256 + (v >> 8)];
    const int last = max_[r];  // valid symbol indexes are 0 .. max (len - 2)
    while (i < last && row[i + 1] <= v) ++i;
    return i;
}

// ---------------------------------------------------------------- encoder --

void RansEncoder::reset() {
    state_ = kLower;
    out_.clear();
}

void RansEncoder::put(uint32_t start, uint32_t freq) {
    if (!freq) throw std::runtime_error("Zero UF rANS frequency");
    const uint32_t limit = freq << (23u - kScaleBits + 8u);
    while (state_ >= limit) {
        out_.push_back(static_cast<uint8_t>(state_));
        state_ >>= 8u;
    }
    state_ = ((state_ / freq) << kScaleBits) + (state_ % freq) + start;
}

void RansEncoder::put_bypass(uint32_t v) {
    constexpr uint32_t limit = (1u << (kScaleBits - kBypassBits)) << (23u - kScaleBits + 8u);
    while (state_ >= limit) {
        out_.push_back(static_cast<uint8_t>(state_));
        state_ >>= 8u;
    }
    state_ = (state_ << kBypassBits) | v;
}

void RansEncoder::encode_one(const RansTables& t, int row, int symbol) {
    const int maximum = t.maximum(row);
    int value = std::abs(symbol) * 2 - (symbol > 0 ? 1 : 0);
    if (value >= maximum) {
        const uint32_t raw = static_cast<uint32_t>(value - maximum);
        value = maximum;
        // digits: count of 2-bit digits of raw, sent as a run of 3s plus a
        // remainder, then the digits LSB first; written last-first
        int count = 0;
        while ((raw >> (count * kBypassBits)) != 0) ++count;
        uint32_t bins[32];
        int nb = 0;
        int rem = count;
        while (rem >= static_cast<int>(kMaxBypass)) {
            bins[nb++] = kMaxBypass;
            rem -= kMaxBypass;
        }
        bins[nb++] = static_cast<uint32_t>(rem);
        for (int i = 0; i < count; ++i) bins[nb++] = (raw >> (i * kBypassBits)) & kMaxBypass;
        for (int i = nb - 1; i >= 0; --i) put_bypass(bins[i]);
    }
    const uint32_t* cdf = t.row(row);
    put(cdf[value], cdf[value + 1] - cdf[value]);
}

void RansEncoder::encode_y(const RansTables& t, const int16_t* packed, size_t n) {
    for (size_t k = n; k-- > 0;) {
        const uint16_t p = static_cast<uint16_t>(packed[k]);
        const int index = p & 0xff;
        if (index >= t.rows()) throw std::runtime_error("UF Y CDF index out of range");
        const int high = p >> 8;
        encode_one(t, index, static_cast<int8_t>(high >= 128 ? high - 256 : high));
    }
}

void RansEncoder::encode_z(const RansTables& t, const int8_t* symbols, size_t n, int offset, int channels) {
    if (offset < 0 || channels <= 0 || static_cast<size_t>(offset) > static_cast<size_t>(t.rows()) ||
        static_cast<size_t>(channels) > static_cast<size_t>(t.rows()) - offset)
        throw std::invalid_argument("UF Z CDF range is invalid");
    for (size_t k = n; k-- > 0;) encode_one(t, offset + static_cast<int>(k % channels), symbols[k]);
}

std::vector<uint8_t> RansEncoder::flush() {
    std::vector<uint8_t> r;
    r.reserve(out_.size() + 4);
    for (int s = 0; s < 32; s += 8) r.push_back(static_cast<uint8_t>(state_ >> s));
    r.insert(r.end(), out_.rbegin(), out_.rend());
    return r;
}

// ---------------------------------------------------------------- decoder --

void RansDecoder::set_stream(const uint8_t* data, size_t n) {
    if (n < 4) throw std::invalid_argument("UF rANS stream is too short");
    data_ = data;
    size_ = n;
    pos_ = 0;
    state_ = 0;
    for (int s = 0; s < 32; s += 8) state_ |= static_cast<uint32_t>(next()) << s;
}

uint8_t RansDecoder::next() {
    if (pos_ >= size_) throw StreamError("Truncated UF rANS stream");
    return data_[pos_++];
}

uint32_t RansDecoder::get_bypass() {
    const uint32_t v = state_ & kMaxBypass;
    state_ >>= kBypassBits;
    if (state_ < kLower) state_ = (state_ << 8u) | next();
    return v;
}

int8_t RansDecoder::decode_one(const RansTables& t, int row) {
    const uint32_t cum = state_ & kProbMask;
    const int idx = t.find(row, cum);
    const uint32_t* cdf = t.row(row);
    const uint32_t freq = cdf[idx + 1] - cdf[idx];
    state_ = freq * (state_ >> kScaleBits) + cum - cdf[idx];
    while (state_ < kLower) state_ = (state_ << 8u) | next();
    uint32_t value = static_cast<uint32_t>(idx);
    const int maximum = t.maximum(row);
    if (value == static_cast<uint32_t>(maximum)) {
        uint32_t part = get_bypass();
        uint32_t count = part;
        while (part == kMaxBypass) {
            part = get_bypass();
            count += part;
            if (count > 16) throw StreamError("UF rANS bypass symbol is too large");
        }
        uint32_t raw = 0;
        for (uint32_t i = 0; i < count; ++i) raw |= get_bypass() << (i * kBypassBits);
        if (raw > 256u - static_cast<uint32_t>(maximum)) throw StreamError("Decoded UF rANS symbol exceeds INT8 range");
        value = raw + static_cast<uint32_t>(maximum);
    }
    const int s = (value & 1u) ? static_cast<int>((value + 1u) / 2u) : -static_cast<int>((value + 1u) / 2u);
    if (s < -128 || s > 127) throw StreamError("Decoded UF rANS symbol exceeds INT8 range");
    return static_cast<int8_t>(s);
}

void RansDecoder::decode_z(const RansTables& t, size_t count, int offset, int channels, int8_t* out) {
    if (offset < 0 || channels <= 0 || static_cast<size_t>(offset) > static_cast<size_t>(t.rows()) ||
        static_cast<size_t>(channels) > static_cast<size_t>(t.rows()) - offset)
        throw std::invalid_argument("UF Z CDF range is invalid");
    for (size_t i = 0; i < count; ++i) out[i] = decode_one(t, offset + static_cast<int>(i % channels));
}

void RansDecoder::decode_y(const RansTables& t, const uint8_t* indexes, size_t n, int8_t* out) {
    for (size_t i = 0; i < n; ++i) {
        if (indexes[i] >= t.rows()) throw StreamError("UF Y CDF index out of range");
        out[i] = decode_one(t, indexes[i]);
    }
}

}  // namespace ufb
