// Host rANS C ABI (include/uf_b200.h): the engine's own implementation of the
// reference's uf::EntropyEncoder / uf::EntropyDecoder wire format
// (src/entropy.cpp), usable without a GPU.
#include "uf_b200.h"

#include "capi_util.h"
#include "rans.h"

#include <cstring>
#include <stdexcept>
#include <vector>

using namespace ufb;

struct ufb_rans {
    RansTables z, y;
};

extern "C" {

ufb_rans* ufb_rans_create(const int32_t* z_cdf, int z_rows, int z_width, const int32_t* z_len, const int32_t* y_cdf,
                          int y_rows, int y_width, const int32_t* y_len) {
    clear_error();
    try {
        if (!z_cdf || !z_len || !y_cdf || !y_len) throw std::invalid_argument("CDF tables are required");
        auto r = new ufb_rans;
        try {
            r->z.set(z_cdf, z_rows, z_width, z_len);
            r->y.set(y_cdf, y_rows, y_width, y_len);
        } catch (...) {
            delete r;
            throw;
        }
        return r;
    } catch (const std::exception& e) {
        fail(UFB_EINVAL, e.what());
        return nullptr;
    }
}

void ufb_rans_destroy(ufb_rans* r) { delete r; }

int64_t ufb_rans_encode(ufb_rans* r, int nparts, const int16_t* const* parts, const size_t* part_lens,
                        const int8_t* z, size_t zn, int z_offset, int z_channels, uint8_t* out, size_t capacity) {
    clear_error();
    try {
        if (!r || (nparts && (!parts || !part_lens)) || (zn && !z)) throw std::invalid_argument("invalid encode call");
        RansEncoder enc;
        enc.reset();
        for (int p = nparts - 1; p >= 0; --p)
            if (part_lens[p]) enc.encode_y(r->y, parts[p], part_lens[p]);
        enc.encode_z(r->z, z, zn, z_offset, z_channels);
        const auto bytes = enc.flush();
        if (out) {
            if (bytes.size() > capacity) throw std::length_error("output buffer too small");
            std::memcpy(out, bytes.data(), bytes.size());
        }
        return static_cast<int64_t>(bytes.size());
    } catch (const std::invalid_argument& e) {
        return err(UFB_EINVAL, e.what());
    } catch (const std::length_error& e) {
        return err(UFB_ERANGE, e.what());
    } catch (const std::exception& e) {
        return err(UFB_ESTREAM, e.what());
    }
}

int ufb_rans_decode(ufb_rans* r, const uint8_t* data, size_t n, size_t zn, int z_offset, int z_channels,
                    int8_t* z_out, int nparts, const uint8_t* const* indexes, const size_t* index_lens,
                    int8_t* const* y_out) {
    clear_error();
    try {
        if (!r || !data || (zn && !z_out) || (nparts && (!indexes || !index_lens || !y_out)))
            throw std::invalid_argument("invalid decode call");
        RansDecoder dec;
        dec.set_stream(data, n);
        dec.decode_z(r->z, zn, z_offset, z_channels, z_out);
        for (int p = 0; p < nparts; ++p)
            if (index_lens[p]) dec.decode_y(r->y, indexes[p], index_lens[p], y_out[p]);
        return UFB_OK;
    } catch (const std::invalid_argument& e) {
        return err(UFB_EINVAL, e.what());
    } catch (const std::exception& e) {
        return err(UFB_ESTREAM, e.what());
    }
}

}  // extern "C"
