// C ABI of the UF16 container, the digests and whole-stream coding
// (include/uf_b200.h; uf16_stream.h, digest.h, stream_codec.h).
#include "uf_b200.h"

#include "capi_engine.h"
#include "digest.h"
#include "interrupt.h"
#include "stream_codec.h"
#include "uf16_stream.h"

#include <cstring>
#include <memory>
#include <stdexcept>
#include <vector>

using namespace ufb;

struct ufb_stream_codec {
    std::unique_ptr<StreamCodec> s;
};

namespace {

// Runs a writer into a scratch vector and copies the bytes to out.
template <class F>
int64_t write_into(uint8_t* out, size_t capacity, F&& fn) {
    int64_t written = 0;
    const int rc = guarded([&] {
        if (!out && capacity) throw std::invalid_argument("null output buffer");
        std::vector<uint8_t> bytes;
        uf16::Writer w(bytes);
        fn(w);
        if (bytes.size() > capacity) throw std::length_error("UF16 output buffer too small");
        if (!bytes.empty()) std::memcpy(out, bytes.data(), bytes.size());
        written = static_cast<int64_t>(bytes.size());
        return 0;
    });
    return rc ? rc : written;
}

uf16::Identity identity(const uint8_t* p) {
    uf16::Identity id{};
    if (p) std::memcpy(id.data(), p, id.size());
    return id;
}

void check_span(const uint8_t* data, size_t size, const size_t* pos) {
    if ((!data && size) || !pos || *pos > size) throw std::invalid_argument("invalid bitstream span");
}

}  // namespace

extern "C" {

int64_t ufb_uf16_write_preamble(const uint8_t* image_identity, const uint8_t* video_identity, uint8_t* out,
                                size_t capacity) {
    return write_into(out, capacity, [&](uf16::Writer& w) {
        if (!image_identity || !video_identity) throw std::invalid_argument("null identity");
        uf16::Preamble p;
        p.integer = true;
        p.image_identity = identity(image_identity);
        p.video_identity = identity(video_identity);
        w.preamble(p);
    });
}

int64_t ufb_uf16_write_sps(int id, uint32_t width, uint32_t height, uint8_t* out, size_t capacity) {
    return write_into(out, capacity, [&](uf16::Writer& w) {
        if (id < 0 || id >= 16) throw std::invalid_argument("Invalid UF SPS");
        w.sps(uf16::Sps{static_cast<uint8_t>(id), width, height});
    });
}

int64_t ufb_uf16_write_packet(int type, int sps_id, int qp, int entropy_parallel, int reset, const uint8_t* payload,
                              size_t length, uint8_t* out, size_t capacity) {
    return write_into(out, capacity, [&](uf16::Writer& w) {
        if ((type != UFB_NAL_INTRA && type != UFB_NAL_PREDICTED) || sps_id < 0 || sps_id >= 16 || qp < 0 ||
            qp >= 256 || entropy_parallel < 0 || entropy_parallel >= 128)
            throw std::invalid_argument("Invalid UF packet");
        uf16::Packet p;
        p.type = static_cast<uf16::Nal>(type);
        p.sps_id = static_cast<uint8_t>(sps_id);
        p.qp = static_cast<uint8_t>(qp);
        p.entropy_parallel = static_cast<uint8_t>(entropy_parallel);
        p.reset = reset != 0;
        p.payload = payload;
        p.length = length;
        w.packet(p);
    });
}

int64_t ufb_uf16_write_uint(uint32_t value, uint8_t* out, size_t capacity) {
    return write_into(out, capacity, [&](uf16::Writer& w) { w.uint_adaptive(value); });
}

int ufb_uf16_read_uint(const uint8_t* data, size_t size, size_t* pos, uint32_t* value) {
    return guarded([&] {
        check_span(data, size, pos);
        if (!value) throw std::invalid_argument("null value");
        uf16::Reader r(data, size);
        r.seek(*pos);
        *value = r.uint_adaptive();
        *pos = r.position();
        return 0;
    });
}

int ufb_uf16_read_preamble(const uint8_t* data, size_t size, size_t* pos, int* integer, uint8_t* image_identity,
                           uint8_t* video_identity) {
    return guarded([&] {
        check_span(data, size, pos);
        if (!integer) throw std::invalid_argument("null output");
        uf16::Reader r(data, size);
        r.seek(*pos);
        const uf16::Preamble p = r.preamble();
        *integer = p.integer ? 1 : 0;
        if (p.integer) {
            if (image_identity) std::memcpy(image_identity, p.image_identity.data(), 32);
            if (video_identity) std::memcpy(video_identity, p.video_identity.data(), 32);
        }
        *pos = r.position();
        return 0;
    });
}

int ufb_uf16_next(const uint8_t* data, size_t size, size_t* pos, ufb_uf16_nal* nal) {
    return guarded([&] {
        check_span(data, size, pos);
        if (!nal) throw std::invalid_argument("null output");
        uf16::Reader r(data, size);
        r.seek(*pos);
        uf16::Nal type;
        uint8_t id;
        if (!r.header(type, id)) return 0;
        ufb_uf16_nal out{};
        out.type = static_cast<int>(type);
        out.sps_id = id;
        if (type == uf16::Nal::sps) {
            const uf16::Sps s = r.sps(id);
            out.width = s.width;
            out.height = s.height;
        } else {
            const uf16::Packet p = r.packet(type, id);
            out.qp = p.qp;
            out.entropy_parallel = p.entropy_parallel;
            out.reset = p.reset ? 1 : 0;
            out.payload_offset = static_cast<uint64_t>(p.payload - data);
            out.payload_length = p.length;
        }
        *nal = out;
        *pos = r.position();
        return 1;
    });
}

int ufb_uf16_scan(const uint8_t* data, size_t size, const char* variant, int64_t expected_frames,
                  ufb_uf16_summary* out) {
    return guarded([&] {
        if ((!data && size) || !variant || !out) throw std::invalid_argument("invalid scan arguments");
        std::optional<uint64_t> expected;
        if (expected_frames >= 0) expected = static_cast<uint64_t>(expected_frames);
        const uf16::Scan s = uf16::scan(data, size, variant, expected);
        ufb_uf16_summary r{};
        r.integer = s.preamble.integer ? 1 : 0;
        std::memcpy(r.image_identity, s.preamble.image_identity.data(), 32);
        std::memcpy(r.video_identity, s.preamble.video_identity.data(), 32);
        r.width = s.dimensions.width;
        r.height = s.dimensions.height;
        r.packets = s.packets;
        r.intra_packets = s.intra_packets;
        r.predicted_packets = s.predicted_packets;
        r.maximum_frames = s.maximum_frames;
        *out = r;
        return 0;
    });
}

int ufb_sha256(const void* data, size_t size, uint8_t* digest32) {
    return guarded([&] {
        if ((!data && size) || !digest32) throw std::invalid_argument("invalid digest arguments");
        Sha256 h;
        h.update(data, size);
        const auto d = h.finish();
        std::memcpy(digest32, d.data(), d.size());
        return 0;
    });
}

int ufb_prepared_identity(const char* format, const char* arithmetic, const char* variant, const char* source_sha256,
                          int count, const char* const* names, const int* dtypes, const int* ndims,
                          const int64_t* shapes, const void* const* data, char* hex65) {
    return guarded([&] {
        if (!format || !arithmetic || !variant || !source_sha256 || count < 0 || !hex65 ||
            (count && (!names || !dtypes || !ndims || !shapes || !data)))
            throw std::invalid_argument("invalid prepared-model table");
        std::vector<IdentityTensor> tensors;
        const int64_t* cursor = shapes;
        for (int i = 0; i < count; ++i) {
            if (!names[i] || ndims[i] < 0) throw std::invalid_argument("invalid prepared-model table");
            tensors.push_back(IdentityTensor{names[i], dtypes[i], std::vector<int64_t>(cursor, cursor + ndims[i]),
                                             data[i]});
            cursor += ndims[i];
        }
        const std::string hex = prepared_identity(format, arithmetic, variant, source_sha256, std::move(tensors));
        std::memcpy(hex65, hex.c_str(), 65);
        return 0;
    });
}

int ufb_codec_state_hash(ufb_codec* c, int which, uint8_t* sha256_32) {
    return guarded([&] {
        if (!c || !sha256_32 || which < 0 || which > 2) throw std::invalid_argument("invalid state request");
        int64_t shape[4];
        if (!c->c->state_shape(which, shape)) return 1;
        std::vector<int16_t> host(static_cast<size_t>(shape[0] * shape[1] * shape[2] * shape[3]));
        c->c->state(which, host.data(), host.size(), shape);
        Sha256 h;
        h.update(host.data(), host.size() * sizeof(int16_t));  // little-endian host
        const auto d = h.finish();
        std::memcpy(sha256_32, d.data(), d.size());
        return 0;
    });
}

void ufb_set_interrupt(int on) { set_interrupt(on != 0); }

int ufb_interrupt_requested(void) { return interrupt_requested() ? 1 : 0; }

ufb_stream_codec* ufb_stream_codec_create(ufb_codec* image, ufb_codec* video, const uint8_t* image_identity,
                                          const uint8_t* video_identity) {
    ufb_stream_codec* out = nullptr;
    guarded([&] {
        if (!image || !image_identity || (video && !video_identity))
            throw std::invalid_argument("stream codec needs an image codec and identities");
        auto h = std::make_unique<ufb_stream_codec>();
        h->s = std::make_unique<StreamCodec>(*image->c, video ? video->c.get() : nullptr, identity(image_identity),
                                             identity(video_identity));
        out = h.release();
        return 0;
    });
    return out;
}

void ufb_stream_codec_destroy(ufb_stream_codec* s) { delete s; }

int ufb_stream_encode(ufb_stream_codec* s, const uint8_t* frames, uint64_t count, uint32_t width, uint32_t height,
                      int qp_i, int qp_p, int reset_interval, int intra_period, uint8_t* out, size_t capacity,
                      size_t* lengths, uint64_t* packets) {
    return guarded([&] {
        if (!s || !frames || !out || !lengths) throw std::invalid_argument("invalid stream encode arguments");
        EncodeSettings e;
        e.width = width;
        e.height = height;
        e.qp_i = qp_i;
        e.qp_p = qp_p;
        e.reset_interval = reset_interval;
        e.intra_period = intra_period;
        StreamStats stats;
        const auto streams = s->s->encode(frames, count, e, &stats);
        for (size_t b = 0; b < streams.size(); ++b)
            if (streams[b].size() > capacity) throw std::length_error("bitstream buffer too small");
        for (size_t b = 0; b < streams.size(); ++b) {
            std::memcpy(out + b * capacity, streams[b].data(), streams[b].size());
            lengths[b] = streams[b].size();
        }
        if (packets) *packets = stats.packets;
        return 0;
    });
}

int ufb_stream_decode(ufb_stream_codec* s, const uint8_t* const* data, const size_t* sizes, uint64_t total_frames,
                      uint64_t total_packets, uint32_t expected_width, uint32_t expected_height, ufb_frame_sink sink,
                      void* user, uint8_t* sha256_out, uint64_t* frames, uint64_t* packets) {
    return guarded([&] {
        if (!s || !data || !sizes) throw std::invalid_argument("invalid stream decode arguments");
        FrameSink fs;
        if (sink)
            fs = [&](int stream, uint64_t frame, const uint8_t* yuv, size_t bytes) {
                sink(user, stream, frame, yuv, bytes);
            };
        const StreamStats st =
            s->s->decode(data, sizes, total_frames, total_packets, expected_width, expected_height, fs);
        if (sha256_out)
            for (size_t b = 0; b < st.yuv_sha256.size(); ++b) std::memcpy(sha256_out + 32 * b, st.yuv_sha256[b].data(), 32);
        if (frames) *frames = st.frames;
        if (packets) *packets = st.packets;
        return 0;
    });
}

}  // extern "C"
