// Whole-stream encode / decode (declarations in stream_codec.h).
#include "stream_codec.h"

#include "digest.h"
#include "interrupt.h"
#include "rans.h"  // StreamError

#include <algorithm>
#include <cstring>
#include <future>
#include <optional>
#include <memory>
#include <stdexcept>

namespace ufb {

namespace {

constexpr int kChunk = 8;  // frames per P packet of the htl / hts video models

}  // namespace

StreamCodec::StreamCodec(Codec& image, Codec* video, const uf16::Identity& image_id, const uf16::Identity& video_id)
    : image_(image), video_(video) {
    if (video && video->batch() != image.batch()) throw std::invalid_argument("image and video codec batches differ");
    if (image.frames_per_packet() != 1 || (video && video->frames_per_packet() != kChunk))
        throw std::invalid_argument("UF prepared models do not match the codec variant");
    preamble_.integer = true;
    preamble_.image_identity = image_id;
    preamble_.video_identity = video ? video_id : uf16::Identity{};
}

// IntegerCodec::encode (src/integer_codec.cpp:215-292): one I packet first,
// then P packets of 8 frames (the last one padded by repeating its last
// frame), a new I packet at every frame index count % intra_period == 1, and
// the feature memory reset when (count + 8) % reset_interval == 1.
std::vector<std::vector<uint8_t>> StreamCodec::encode(const uint8_t* frames, uint64_t count, const EncodeSettings& s,
                                                      StreamStats* stats) {
    if (!frames || !s.width || !s.height || s.width % 2 || s.height % 2 || s.qp_i < 0 || s.qp_i >= 64 ||
        s.qp_p < 0 || s.qp_p >= 64 || (s.intra_period > 1 && s.intra_period % kChunk))
        throw std::invalid_argument("Invalid UF encode settings");
    const int B = batch();
    const size_t frame_bytes = static_cast<size_t>(3) * s.width * s.height;
    std::vector<std::vector<uint8_t>> out(B);
    for (int b = 0; b < B; ++b) {
        uf16::Writer w(out[b]);
        w.preamble(preamble_);
        w.sps(uf16::Sps{0, s.width, s.height});
    }
    std::vector<uint8_t> staging(static_cast<size_t>(B) * kChunk * frame_bytes);
    std::vector<std::vector<uint8_t>> payloads;
    uint64_t done = 0, packets = 0;
    while (done < count) {
        check_interrupt();
        const bool intra = done == 0 || s.intra_period == 1 ||
                           (s.intra_period > 1 && done != 1 && done % static_cast<uint64_t>(s.intra_period) == 1);
        const uint64_t valid = std::min<uint64_t>(intra ? 1 : kChunk, count - done);
        const int coded = intra ? 1 : kChunk;
        if (!intra && !video_) throw std::runtime_error("UF video model is required for P packets");
        for (int b = 0; b < B; ++b)
            for (int i = 0; i < coded; ++i) {
                const uint64_t src = done + std::min<uint64_t>(static_cast<uint64_t>(i), valid - 1);
                std::memcpy(staging.data() + (static_cast<size_t>(b) * coded + i) * frame_bytes,
                            frames + (static_cast<size_t>(b) * count + src) * frame_bytes, frame_bytes);
            }
        const bool reset = !intra && s.reset_interval > 0 &&
                           (done + kChunk) % static_cast<uint64_t>(s.reset_interval) == 1;
        const int h = static_cast<int>(s.height), wd = static_cast<int>(s.width);
        if (intra) {
            image_.compress(staging.data(), 3, h, wd, s.qp_i, false, payloads, nullptr);
            if (video_) video_->set_reference_from(image_);
        } else {
            video_->compress(staging.data(), 3 * kChunk, h, wd, s.qp_p, reset, payloads, nullptr);
        }
        for (int b = 0; b < B; ++b) {
            uf16::Packet p;
            p.type = intra ? uf16::Nal::intra : uf16::Nal::predicted;
            p.qp = static_cast<uint8_t>(intra ? s.qp_i : s.qp_p);
            p.entropy_parallel = 1;
            p.reset = reset;
            p.payload = payloads[b].data();
            p.length = payloads[b].size();
            uf16::Writer(out[b]).packet(p);
        }
        done += valid;
        ++packets;
    }
    if (!done) throw std::runtime_error("UF input yielded no frames");
    if (stats) {
        stats->frames = done;
        stats->packets = packets;
    }
    return out;
}

// IntegerCodec::decode_stream_impl (src/integer_codec.cpp:405-493).
StreamStats StreamCodec::decode(const uint8_t* const* data, const size_t* sizes, uint64_t total_frames,
                                uint64_t total_packets, uint32_t expected_width, uint32_t expected_height,
                                const FrameSink& sink) {
    const int B = batch();
    if (!data || !sizes) throw std::invalid_argument("no bitstreams");
    std::vector<uf16::Reader> in;
    in.reserve(B);
    for (int b = 0; b < B; ++b) {
        if (!data[b] && sizes[b]) throw std::invalid_argument("null bitstream");
        in.emplace_back(data[b], sizes[b]);
        const uf16::Preamble p = in[b].preamble();
        if (!p.integer || p.image_identity != preamble_.image_identity ||
            p.video_identity != preamble_.video_identity)
            throw StreamError("UF integer runtime/prepared-model identity mismatch");
    }
    std::vector<std::unique_ptr<Sha256>> digests;
    for (int b = 0; b < B; ++b) digests.push_back(std::make_unique<Sha256>());
    std::array<std::optional<uf16::Sps>, 16> table{};
    StreamStats stats;
    bool first = true;
    std::vector<const uint8_t*> payloads(B);
    std::vector<size_t> lengths(B);
    std::vector<uint8_t> yuv;
    const auto differ = [] { return StreamError("UF streams of one batch differ in packet structure"); };
    for (;;) {
        check_interrupt();
        uf16::Nal type;
        uint8_t id;
        const bool more = in[0].header(type, id);
        for (int b = 1; b < B; ++b) {
            uf16::Nal t2;
            uint8_t id2;
            if (in[b].header(t2, id2) != more || (more && (t2 != type || id2 != id))) throw differ();
        }
        if (!more) break;
        if (type == uf16::Nal::sps) {
            const uf16::Sps s = in[0].sps(id);
            for (int b = 1; b < B; ++b) {
                const uf16::Sps s2 = in[b].sps(id);
                if (s2.width != s.width || s2.height != s.height) throw differ();
            }
            if ((expected_width && s.width != expected_width) || (expected_height && s.height != expected_height))
                throw StreamError("Bitstream dimensions differ from archive metadata");
            table[id] = s;
            continue;
        }
        if (!table[id] || stats.frames >= total_frames) throw StreamError("Unexpected UF packet or unknown SPS");
        const uf16::Sps& s = *table[id];
        uf16::Packet p0;
        for (int b = 0; b < B; ++b) {
            const uf16::Packet p = in[b].packet(type, id);
            if (b == 0) p0 = p;
            else if (p.qp != p0.qp || p.reset != p0.reset || p.entropy_parallel != p0.entropy_parallel) throw differ();
            payloads[b] = p.payload;
            lengths[b] = p.length;
        }
        const bool intra = type == uf16::Nal::intra;
        if (first && !intra) throw StreamError("UF stream must start with an I packet");
        first = false;
        // IntegerModel::decompress (src/integer_model.cpp:336-343) and the
        // YUV420 conversion require these
        if (p0.entropy_parallel != 1 || p0.qp >= 64 || s.width % 2 || s.height % 2)
            throw std::invalid_argument("Unsupported UF integer packet parameters");
        const size_t yuv_frame = static_cast<size_t>(s.width) * s.height * 3 / 2;
        const int F = intra ? 1 : kChunk;
        yuv.resize(static_cast<size_t>(B) * F * yuv_frame);
        if (intra) {
            image_.decompress(payloads.data(), lengths.data(), s.width, s.height, p0.qp, false, nullptr, yuv.data());
            if (video_) video_->set_reference_from(image_);
        } else {
            if (!video_) throw std::runtime_error("UF P packet requires a video model");
            video_->decompress(payloads.data(), lengths.data(), s.width, s.height, p0.qp, p0.reset, nullptr,
                               yuv.data());
        }
        const int valid = static_cast<int>(std::min<uint64_t>(F, total_frames - stats.frames));
        // per-stream digests run in parallel; the sink sees frames in order
        std::vector<std::future<void>> jobs;
        for (int b = 1; b < B; ++b)
            jobs.push_back(std::async(std::launch::async, [&, b] {
                digests[b]->update(yuv.data() + static_cast<size_t>(b) * F * yuv_frame, valid * yuv_frame);
            }));
        digests[0]->update(yuv.data(), valid * yuv_frame);
        for (auto& j : jobs) j.get();
        if (sink)
            for (int b = 0; b < B; ++b)
                for (int f = 0; f < valid; ++f) {
                    check_interrupt();
                    sink(b, stats.frames + f, yuv.data() + (static_cast<size_t>(b) * F + f) * yuv_frame, yuv_frame);
                }
        stats.frames += valid;
        ++stats.packets;
    }
    if (stats.frames != total_frames || stats.packets != total_packets)
        throw StreamError("Incomplete UF integer bitstream");
    for (int b = 0; b < B; ++b) stats.yuv_sha256.push_back(digests[b]->finish());
    return stats;
}

}  // namespace ufb
