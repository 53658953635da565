// Whole-stream encode and decode over the engine's codecs: the reference's
// uf::IntegerCodec::encode / decode_stream_impl (src/integer_codec.cpp:215-292,
// 405-493) on the UF16 container of uf16_stream.h.
//
// A StreamCodec drives an image codec (I packets) and an optional video codec
// (P packets of 8 frames) of the same batch B: B independent streams are coded
// in lock step, each into its own bitstream.  Streams of one batch share the
// packet structure (types, QPs, reset flags, dimensions); decoding rejects a
// batch whose streams differ in it.
#pragma once

#include "engine.h"
#include "uf16_stream.h"

#include <array>
#include <cstdint>
#include <functional>
#include <vector>

namespace ufb {

struct EncodeSettings {
    uint32_t width = 0, height = 0;
    int qp_i = 0, qp_p = 0;
    int reset_interval = 0;  // <= 0: never reset the feature memory
    int intra_period = -1;   // <= 0: one I packet, 1: all intra, else a multiple of 8
};

struct StreamStats {
    uint64_t frames = 0;
    uint64_t packets = 0;
    std::vector<std::array<uint8_t, 32>> yuv_sha256;  // per stream, of the raw YUV420 frames
};

// Decoded frame of stream b: raw YUV420 (width * height * 3 / 2 bytes).
using FrameSink = std::function<void(int stream, uint64_t frame, const uint8_t* yuv, size_t bytes)>;

class StreamCodec {
public:
    StreamCodec(Codec& image, Codec* video, const uf16::Identity& image_id, const uf16::Identity& video_id);

    // IntegerCodec::encode of `count` frames per stream: frames host uint8
    // YUV444 [B][count][3][height][width].  Returns one bitstream per stream.
    std::vector<std::vector<uint8_t>> encode(const uint8_t* frames, uint64_t count, const EncodeSettings& s,
                                             StreamStats* stats);

    // IntegerCodec::decode_stream_impl of B bitstreams.  expected_width /
    // expected_height (0: unchecked) are the archive's dimensions.
    StreamStats decode(const uint8_t* const* data, const size_t* sizes, uint64_t total_frames,
                       uint64_t total_packets, uint32_t expected_width, uint32_t expected_height,
                       const FrameSink& sink);

    int batch() const { return image_.batch(); }

private:
    Codec& image_;
    Codec* video_;
    uf16::Preamble preamble_;
};

}  // namespace ufb
