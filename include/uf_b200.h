/*
 * uf_b200.h -- C ABI of the B200 (sm_100a) INT16 engine for the DCVC-UF HT-L
 * per-frame hot path.
 *
 * Arithmetic contract: "uf-int16-q9-w13-acc64-rna-sat-v1" (reference
 * include/uf/int16_ops.hpp:10-13): features Q9, weights Q13, exact int64 dot
 * products, rna(sum / 8192) with ties away from zero, + int16 Q9 bias, int16
 * saturation.  Results are bit-identical to the reference's CPU path.
 *
 * Conventions
 *   - Operator entry points take DEVICE pointers to dense NCHW tensors (the
 *     reference's torch::Tensor layout), plain sizes, and a cudaStream_t passed
 *     as void* (NULL = the legacy default stream).  They are asynchronous on
 *     that stream; the caller owns every input and output buffer.
 *   - Return value: 0 on success, a negative UFB_E* code on failure; the
 *     message is available from ufb_last_error() (thread-local).  Argument
 *     checks mirror the reference's TORCH_CHECKs and are done before any launch.
 *   - Kernel pipeline timeouts (a bounded wait that gave up) are recorded in a
 *     per-device status word read by ufb_device_status().
 */
#ifndef UF_B200_H
#define UF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UFB_OK 0
#define UFB_EINVAL -1   /* invalid argument (reference: std::invalid_argument / TORCH_CHECK) */
#define UFB_ERANGE -2   /* size exceeds an indexing or exactness bound (std::overflow_error) */
#define UFB_ECUDA -3    /* CUDA runtime error */
#define UFB_ESTREAM -4  /* corrupt or truncated entropy-coded stream (std::runtime_error) */
#define UFB_ESTATE -5   /* call not valid in the current codec state (std::runtime_error) */
#define UFB_EINTR -6    /* "UF operation interrupted" (ufb_set_interrupt; uf::ProcessInterrupt::check) */

/* Library version (major * 10000 + minor * 100 + patch). */
int ufb_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* ufb_last_error(void);

/* Testing aid (no reference counterpart): caps the persistent tensor-core and
 * depthwise convolution grids at n CTAs per launch (0 removes the cap), so
 * small problems still run many tiles per CTA.  Process-wide; not for
 * production. */
int ufb_set_conv_max_ctas(int n);

/* Testing aid (no reference counterpart): enable (1, the default) or disable
 * (0) the narrow recombination of the tensor-core convolution epilogue, used
 * for model layers whose weights keep LL + 256 X + 4096 within 32 bits for
 * every input.  Both settings give identical outputs; the switch lets tests
 * compare them.  Process-wide; not for production. */
int ufb_set_conv_narrow(int enable);

/* Synchronise `device` and return then clear its kernel status word:
 * 0 when no kernel reported a pipeline timeout since the last call, else the
 * first recorded code (1..4 = TMA producer / MMA / epilogue / drain wait). */
int ufb_device_status(int device);

/* ---------------------------------------------------------------------------
 * Operators.  Each replaces one function of the reference's CUDA extension,
 * include/uf/cuda_ops.hpp:10-23 (definitions src/cuda/conv.cu:114-135 and
 * src/cuda/elementwise.cu:49-98), with the same argument meaning and checks;
 * the output is caller-allocated instead of returned.
 * ------------------------------------------------------------------------- */

/* uf_conv (include/uf/cuda_ops.hpp:10-12): exact INT16 convolution.
 * x [n, ci, h, w], weight [co, ci/groups, kh, kw], bias [co] or NULL with
 * bias_bits 16 (int16, the reference's type) or 32 (int32, widened exactly as
 * src/int16_ops.cpp:163-167 does on the CPU path), out [n, co, oh, ow].
 * groups == 1, stride 1 or 2 (equal in both directions) and ci*kh*kw <= 8192
 * run on the tcgen05 tensor cores, depthwise 3x3 (stride 1, padding 1, int16
 * or no bias) on the depthwise kernel; other geometries use the direct int64
 * kernel (as the reference does). */
int ufb_conv2d(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
               const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w, int groups,
               int16_t* out, void* stream);

/* uf_conv_generic (include/uf/cuda_ops.hpp:13-15): same contract, always the
 * direct int64 kernel (no tensor cores). */
int ufb_conv2d_generic(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh,
                       int kw, const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w,
                       int groups, int16_t* out, void* stream);

/* uf_conv_baseline (include/uf/cuda_ops.hpp:16-18): same contract; the
 * tensor-core path whenever the geometry allows it. */
int ufb_conv2d_baseline(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh,
                        int kw, const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w,
                        int groups, int16_t* out, void* stream);

/* uf_add (include/uf/cuda_ops.hpp:19): out = sat(sum of 2..4 tensors). */
int ufb_add(int count, const int16_t* const* values, int64_t numel, int16_t* out, void* stream);

/* uf_mul (include/uf/cuda_ops.hpp:20): out = sat(rna(x * scale / 512)); both
 * 4-D, every scale extent 1 or equal to x's (broadcast). */
int ufb_mul(const int16_t* x, const int64_t* x_shape, const int16_t* scale, const int64_t* scale_shape,
            int16_t* out, void* stream);

/* uf_lut (include/uf/cuda_ops.hpp:21): out = table[x + 32768]; table has 65536
 * entries of table_bits 16 (int16) or 8 (uint8); out has the table's type. */
int ufb_lut(const int16_t* x, int64_t numel, const void* table, int table_bits, void* out, void* stream);

/* uf_bytes (include/uf/cuda_ops.hpp:22): out = rna((2 v - 255) * 512 / 510). */
int ufb_bytes(const uint8_t* x, int64_t numel, int16_t* out, void* stream);

/* uf_wsilu4 (include/uf/cuda_ops.hpp:23): x [n, 4c, h, w] -> out [n, c, h, w],
 * out[:, k] = sat(sum_{j<4} table[x[:, 4k + j] + 32768]). */
int ufb_wsilu4(const int16_t* x, int n, int c4, int h, int w, const int16_t* table, int16_t* out, void* stream);

/* Fixed-point backward bilinear warp (no reference counterpart: the
 * reference's only warp is the float DCVC-FM kernel block_mc_forward,
 * src/dcvc_fm_motion.cu:29-111, which no build target compiles).
 * feature [n, c, h, w] int16, flow [n, 2, h, w] int16 in Q9 pixels (x, y),
 * border clamp, out = sat(rna(sum of Q18 bilinear weights * taps / 2^18)).
 * Pipeline timeouts of its bounded waits are reported by ufb_device_status
 * (code 11). */
int ufb_warp(const int16_t* feature, const int16_t* flow, int n, int c, int h, int w, int16_t* out,
             void* stream);

/* ---------------------------------------------------------------------------
 * Split-layout operators.  The engine keeps activations in HBM as "split
 * NHWC": per pixel, a row of 2 * pitch bytes holding the low bytes (u8) of its
 * channels followed by their high bytes (s8); value = lo + 256 * hi.  pitch
 * and any channel offset are multiples of 16.  Callers that keep activations
 * resident in this layout avoid the NCHW conversions of ufb_conv2d.
 * ------------------------------------------------------------------------- */

/* NCHW int16 -> split (pixel_unshuffle(factor) fused; factor 1 = layout only).
 * out holds n x (h/f) x (w/f) pixels of c*f*f channels with row pitch `pitch`. */
int ufb_to_split(const int16_t* x, int n, int c, int h, int w, int factor, uint8_t* out, int pitch, void* stream);

/* split -> NCHW int16 (pixel_shuffle(factor) fused).  x holds n x h x w pixels
 * of c channels; out is [n, c/(f*f), h*f, w*f]. */
int ufb_from_split(const uint8_t* x, int n, int c, int h, int w, int pitch, int factor, int16_t* out,
                   void* stream);

/* Bytes of the prepared weight planes for a [co, ci, kh, kw] convolution. */
int64_t ufb_weight_bytes(int co, int ci, int kh, int kw);

/* Prepare int16 [co, ci, kh, kw] weights (device) into tensor-core planes
 * (device, ufb_weight_bytes() bytes). */
int ufb_prepare_weights(const int16_t* weight, int co, int ci, int kh, int kw, uint8_t* planes, void* stream);

/* uf_conv on split activations with prepared weights: stride 1, zero padding
 * (pad_h, pad_w), groups 1, ci*kh*kw <= 8192.  Uses no scratch memory. */
int ufb_conv2d_split(const uint8_t* x, int n, int ci, int h, int w, int x_pitch, const uint8_t* planes, int co,
                     int kh, int kw, const void* bias, int bias_bits, int pad_h, int pad_w, uint8_t* out,
                     int out_pitch, void* stream);

/* ---------------------------------------------------------------------------
 * Host rANS coder (no GPU needed).  Same wire format as the reference's
 * uf::EntropyEncoder / uf::EntropyDecoder (include/uf/entropy.hpp:12-46,
 * src/entropy.cpp:63-247): Y parts encoded last-first then Z, flushed as the
 * final state followed by the emitted bytes reversed; decode runs Z first,
 * then the Y parts in order.  CDF tables are the prepared model's
 * tables.{z,y}_cdf ([rows, width] int32) and tables.{z,y}_lengths.
 * ------------------------------------------------------------------------- */
typedef struct ufb_rans ufb_rans;

ufb_rans* ufb_rans_create(const int32_t* z_cdf, int z_rows, int z_width, const int32_t* z_len, const int32_t* y_cdf,
                          int y_rows, int y_width, const int32_t* y_len);
void ufb_rans_destroy(ufb_rans* r);

/* Encode Y parts (packed (symbol << 8) | cdf_index int16, EntropyEncoder::encode_y)
 * and Z symbols (NHWC int8, row z_offset + i % z_channels, encode_z) into one
 * stream (reset, parts last-first, Z, flush).  Returns the stream length (out
 * may be NULL to query it) or a negative UFB_E* code. */
int64_t ufb_rans_encode(ufb_rans* r, int nparts, const int16_t* const* parts, const size_t* part_lens,
                        const int8_t* z, size_t zn, int z_offset, int z_channels, uint8_t* out, size_t capacity);

/* Decode zn Z symbols, then each Y part's symbols from its CDF indexes
 * (EntropyDecoder::set_stream / decode_z / decode_y).  Corrupt or truncated
 * streams return UFB_ESTREAM with the reference's message. */
int ufb_rans_decode(ufb_rans* r, const uint8_t* data, size_t n, size_t zn, int z_offset, int z_channels,
                    int8_t* z_out, int nparts, const uint8_t* const* indexes, const size_t* index_lens,
                    int8_t* const* y_out);

/* ---------------------------------------------------------------------------
 * Model and codec (the reference's uf::Layers / uf::IntegerModel,
 * include/uf/layers.hpp:36-49 and include/uf/integer_model.hpp:19-73).
 * ------------------------------------------------------------------------- */
typedef struct ufb_model ufb_model;
typedef struct ufb_codec ufb_codec;

/* Upload a prepared model (uf::PreparedModel::tensors, include/uf/prepared.hpp:12-21)
 * to `device`: `count` host tensors with names, dtype codes (0 int16, 1 uint8,
 * 2 int32, 3 int8, 4 int64), ranks, concatenated shapes and host data.
 * variant: "htl" or "image" (the layer topology is derived from tensor
 * names as src/layers.cpp does).  The caller may free the host data on
 * return.  NULL on failure (see ufb_last_error). */
ufb_model* ufb_model_create(int device, const char* variant, int count, const char* const* names, const int* dtypes,
                            const int* ndims, const int64_t* shapes, const void* const* data);
void ufb_model_destroy(ufb_model* m);

/* uf::Layers::run(module, args) (src/layers.cpp:132-184) on host NCHW int16
 * tensors (shapes: 4 per argument).  A QP-table argument of the reference
 * (Layers::parameter(q_name, qp)) is named by q_name / qp.  "enc" / "dec" of
 * the image model include their pixel (un)shuffle(8) as in the reference.
 * The result is written to out (capacity elements), its shape to out_shape. */
int ufb_model_run(ufb_model* m, const char* module, int nargs, const int16_t* const* args, const int64_t* shapes,
                  const char* q_name, int qp, int16_t* out, int64_t capacity, int64_t* out_shape);

/* A codec holds the decoded-picture buffer (reference / memory / context) of
 * `batch` independent streams that are decoded together; every stream of a
 * batch shares the model, packet QP and reset flag, and has its own payload. */
ufb_codec* ufb_codec_create(ufb_model* model, int batch);
void ufb_codec_destroy(ufb_codec* c);

/* IntegerModel::set_skip_threshold: trunc(t * 512 + 0.5) must lie in [0, 32767]. */
int ufb_codec_set_skip_threshold(ufb_codec* c, double threshold);

/* IntegerModel::clear_dpb. */
int ufb_codec_clear_dpb(ufb_codec* c);

/* IntegerModel::add_ref_feature_from_frame: frames host int16 [batch][3][h][w]. */
int ufb_codec_add_ref_frames(ufb_codec* c, const int16_t* frames, int height, int width);

/* IntegerModel::decompress for every stream (src/integer_model.cpp:336-359).
 * frames_out: host int16 [batch][F][3][Hp][Wp] (Hp, Wp = height, width padded
 * to 16) or NULL; yuv_out: host uint8 [batch][F][width*height*3/2] YUV420
 * (IntegerCodec::raw_frame, src/integer_codec.cpp:294-323) or NULL.
 * Returns F (8 for a video model, 1 for the image model) or a UFB_E* code. */
int ufb_codec_decompress(ufb_codec* c, const uint8_t* const* payloads, const size_t* lengths, uint32_t width,
                         uint32_t height, int qp, int entropy_parallel, int reset, int16_t* frames_out,
                         uint8_t* yuv_out);

/* IntegerModel::compress (src/integer_model.cpp:312-334) with the frame
 * conversion of IntegerCodec::frame_tensor fused: frames host uint8 YUV444
 * [batch][channels][height][width] (channels = 3 per frame).  Each stream's
 * payload is written at payload_out + b * capacity, its length to lengths[b].
 * frames_out (optional) receives the reconstruction as in decompress.
 * Returns the number of reconstructed frames or a UFB_E* code. */
int ufb_codec_compress(ufb_codec* c, const uint8_t* frames, int channels, int height, int width, int qp, int reset,
                       uint8_t* payload_out, size_t capacity, size_t* lengths, int16_t* frames_out);

/* DPB state views (IntegerModel::reference/memory/context): which 0, 1, 2.
 * Writes NCHW int16 and its shape; returns 1 when the state is undefined. */
int ufb_codec_state(ufb_codec* c, int which, int16_t* out, int64_t capacity, int64_t* shape4);

/* SHA-256 of a DPB state tensor (which 0, 1, 2) as NCHW int16 little-endian
 * bytes -- the tensor_hash of the reference's check-int16 state records
 * (src/int16_validation.cpp:110-144).  Returns 0, or 1 (digest untouched) when
 * the state is undefined. */
int ufb_codec_state_hash(ufb_codec* c, int which, uint8_t* sha256_32);

/* Process-wide cancellation (uf::ProcessInterrupt, include/uf/process.hpp:66-79):
 * while set, codec compress/decompress calls and the stream encoder / decoder
 * (between packets and frames) stop with UFB_EINTR "UF operation interrupted".
 * Lock-free, so a signal handler may call it. */
void ufb_set_interrupt(int on);
int ufb_interrupt_requested(void);

/* Seconds the last decompress/compress spent in host entropy coding. */
double ufb_codec_host_seconds(ufb_codec* c);

/* IntegerCodec's I-to-P hand-off (video->add_ref_feature_from_frame(frames.at(0)),
 * src/integer_codec.cpp:453-456) without leaving the GPU: the video codec's
 * DPB is cleared and its reference becomes the image codec's last
 * reconstruction (same batch). */
int ufb_codec_set_reference_from(ufb_codec* video, ufb_codec* image);

/* Run the codec's work on a caller-owned CUDA stream (NULL: the codec's own
 * stream, the default).  Like the reference's pooled per-codec stream
 * (src/integer_codec.cpp:30-49), all of a codec's kernels use one stream. */
int ufb_codec_set_stream(ufb_codec* c, void* stream);

/* Measurement: with profiling on, every tensor-core convolution launch is
 * bracketed by CUDA events on the codec's stream.  ufb_codec_stats reports the
 * kernels launched, the convolution launches, their algorithmic int16 MACs and
 * summed event time (ms) since the last reset (reset != 0 clears them). */
int ufb_codec_profile(ufb_codec* c, int enable);
int ufb_codec_stats(ufb_codec* c, int reset, int64_t* launches, int64_t* conv_launches, double* conv_int16_macs,
                    double* conv_ms);
/* Per launch shape breakdown of the profiled convolutions (tensor-core and
 * depthwise) since the last reset, one tab-separated line per shape:
 * "<shape>\t<launches>\t<int16 MACs>\t<ms>\t<algorithmic DRAM bytes>" (the launches'
 * inputs and residuals read once, outputs written once, weights).  Writes at most capacity - 1 bytes
 * plus a terminating zero and sets *length to the full text length. */
int ufb_codec_shape_table(ufb_codec* c, char* text, int64_t capacity, int64_t* length);

/* ---------------------------------------------------------------------------
 * UF16 bitstream container (include/uf/bitstream.hpp:20-107,
 * src/bitstream.cpp:173-360): host-only, no GPU needed.
 *
 *   preamble  "UF16" 01 00 00 00 + image identity (32 B) + video identity (32 B)
 *   NAL unit  header byte type << 4 | sps_id (type 0 SPS, 1 I packet, 2 P packet)
 *   SPS       adaptive height, adaptive width
 *   packet    qp, entropy_parallel << 1 | reset, adaptive payload length, payload
 *   adaptive  1, 2 or 4 bytes for values below 2^7, 2^14, 2^30
 *
 * Writers append at out (capacity bytes) and return the bytes written, or a
 * negative UFB_E* code (UFB_ERANGE when capacity is too small or a value
 * exceeds 30 bits, UFB_EINVAL for an invalid SPS or packet).  Readers start at
 * *pos and advance it; a truncated or malformed stream gives UFB_ESTREAM with
 * the reference's message ("Truncated UF bitstream", "Unsupported UF NAL
 * type", ...).
 * ------------------------------------------------------------------------- */
#define UFB_NAL_SPS 0
#define UFB_NAL_INTRA 1
#define UFB_NAL_PREDICTED 2

typedef struct ufb_uf16_nal {
    int type;                  /* UFB_NAL_* */
    int sps_id;                /* 0..15 */
    uint32_t width, height;    /* SPS */
    int qp;                    /* packets: 0..255 on the wire */
    int entropy_parallel;      /* packets: flags >> 1 */
    int reset;                 /* packets: flags & 1 (reset_feature_memory) */
    uint64_t payload_offset;   /* packets: payload position in the stream */
    uint64_t payload_length;
} ufb_uf16_nal;

typedef struct ufb_uf16_summary {
    int integer;               /* 1: UF16 preamble present */
    uint8_t image_identity[32];
    uint8_t video_identity[32];
    uint32_t width, height;    /* dimensions of the coded packets */
    uint64_t packets, intra_packets, predicted_packets;
    uint64_t maximum_frames;   /* I packets count 1, P packets 8 ("ld": 1) */
} ufb_uf16_summary;

/* write_preamble of an integer stream (72 bytes). */
int64_t ufb_uf16_write_preamble(const uint8_t* image_identity, const uint8_t* video_identity, uint8_t* out,
                                size_t capacity);
/* write_sps: id < 16, width and height nonzero. */
int64_t ufb_uf16_write_sps(int id, uint32_t width, uint32_t height, uint8_t* out, size_t capacity);
/* write_packet: type UFB_NAL_INTRA or UFB_NAL_PREDICTED, sps_id < 16,
 * 0 <= qp < 256, 0 <= entropy_parallel < 128, length < 2^30. */
int64_t ufb_uf16_write_packet(int type, int sps_id, int qp, int entropy_parallel, int reset, const uint8_t* payload,
                              size_t length, uint8_t* out, size_t capacity);
/* write_uint_adaptive / read_uint_adaptive. */
int64_t ufb_uf16_write_uint(uint32_t value, uint8_t* out, size_t capacity);
int ufb_uf16_read_uint(const uint8_t* data, size_t size, size_t* pos, uint32_t* value);
/* read_preamble: *integer = 0 (nothing consumed) when the stream does not
 * start with 'U'; identities are written only for an integer stream. */
int ufb_uf16_read_preamble(const uint8_t* data, size_t size, size_t* pos, int* integer, uint8_t* image_identity,
                           uint8_t* video_identity);
/* Next NAL unit (read_optional_header + read_sps / read_packet): returns 1
 * and fills *nal, or 0 at the clean end of the stream. */
int ufb_uf16_next(const uint8_t* data, size_t size, size_t* pos, ufb_uf16_nal* nal);
/* scan_bitstream: variant "ld", "hts" or "htl"; expected_frames < 0 for none. */
int ufb_uf16_scan(const uint8_t* data, size_t size, const char* variant, int64_t expected_frames,
                  ufb_uf16_summary* out);

/* SHA-256 of size bytes (OpenSSL EVP, as the reference). */
int ufb_sha256(const void* data, size_t size, uint8_t* digest32);

/* prepared_identity (src/prepared.cpp:64-105): the content hash of a prepared
 * model, 64 lowercase hex digits and a terminating zero written to hex65.
 * The tensor table is the one ufb_model_create takes; format is normally
 * "dcvc-uf-prepared-v1" and arithmetic "uf-int16-q9-w13-acc64-rna-sat-v1". */
int ufb_prepared_identity(const char* format, const char* arithmetic, const char* variant, const char* source_sha256,
                          int count, const char* const* names, const int* dtypes, const int* ndims,
                          const int64_t* shapes, const void* const* data, char* hex65);

/* ---------------------------------------------------------------------------
 * Whole streams (uf::IntegerCodec::encode / decode_stream_impl,
 * src/integer_codec.cpp:215-292, 405-493): an image codec and an optional
 * video codec of the same batch B code B independent UF16 streams in lock
 * step.  The stream codec borrows both codecs (destroy it first).
 * ------------------------------------------------------------------------- */
typedef struct ufb_stream_codec ufb_stream_codec;

/* Identities: the 32-byte prepared-model identities written to (and required
 * in) the preamble; video_identity is ignored (zeros) without a video codec. */
ufb_stream_codec* ufb_stream_codec_create(ufb_codec* image, ufb_codec* video, const uint8_t* image_identity,
                                          const uint8_t* video_identity);
void ufb_stream_codec_destroy(ufb_stream_codec* s);

/* IntegerCodec::encode of count frames per stream: frames host uint8 YUV444
 * [B][count][3][height][width].  Packet structure as the reference: an I packet
 * first and wherever frame % intra_period == 1 (intra_period 1: all intra;
 * <= 0: only the first), P packets of 8 frames (the last padded by repeating
 * its last frame), reset when (frame + 8) % reset_interval == 1.  Stream b is
 * written at out + b * capacity, its length to lengths[b]; *packets receives
 * the packet count.  Returns 0 or a UFB_E* code. */
int ufb_stream_encode(ufb_stream_codec* s, const uint8_t* frames, uint64_t count, uint32_t width, uint32_t height,
                      int qp_i, int qp_p, int reset_interval, int intra_period, uint8_t* out, size_t capacity,
                      size_t* lengths, uint64_t* packets);

/* Decoded-frame callback: raw YUV420 frame `frame` of stream `stream`. */
typedef void (*ufb_frame_sink)(void* user, int stream, uint64_t frame, const uint8_t* yuv, size_t bytes);

/* IntegerCodec::decode_stream_impl of B streams (data[b], sizes[b]): checks
 * the preamble identities, decodes every packet, hands each frame to sink
 * (may be NULL) and returns in sha256_out [B][32] the SHA-256 of each
 * stream's raw YUV420 frames (the archive's decoded_yuv_sha256).  The frame
 * and packet counts must equal total_frames / total_packets ("Incomplete UF
 * integer bitstream" otherwise); expected_width / expected_height (0: any)
 * are the archive metadata's dimensions. */
int ufb_stream_decode(ufb_stream_codec* s, const uint8_t* const* data, const size_t* sizes, uint64_t total_frames,
                      uint64_t total_packets, uint32_t expected_width, uint32_t expected_height, ufb_frame_sink sink,
                      void* user, uint8_t* sha256_out, uint64_t* frames, uint64_t* packets);

/* ---------------------------------------------------------------------------
 * No-allocation convolution (no counterpart in the reference: its uf_conv
 * always allocates its output and temporaries through the caller's allocator).
 * ------------------------------------------------------------------------- */

/* Fixed scratch capacity of ufb_conv2d_noalloc, per GPU, in bytes. */
#define UFB_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)

/* ufb_conv2d without any device allocation, for callers that cannot allocate
 * GPU memory while they process -- for example a host application that
 * reserves all device memory up front and hands this library only input and
 * output buffers, or a real-time frame loop where an allocation could stall
 * or fail part-way through a stream.  Same arguments, checks and results as
 * ufb_conv2d; the caller still owns x, weight, bias and out.
 *
 * Tensor-core geometries stage the input, the prepared weights and the output
 * in one fixed device array of UFB_NOALLOC_SCRATCH_BYTES that the library
 * holds on every GPU it is loaded on until the process exits; a call whose
 * staging would exceed it fails with UFB_ERANGE and a message giving the
 * needed size.  Other geometries (grouped, strided, K > 8192) use the direct
 * kernel, which needs no scratch.
 *
 * The first call on a device resolves the array's device address with that
 * device current; make that first call before any stream capture.  All calls
 * on a device share the one array and it keeps the last call's contents, so
 * calls that overlap on the GPU (different streams, or host threads) race:
 * serialise them.  No part of the array needs to start at zero. */
int ufb_conv2d_noalloc(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                       const void* bias, int bias_bits, int stride_h, int stride_w, int pad_h, int pad_w, int groups,
                       int16_t* out, void* stream);

/* Measurement utility (no reference counterpart): launches `ctas` CTAs that
 * each issue `iters` x 4 dense tcgen05 kind::i8 M=128 N=256 K=32 MMAs from
 * resident shared-memory tiles; *int8_ops receives the operation count
 * (2 per multiply-add).  The caller times the launch on `stream` to obtain
 * the int8 tensor-pipe peak used as the convolution roofline. */
int ufb_probe_i8_peak(int iters, int ctas, void* stream, int64_t* int8_ops);

#ifdef __cplusplus
}
#endif

#endif /* UF_B200_H */
