// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// C-ABI shim around the reference's own CPU INT16 path, so tests and the
// bench's CPU arm can run the UNMODIFIED reference sources
//   src/int16_ops.cpp, src/layers.cpp, src/integer_model.cpp, src/entropy.cpp,
//   src/bitstream.cpp, src/integer_codec.cpp, src/bitstream_output.cpp,
//   src/inference_environment.cpp
// (compiled in place from the reference checkout by oracle/Makefile) on the
// same seeded inputs the CUDA engine receives.  Only a few symbols the
// reference declares but whose defining files drag in unrelated subsystems are
// supplied here: uf::ProcessInterrupt::check() (include/uf/process.hpp:68-79;
// a no-op, nothing here installs signal handlers), uf::PreparedModel::tensor()
// (include/uf/prepared.hpp:19-20; a plain map lookup),
// uf::python_path_normalize (include/uf/python_path.hpp:25; the identity,
// reached only by uf::filesize, which nothing here calls) and the owning
// descriptor uf::FileDescriptor's destructor, reset and checked close
// (include/uf/process.hpp:16-32; POSIX close(2) on the owned descriptor), which
// the bitstream file writer of src/bitstream_output.cpp uses.
//
// Every entry point returns 0 on success and -1 on a thrown exception, whose
// message is kept in a thread-local string (ufref_last_error()).
#include "uf/bitstream.hpp"
#include "uf/entropy.hpp"
#include "uf/int16_ops.hpp"
#include "uf/integer_codec.hpp"
#include "uf/integer_model.hpp"
#include "uf/layers.hpp"
#include "uf/prepared.hpp"
#include "uf/process.hpp"
#include "uf/python_path.hpp"

#include <ATen/Parallel.h>
#include <torch/torch.h>

#include <array>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <optional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <system_error>
#include <vector>

#include <cerrno>
#include <unistd.h>

namespace uf {
void ProcessInterrupt::check() {}
const torch::Tensor& PreparedModel::tensor(const std::string& name) const {
    const auto it = tensors.find(name);
    if (it == tensors.end()) throw std::runtime_error("Missing prepared UF tensor: " + name);
    return it->second;
}
std::filesystem::path python_path_normalize(const std::filesystem::path& path) { return path; }
FileDescriptor::~FileDescriptor() { reset(); }
void FileDescriptor::reset(int value) {
    const int old = value_;
    value_ = value;
    if (old >= 0 && old != value) ::close(old);
}
void FileDescriptor::close_checked(const std::string& context) {
    const int fd = value_;
    value_ = -1;
    if (fd >= 0 && ::close(fd) != 0) throw std::system_error(errno, std::generic_category(), context);
}
}  // namespace uf

namespace {

thread_local std::string g_error;

template <class F>
int guarded(F&& fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
    } catch (...) {
        g_error = "unknown exception";
    }
    return -1;
}

// dtype codes shared with oracle/__init__.py
torch::ScalarType dtype_of(int code) {
    switch (code) {
        case 0: return torch::kInt16;
        case 1: return torch::kUInt8;
        case 2: return torch::kInt32;
        case 3: return torch::kInt8;
        case 4: return torch::kInt64;
    }
    throw std::invalid_argument("bad dtype code");
}

torch::Tensor wrap(const void* data, std::vector<int64_t> shape, torch::ScalarType type) {
    return torch::from_blob(const_cast<void*>(data), shape, torch::TensorOptions().dtype(type)).clone();
}

void emit(const torch::Tensor& value, void* out, int64_t capacity_bytes, int64_t* shape4) {
    const auto t = value.contiguous();
    const auto bytes = static_cast<int64_t>(t.numel() * t.element_size());
    if (bytes > capacity_bytes) throw std::length_error("output buffer too small");
    if (bytes) std::memcpy(out, t.data_ptr(), bytes);
    if (shape4) {
        for (int d = 0; d < 4; ++d) shape4[d] = d < t.dim() ? t.size(d) : 1;
    }
}

struct RefModel {
    uf::PreparedModel prepared;
    std::unique_ptr<uf::IntegerModel> model;
    std::unique_ptr<uf::Layers> layers;
    std::vector<uint8_t> payload;
    std::vector<torch::Tensor> frames;
};

}  // namespace

extern "C" {

const char* ufref_last_error() { return g_error.c_str(); }

int ufref_set_threads(int threads) {
    return guarded([&] { torch::set_num_threads(threads); });
}

int ufref_get_threads() { return at::get_num_threads(); }

// uf::int16::conv2d on CPU == conv2d_reference (src/int16_ops.cpp:132-171).
// bias_dtype: 0 = int16, 2 = int32 (the reference widens either to int64).
int ufref_conv2d(const int16_t* x, const int64_t* xs, const int16_t* w, const int64_t* ws,
                 const void* bias, int bias_dtype, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, int64_t groups, int16_t* out, int64_t capacity, int64_t* os) {
    return guarded([&] {
        const auto input = wrap(x, {xs[0], xs[1], xs[2], xs[3]}, torch::kInt16);
        const auto weight = wrap(w, {ws[0], ws[1], ws[2], ws[3]}, torch::kInt16);
        torch::Tensor b;
        if (bias) b = wrap(bias, {ws[0]}, dtype_of(bias_dtype));
        emit(uf::int16::conv2d(input, weight, b, sh, sw, ph, pw, groups), out, capacity * 2, os);
    });
}

int ufref_add(int count, const int16_t* const* values, int64_t numel, int16_t* out) {
    return guarded([&] {
        std::vector<torch::Tensor> operands;
        for (int i = 0; i < count; ++i) operands.push_back(wrap(values[i], {numel}, torch::kInt16));
        emit(uf::int16::add(operands), out, numel * 2, nullptr);
    });
}

int ufref_multiply(const int16_t* x, const int64_t* xs, const int16_t* s, const int64_t* ss,
                   int16_t* out) {
    return guarded([&] {
        const auto value = wrap(x, {xs[0], xs[1], xs[2], xs[3]}, torch::kInt16);
        const auto scale = wrap(s, {ss[0], ss[1], ss[2], ss[3]}, torch::kInt16);
        emit(uf::int16::multiply(value, scale), out, value.numel() * 2, nullptr);
    });
}

int ufref_lookup(const int16_t* x, int64_t numel, const void* table, int table_dtype, void* out) {
    return guarded([&] {
        const auto value = wrap(x, {numel}, torch::kInt16);
        const auto lut = wrap(table, {65536}, dtype_of(table_dtype));
        const auto result = uf::int16::lookup(value, lut);
        emit(result, out, numel * result.element_size(), nullptr);
    });
}

int ufref_wsilu4(const int16_t* x, const int64_t* xs, const int16_t* table, int16_t* out) {
    return guarded([&] {
        const auto value = wrap(x, {xs[0], xs[1], xs[2], xs[3]}, torch::kInt16);
        const auto lut = wrap(table, {65536}, torch::kInt16);
        emit(uf::int16::wsilu4(value, lut), out, value.numel() / 4 * 2, nullptr);
    });
}

int ufref_from_bytes(const uint8_t* x, int64_t numel, int16_t* out) {
    return guarded([&] {
        emit(uf::int16::from_bytes(wrap(x, {numel}, torch::kUInt8)), out, numel * 2, nullptr);
    });
}

int ufref_divide_round(const int64_t* x, int64_t numel, int64_t denominator, int64_t* out) {
    return guarded([&] {
        emit(uf::int16::divide_round(wrap(x, {numel}, torch::kInt64), denominator), out,
             numel * 8, nullptr);
    });
}

int ufref_symbols(const int16_t* x, int64_t numel, int8_t* out) {
    return guarded([&] { emit(uf::int16::symbols(wrap(x, {numel}, torch::kInt16)), out, numel, nullptr); });
}

int ufref_reciprocal(const int16_t* x, int64_t numel, int16_t* out) {
    return guarded([&] { emit(uf::int16::reciprocal(wrap(x, {numel}, torch::kInt16)), out, numel * 2, nullptr); });
}

int ufref_pixel_shuffle(const int16_t* x, const int64_t* xs, int64_t factor, int unshuffle,
                        int16_t* out, int64_t* os) {
    return guarded([&] {
        const auto value = wrap(x, {xs[0], xs[1], xs[2], xs[3]}, torch::kInt16);
        const auto result = unshuffle ? uf::pixel_unshuffle(value, factor) : uf::pixel_shuffle(value, factor);
        emit(result, out, value.numel() * 2, os);
    });
}

// ---- model (uf::IntegerModel / uf::Layers, src/integer_model.cpp, src/layers.cpp) ----

void* ufref_model_new(const char* variant, int count, const char* const* names, const int* dtypes,
                      const int* ndims, const int64_t* shapes, const void* const* data) {
    auto handle = std::make_unique<RefModel>();
    const int rc = guarded([&] {
        auto& p = handle->prepared;
        p.format = "dcvc-uf-prepared-v1";
        p.arithmetic = uf::int16::arithmetic_id;
        p.variant = variant;
        const int64_t* cursor = shapes;
        for (int i = 0; i < count; ++i) {
            std::vector<int64_t> shape(cursor, cursor + ndims[i]);
            cursor += ndims[i];
            p.tensors[names[i]] = wrap(data[i], shape, dtype_of(dtypes[i]));
        }
        handle->model = std::make_unique<uf::IntegerModel>(p, torch::kCPU, true);
        handle->layers = std::make_unique<uf::Layers>(p, torch::kCPU);
    });
    return rc == 0 ? handle.release() : nullptr;
}

void ufref_model_free(void* h) { delete static_cast<RefModel*>(h); }

int ufref_model_set_skip(void* h, double threshold) {
    return guarded([&] { static_cast<RefModel*>(h)->model->set_skip_threshold(threshold); });
}

int ufref_model_clear_dpb(void* h) {
    return guarded([&] { static_cast<RefModel*>(h)->model->clear_dpb(); });
}

int ufref_model_add_ref(void* h, const int16_t* frame, const int64_t* fs) {
    return guarded([&] {
        static_cast<RefModel*>(h)->model->add_ref_feature_from_frame(
            wrap(frame, {fs[0], fs[1], fs[2], fs[3]}, torch::kInt16));
    });
}

// IntegerModel::compress (src/integer_model.cpp:312-334).  The payload and the
// reconstructed frames are kept in the handle; fetch them with the getters.
int ufref_model_compress(void* h, const int16_t* frames, const int64_t* fs, int qp, int reset) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        auto result = m->model->compress(wrap(frames, {fs[0], fs[1], fs[2], fs[3]}, torch::kInt16),
                                         qp, reset != 0);
        m->payload = std::move(result.payload);
        m->frames = std::move(result.frames);
    });
}

// IntegerModel::decompress (src/integer_model.cpp:336-359).
int ufref_model_decompress(void* h, const uint8_t* payload, int64_t length, uint32_t width,
                           uint32_t height, int qp, int reset) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        std::vector<uint8_t> bytes(payload, payload + length);
        m->frames = m->model->decompress(bytes, width, height, qp, 1, reset != 0);
    });
}

int64_t ufref_model_payload(void* h, uint8_t* out, int64_t capacity) {
    auto* m = static_cast<RefModel*>(h);
    const auto n = static_cast<int64_t>(m->payload.size());
    if (out && capacity >= n && n) std::memcpy(out, m->payload.data(), n);
    return n;
}

int ufref_model_frame_count(void* h) { return static_cast<int>(static_cast<RefModel*>(h)->frames.size()); }

int ufref_model_frame(void* h, int index, int16_t* out, int64_t capacity, int64_t* shape4) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        emit(m->frames.at(index), out, capacity * 2, shape4);
    });
}

// which: 0 = reference, 1 = memory, 2 = context.  Returns 1 when the state is
// undefined (Python None), 0 after copying, -1 on error.
int ufref_model_state(void* h, int which, int16_t* out, int64_t capacity, int64_t* shape4) {
    int undefined = 0;
    const int rc = guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        const auto& t = which == 0 ? m->model->reference() : which == 1 ? m->model->memory() : m->model->context();
        if (!t.defined()) { undefined = 1; return; }
        emit(t, out, capacity * 2, shape4);
    });
    return rc ? rc : undefined;
}

// uf::Layers::run (src/layers.cpp:132-184) for per-module parity: args are
// int16 NCHW tensors; the result is copied to out.
int ufref_layers_run(void* h, const char* module, int count, const int16_t* const* args,
                     const int64_t* shapes, int16_t* out, int64_t capacity, int64_t* shape4) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        std::vector<torch::Tensor> values;
        for (int i = 0; i < count; ++i) {
            const int64_t* s = shapes + 4 * i;
            values.push_back(wrap(args[i], {s[0], s[1], s[2], s[3]}, torch::kInt16));
        }
        emit(m->layers->run(module, values), out, capacity * 2, shape4);
    });
}

// uf::Layers::parameter (src/layers.cpp:63-72), i.e. table[qp:qp+1,:,None,None].
int ufref_layers_parameter(void* h, const char* name, int64_t qp, int16_t* out, int64_t capacity,
                           int64_t* shape4) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        emit(m->layers->parameter(name, qp), out, capacity * 2, shape4);
    });
}

int ufref_layers_reconstruct(void* h, const int16_t* feature, const int64_t* fs, int for_reset,
                             int index, int16_t* out, int64_t capacity, int64_t* shape4) {
    return guarded([&] {
        auto* m = static_cast<RefModel*>(h);
        const auto frames = m->layers->reconstruct(wrap(feature, {fs[0], fs[1], fs[2], fs[3]}, torch::kInt16),
                                                   for_reset != 0);
        emit(frames.at(index), out, capacity * 2, shape4);
    });
}

// ---- rANS (src/entropy.cpp) ----

struct RefRans {
    uf::EntropyEncoder encoder;
    uf::EntropyDecoder decoder;
    std::vector<uint8_t> out;
};

void* ufref_rans_new(const int32_t* z_cdf, int64_t z_rows, int64_t z_width, const int32_t* z_len,
                     const int32_t* y_cdf, int64_t y_rows, int64_t y_width, const int32_t* y_len) {
    auto r = std::make_unique<RefRans>();
    const int rc = guarded([&] {
        std::vector<int32_t> zc(z_cdf, z_cdf + z_rows * z_width), zl(z_len, z_len + z_rows);
        std::vector<int32_t> yc(y_cdf, y_cdf + y_rows * y_width), yl(y_len, y_len + y_rows);
        r->encoder.set_cdf(0, zc, zl);
        r->encoder.set_cdf(1, yc, yl);
        r->decoder.set_cdf(0, zc, zl);
        r->decoder.set_cdf(1, yc, yl);
    });
    return rc == 0 ? r.release() : nullptr;
}

void ufref_rans_free(void* h) { delete static_cast<RefRans*>(h); }

int ufref_rans_reset(void* h) { return guarded([&] { static_cast<RefRans*>(h)->encoder.reset(); }); }

int ufref_rans_encode_y(void* h, const int16_t* packed, int64_t n) {
    return guarded([&] { static_cast<RefRans*>(h)->encoder.encode_y(std::vector<int16_t>(packed, packed + n)); });
}

int ufref_rans_encode_z(void* h, const int8_t* symbols, int64_t n, int offset, int channels) {
    return guarded([&] {
        static_cast<RefRans*>(h)->encoder.encode_z(std::vector<int8_t>(symbols, symbols + n), offset, channels);
    });
}

int64_t ufref_rans_flush(void* h, uint8_t* out, int64_t capacity) {
    auto* r = static_cast<RefRans*>(h);
    int64_t n = -1;
    guarded([&] {
        r->out = r->encoder.flush();
        n = static_cast<int64_t>(r->out.size());
    });
    if (n >= 0 && out && capacity >= n && n) std::memcpy(out, r->out.data(), n);
    return n;
}

int ufref_rans_set_stream(void* h, const uint8_t* data, int64_t n) {
    return guarded([&] { static_cast<RefRans*>(h)->decoder.set_stream(std::vector<uint8_t>(data, data + n)); });
}

int ufref_rans_decode_z(void* h, int64_t count, int offset, int channels, int8_t* out) {
    return guarded([&] {
        const auto v = static_cast<RefRans*>(h)->decoder.decode_z(count, offset, channels);
        if (!v.empty()) std::memcpy(out, v.data(), v.size());
    });
}

int ufref_rans_decode_y(void* h, const uint8_t* indexes, int64_t n, int8_t* out) {
    return guarded([&] {
        const auto v = static_cast<RefRans*>(h)->decoder.decode_y(std::vector<uint8_t>(indexes, indexes + n));
        if (!v.empty()) std::memcpy(out, v.data(), v.size());
    });
}

}  // extern "C"

// ---- UF16 container (src/bitstream.cpp) over std::stringstream ----

namespace {

// Copies a writer's output to out; returns the byte count the writer reported.
template <class F>
int64_t ref_write(uint8_t* out, int64_t capacity, F&& fn) {
    int64_t n = -1;
    std::string bytes;
    const int rc = guarded([&] {
        std::ostringstream s(std::ios::binary);
        n = static_cast<int64_t>(fn(s));
        bytes = s.str();
        if (static_cast<int64_t>(bytes.size()) != n) throw std::runtime_error("writer count differs from bytes");
        if (n > capacity) throw std::length_error("output buffer too small");
    });
    if (rc) return -1;
    if (n) std::memcpy(out, bytes.data(), static_cast<size_t>(n));
    return n;
}

std::array<std::uint8_t, 32> id32(const uint8_t* p) {
    std::array<std::uint8_t, 32> a{};
    std::memcpy(a.data(), p, 32);
    return a;
}

}  // namespace

extern "C" {

int64_t ufref_bs_write_uint(uint32_t value, uint8_t* out, int64_t capacity) {
    return ref_write(out, capacity, [&](std::ostream& s) { return uf::write_uint_adaptive(s, value); });
}

int64_t ufref_bs_write_preamble(const uint8_t* image_id, const uint8_t* video_id, uint8_t* out, int64_t capacity) {
    return ref_write(out, capacity, [&](std::ostream& s) {
        uf::Preamble p;
        p.integer = true;
        p.image_identity = id32(image_id);
        p.video_identity = id32(video_id);
        const auto before = s.tellp();
        uf::write_preamble(s, p);
        return static_cast<size_t>(s.tellp() - before);
    });
}

int64_t ufref_bs_write_sps(int id, uint32_t width, uint32_t height, uint8_t* out, int64_t capacity) {
    return ref_write(out, capacity, [&](std::ostream& s) {
        return uf::write_sps(s, uf::Sps{static_cast<std::uint8_t>(id), width, height});
    });
}

int64_t ufref_bs_write_packet(int type, int sps_id, int qp, int entropy_parallel, int reset, const uint8_t* payload,
                              int64_t length, uint8_t* out, int64_t capacity) {
    return ref_write(out, capacity, [&](std::ostream& s) {
        uf::Packet p{static_cast<uf::NalType>(type), static_cast<std::uint8_t>(sps_id), static_cast<std::uint8_t>(qp),
                     static_cast<std::uint8_t>(entropy_parallel), reset != 0,
                     std::vector<std::uint8_t>(payload, payload + length)};
        return uf::write_packet(s, p);
    });
}

// scan_bitstream; summary[0..6] = integer, width, height, packets,
// intra_packets, predicted_packets, maximum_frames; identities to ids[64].
int ufref_bs_scan(const uint8_t* data, int64_t size, const char* variant, int64_t expected_frames, int64_t* summary,
                  uint8_t* ids) {
    return guarded([&] {
        std::istringstream s(std::string(reinterpret_cast<const char*>(data), static_cast<size_t>(size)),
                             std::ios::binary);
        std::optional<std::uint64_t> expected;
        if (expected_frames >= 0) expected = static_cast<std::uint64_t>(expected_frames);
        const auto r = uf::scan_bitstream(s, variant, expected);
        summary[0] = r.preamble.integer;
        summary[1] = r.dimensions.width;
        summary[2] = r.dimensions.height;
        summary[3] = static_cast<int64_t>(r.packets);
        summary[4] = static_cast<int64_t>(r.intra_packets);
        summary[5] = static_cast<int64_t>(r.predicted_packets);
        summary[6] = static_cast<int64_t>(r.maximum_frames);
        std::memcpy(ids, r.preamble.image_identity.data(), 32);
        std::memcpy(ids + 32, r.preamble.video_identity.data(), 32);
    });
}

// read_preamble then every NAL unit: per unit 7 values (type, sps_id, width,
// height, qp, entropy_parallel << 1 | reset, payload length) and the payloads
// concatenated; returns the unit count in *units.
int ufref_bs_parse(const uint8_t* data, int64_t size, int64_t* integer, int64_t* records, int64_t max_units,
                   int64_t* units, uint8_t* payloads, int64_t payload_capacity) {
    return guarded([&] {
        std::istringstream s(std::string(reinterpret_cast<const char*>(data), static_cast<size_t>(size)),
                             std::ios::binary);
        *integer = uf::read_preamble(s).integer;
        int64_t n = 0, used = 0;
        while (const auto h = uf::read_optional_header(s)) {
            if (n >= max_units) throw std::length_error("too many units");
            int64_t* r = records + 7 * n;
            r[0] = static_cast<int64_t>(h->type);
            r[1] = h->sps_id;
            r[2] = r[3] = r[4] = r[5] = r[6] = 0;
            if (h->type == uf::NalType::sps) {
                const auto sps = uf::read_sps(s, h->sps_id);
                r[2] = sps.width;
                r[3] = sps.height;
            } else {
                const auto p = uf::read_packet(s, h->type, h->sps_id);
                r[4] = p.qp;
                r[5] = p.entropy_parallel << 1 | p.reset_feature_memory;
                r[6] = static_cast<int64_t>(p.payload.size());
                if (used + r[6] > payload_capacity) throw std::length_error("payload buffer too small");
                if (!p.payload.empty()) std::memcpy(payloads + used, p.payload.data(), p.payload.size());
                used += r[6];
            }
            ++n;
        }
        *units = n;
    });
}

}  // extern "C"

// ---- uf::IntegerCodec (src/integer_codec.cpp): the reference's own stream
// encode / decode loops and raw_frame, over in-memory frames ----

namespace {

struct RefCodec {
    std::unique_ptr<uf::IntegerCodec> codec;
};

void fill_prepared(uf::PreparedModel& p, const char* variant, const char* identity_hex, int count,
                   const char* const* names, const int* dtypes, const int* ndims, const int64_t* shapes,
                   const void* const* data) {
    p.format = "dcvc-uf-prepared-v1";
    p.arithmetic = uf::int16::arithmetic_id;
    p.variant = variant;
    p.identity = identity_hex;
    const int64_t* cursor = shapes;
    for (int i = 0; i < count; ++i) {
        std::vector<int64_t> shape(cursor, cursor + ndims[i]);
        cursor += ndims[i];
        p.tensors[names[i]] = wrap(data[i], shape, dtype_of(dtypes[i]));
    }
}

}  // namespace

extern "C" {

// IntegerCodec(image, video, variant, kCPU, skip_threshold).  The constructor
// applies the reference's inference environment, which sets one intra-op
// thread (src/inference_environment.cpp:11-21); `threads` > 0 is requested
// afterwards, but the codec's loops were observed to keep running on one core,
// as the reference runs them by design.  video_count < 0: no video model.
void* ufref_codec_new(const char* variant, double skip_threshold, int threads,
                      const char* image_identity, int image_count, const char* const* image_names,
                      const int* image_dtypes, const int* image_ndims, const int64_t* image_shapes,
                      const void* const* image_data,
                      const char* video_identity, int video_count, const char* const* video_names,
                      const int* video_dtypes, const int* video_ndims, const int64_t* video_shapes,
                      const void* const* video_data) {
    auto handle = std::make_unique<RefCodec>();
    const int rc = guarded([&] {
        uf::PreparedModel image, video;
        fill_prepared(image, "image", image_identity, image_count, image_names, image_dtypes, image_ndims,
                      image_shapes, image_data);
        if (video_count >= 0)
            fill_prepared(video, variant, video_identity, video_count, video_names, video_dtypes, video_ndims,
                          video_shapes, video_data);
        handle->codec = std::make_unique<uf::IntegerCodec>(image, video_count >= 0 ? &video : nullptr, variant,
                                                           torch::kCPU, skip_threshold);
        if (threads > 0) torch::set_num_threads(threads);
    });
    return rc == 0 ? handle.release() : nullptr;
}

void ufref_codec_free(void* h) { delete static_cast<RefCodec*>(h); }

// IntegerCodec::encode over `frames` ([count, 3, height, width] uint8 YUV444,
// the FrameSource contract of include/uf/integer_codec.hpp:25-27), written to
// `output` (a path that must not exist yet).  stats[0..1] = frames, packets.
int ufref_codec_encode(void* h, const uint8_t* frames, int64_t count, uint32_t width, uint32_t height, int qp_i,
                       int qp_p, int reset_interval, int intra_period, const char* output, int64_t* stats) {
    return guarded([&] {
        const size_t frame_bytes = static_cast<size_t>(width) * height * 3;
        int64_t next = 0;
        uf::FrameSource source = [&]() -> std::optional<std::vector<std::uint8_t>> {
            if (next >= count) return std::nullopt;
            const uint8_t* f = frames + static_cast<size_t>(next++) * frame_bytes;
            return std::vector<std::uint8_t>(f, f + frame_bytes);
        };
        const auto s = static_cast<RefCodec*>(h)->codec->encode(source, output, width, height, qp_i, qp_p,
                                                                reset_interval, intra_period);
        stats[0] = static_cast<int64_t>(s.frames);
        stats[1] = static_cast<int64_t>(s.packets);
    });
}

// IntegerCodec::decode_stream over an in-memory archive.  digest_hex receives
// the decoded-YUV SHA-256 (65 bytes incl. NUL); when yuv_out is non-null each
// raw YUV420 frame the FrameSink receives is appended there (capacity bytes).
int ufref_codec_decode(void* h, const uint8_t* data, int64_t size, int64_t total_frames, int64_t total_packets,
                       char* digest_hex, uint8_t* yuv_out, int64_t capacity, int64_t* stats) {
    return guarded([&] {
        std::istringstream s(std::string(reinterpret_cast<const char*>(data), static_cast<size_t>(size)),
                             std::ios::binary);
        int64_t used = 0;
        uf::FrameSink sink;
        if (yuv_out) {
            sink = [&](const std::vector<std::uint8_t>& raw) {
                if (used + static_cast<int64_t>(raw.size()) > capacity) throw std::length_error("yuv buffer too small");
                std::memcpy(yuv_out + used, raw.data(), raw.size());
                used += static_cast<int64_t>(raw.size());
            };
        }
        const auto r = static_cast<RefCodec*>(h)->codec->decode_stream(s, static_cast<std::uint64_t>(total_frames),
                                                                        static_cast<std::uint64_t>(total_packets),
                                                                        sink);
        if (r.decoded_yuv_sha256.size() != 64) throw std::runtime_error("unexpected digest length");
        std::memcpy(digest_hex, r.decoded_yuv_sha256.c_str(), 65);
        stats[0] = static_cast<int64_t>(r.frames);
        stats[1] = static_cast<int64_t>(r.packets);
        stats[2] = used;
    });
}

// IntegerCodec::raw_frame (src/integer_codec.cpp:294-323): an int16 frame
// tensor [1, 3, fh, fw] -> YUV420 bytes of width x height (Y then U then V).
int64_t ufref_raw_frame(const int16_t* frame, const int64_t* fs, int64_t width, int64_t height, uint8_t* out,
                        int64_t capacity) {
    int64_t n = -1;
    std::vector<std::uint8_t> raw;
    const int rc = guarded([&] {
        raw = uf::IntegerCodec::raw_frame(wrap(frame, {fs[0], fs[1], fs[2], fs[3]}, torch::kInt16), width, height);
        if (static_cast<int64_t>(raw.size()) > capacity) throw std::length_error("output buffer too small");
        n = static_cast<int64_t>(raw.size());
    });
    if (rc) return -1;
    if (n) std::memcpy(out, raw.data(), static_cast<size_t>(n));
    return n;
}

}  // extern "C"
