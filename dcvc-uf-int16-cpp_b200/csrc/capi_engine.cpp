// Engine-level C ABI (include/uf_b200.h): prepared-model upload, module runs
// (uf::Layers::run) and per-stream codec state (uf::IntegerModel).
#include "uf_b200.h"

#include "capi_engine.h"
#include "capi_util.h"
#include "engine.h"
#include "engine_kernels.h"
#include "kernels.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <stdexcept>

using namespace ufb;

extern "C" {

ufb_model* ufb_model_create(int device, const char* variant, int count, const char* const* names, const int* dtypes,
                            const int* ndims, const int64_t* shapes, const void* const* data) {
    ufb_model* out = nullptr;
    guarded([&] {
        if (!variant || count <= 0 || !names || !dtypes || !ndims || !shapes || !data)
            throw std::invalid_argument("invalid prepared-model table");
        std::vector<HostTensor> tensors;
        const int64_t* cursor = shapes;
        for (int i = 0; i < count; ++i) {
            HostTensor t;
            t.name = names[i];
            t.dtype = dtypes[i];
            t.shape.assign(cursor, cursor + ndims[i]);
            cursor += ndims[i];
            t.data = data[i];
            tensors.push_back(std::move(t));
        }
        auto h = std::make_unique<ufb_model>(device);
        h->m = std::make_unique<Model>(device, variant, tensors);
        ck(cudaStreamCreateWithFlags(&h->s, cudaStreamNonBlocking), "stream");
        ck(cudaMalloc(&h->status, sizeof(int)), "status");
        ck(cudaMemset(h->status, 0, sizeof(int)), "status");
        out = h.release();
        return 0;
    });
    return out;
}

void ufb_model_destroy(ufb_model* m) {
    if (!m) return;
    if (m->s) {
        cudaStreamSynchronize(m->s);
        cudaStreamDestroy(m->s);
    }
    if (m->status) cudaFree(m->status);
    delete m;
}

int ufb_model_run(ufb_model* m, const char* module, int nargs, const int16_t* const* args, const int64_t* shapes,
                  const char* q_name, int qp, int16_t* out, int64_t capacity, int64_t* out_shape) {
    return guarded([&] {
        if (!m || !module || nargs <= 0 || !args || !shapes || !out || !out_shape)
            throw std::invalid_argument("invalid module call");
        const std::string mod = module;
        const Model& model = *m->m;
        DeviceGuard device(model.device());
        Runner r(model, m->pool, m->s, m->status);
        const bool image = model.variant() == "image";
        const bool unshuffle8 = (mod == "enc" && image) || mod == "encoder";
        std::vector<Tensor> xs;
        std::vector<std::pair<void*, size_t>> scratch;
        for (int i = 0; i < nargs; ++i) {
            const int64_t* s = shapes + 4 * i;
            const int f = (i == 0 && unshuffle8) ? 8 : 1;
            const size_t bytes = static_cast<size_t>(s[0] * s[1] * s[2] * s[3]) * 2;
            void* d = m->pool.get(bytes);
            scratch.push_back({d, bytes});
            ck(cudaMemcpyAsync(d, args[i], bytes, cudaMemcpyHostToDevice, m->s), "argument upload");
            Tensor t = r.alloc(static_cast<int>(s[0]), static_cast<int>(s[2] / f), static_cast<int>(s[3] / f),
                               static_cast<int>(s[1] * f * f));
            ck(nchw_to_split(static_cast<int16_t*>(d), static_cast<int>(s[0]), static_cast<int>(s[1]),
                             static_cast<int>(s[2]), static_cast<int>(s[3]), f, t.a, m->s),
               "argument layout");
            xs.push_back(t);
        }
        const int16_t* q = nullptr;
        if (q_name && *q_name) {
            const ParamTable* p = model.param(q_name);
            if (!p) throw std::runtime_error(std::string("Missing prepared UF tensor: ") + q_name);
            if (qp < 0 || qp >= p->rows) throw std::invalid_argument("qp out of range");
            q = p->data + static_cast<size_t>(qp) * p->cols;
        }
        const Tensor y = r.run(mod, xs, q);
        const int f = (mod == "dec" && image) ? 8 : 1;
        const int64_t n = static_cast<int64_t>(y.a.n) * y.a.c * y.a.h * y.a.w;
        if (n > capacity) throw std::length_error("output buffer too small");
        void* d = m->pool.get(n * 2);
        ck(split_to_nchw(y.a, f, static_cast<int16_t*>(d), m->s), "output layout");
        ck(cudaMemcpyAsync(out, d, n * 2, cudaMemcpyDeviceToHost, m->s), "output download");
        ck(cudaStreamSynchronize(m->s), "module run");
        int st = 0;
        ck(cudaMemcpy(&st, m->status, sizeof(int), cudaMemcpyDeviceToHost), "status");
        if (st) {
            cudaMemset(m->status, 0, sizeof(int));
            throw std::runtime_error("kernel pipeline timeout");
        }
        m->pool.put(d, n * 2);
        for (auto& p : scratch) m->pool.put(p.first, p.second);
        out_shape[0] = y.a.n;
        out_shape[1] = y.a.c / (f * f);
        out_shape[2] = static_cast<int64_t>(y.a.h) * f;
        out_shape[3] = static_cast<int64_t>(y.a.w) * f;
        return 0;
    });
}

ufb_codec* ufb_codec_create(ufb_model* model, int batch) {
    ufb_codec* out = nullptr;
    guarded([&] {
        if (!model) throw std::invalid_argument("model is null");
        auto c = std::make_unique<ufb_codec>();
        c->c = std::make_unique<Codec>(*model->m, batch);
        out = c.release();
        return 0;
    });
    return out;
}

void ufb_codec_destroy(ufb_codec* c) { delete c; }

int ufb_codec_set_skip_threshold(ufb_codec* c, double threshold) {
    return guarded([&] {
        if (!c) throw std::invalid_argument("codec is null");
        c->c->set_skip_threshold(threshold);
        return 0;
    });
}

int ufb_codec_clear_dpb(ufb_codec* c) {
    return guarded([&] {
        if (!c) throw std::invalid_argument("codec is null");
        c->c->clear_dpb();
        return 0;
    });
}

int ufb_codec_add_ref_frames(ufb_codec* c, const int16_t* frames, int height, int width) {
    return guarded([&] {
        if (!c || !frames || height <= 0 || width <= 0) throw std::invalid_argument("invalid reference frames");
        c->c->add_ref_frames(frames, height, width);
        return 0;
    });
}

int ufb_codec_decompress(ufb_codec* c, const uint8_t* const* payloads, const size_t* lengths, uint32_t width,
                         uint32_t height, int qp, int entropy_parallel, int reset, int16_t* frames_out,
                         uint8_t* yuv_out) {
    return guarded([&] {
        if (!c || !payloads || !lengths) throw std::invalid_argument("invalid payloads");
        if (entropy_parallel != 1) throw std::invalid_argument("Unsupported UF integer packet parameters");
        for (int b = 0; b < c->c->batch(); ++b)
            if (!payloads[b]) throw std::invalid_argument("payload is null");
        return c->c->decompress(payloads, lengths, width, height, qp, reset != 0, frames_out, yuv_out);
    });
}

int ufb_codec_compress(ufb_codec* c, const uint8_t* frames, int channels, int height, int width, int qp, int reset,
                       uint8_t* payload_out, size_t capacity, size_t* lengths, int16_t* frames_out) {
    return guarded([&] {
        if (!c || !frames || !payload_out || !lengths || channels <= 0 || channels % 3 || height <= 0 || width <= 0)
            throw std::invalid_argument("invalid frames");
        std::vector<std::vector<uint8_t>> payloads;
        const int n = c->c->compress(frames, channels, height, width, qp, reset != 0, payloads, frames_out);
        for (int b = 0; b < c->c->batch(); ++b) {
            if (payloads[b].size() > capacity) throw std::length_error("payload buffer too small");
            std::memcpy(payload_out + static_cast<size_t>(b) * capacity, payloads[b].data(), payloads[b].size());
            lengths[b] = payloads[b].size();
        }
        return n;
    });
}

int ufb_codec_state(ufb_codec* c, int which, int16_t* out, int64_t capacity, int64_t* shape4) {
    return guarded([&] {
        if (!c || !out || !shape4 || which < 0 || which > 2) throw std::invalid_argument("invalid state request");
        return c->c->state(which, out, static_cast<size_t>(capacity), shape4) ? 0 : 1;
    });
}

double ufb_codec_host_seconds(ufb_codec* c) { return c ? c->c->last_host_seconds() : 0.0; }

int ufb_codec_set_reference_from(ufb_codec* video, ufb_codec* image) {
    return guarded([&] {
        if (!video || !image) throw std::invalid_argument("codec is null");
        video->c->set_reference_from(*image->c);
        return 0;
    });
}

int ufb_codec_set_stream(ufb_codec* c, void* stream) {
    return guarded([&] {
        if (!c) throw std::invalid_argument("codec is null");
        c->c->set_stream(static_cast<cudaStream_t>(stream));
        return 0;
    });
}

int ufb_codec_profile(ufb_codec* c, int enable) {
    return guarded([&] {
        if (!c) throw std::invalid_argument("codec is null");
        c->c->stats().profile = enable != 0;
        return 0;
    });
}

int ufb_codec_stats(ufb_codec* c, int reset, int64_t* launches, int64_t* conv_launches, double* conv_int16_macs,
                    double* conv_ms) {
    return guarded([&] {
        if (!c) throw std::invalid_argument("codec is null");
        EngineStats& st = c->c->stats();
        if (launches) *launches = st.launches;
        if (conv_launches) *conv_launches = st.conv_launches;
        if (conv_int16_macs) *conv_int16_macs = st.conv_int16_macs;
        if (conv_ms) *conv_ms = st.conv_ms;
        if (reset) st.reset();
        return 0;
    });
}

int ufb_codec_shape_table(ufb_codec* c, char* text, int64_t capacity, int64_t* length) {
    return guarded([&] {
        if (!c || !length) throw std::invalid_argument("codec or length is null");
        EngineStats& st = c->c->stats();
        std::string out;
        char line[256];
        for (const auto& kv : st.shapes) {
            snprintf(line, sizeof(line), "%s\t%lld\t%.9g\t%.6f\t%.9g\n", kv.first.c_str(), kv.second.launches,
                     kv.second.int16_macs, kv.second.ms, kv.second.hbm_bytes);
            out += line;
        }
        *length = static_cast<int64_t>(out.size());
        if (text && capacity > 0) {
            const size_t n = std::min<size_t>(out.size(), static_cast<size_t>(capacity - 1));
            memcpy(text, out.data(), n);
            text[n] = 0;
        }
        return 0;
    });
}

}  // extern "C"
