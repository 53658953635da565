#include "engine.h"
#include "interrupt.h"

#include <cstdio>

#include "engine_kernels.h"
#include "kernels.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace ufb {

namespace {

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(e));
}

bool begins(const std::string& v, const std::string& p) { return v.rfind(p, 0) == 0; }

bool ends(const std::string& v, const std::string& s) {
    return v.size() >= s.size() && v.compare(v.size() - s.size(), s.size(), s) == 0;
}

int pitch_for(int c) { return (c + 15) / 16 * 16; }

}  // namespace

// ------------------------------------------------------------------ pool ----

DevicePool::~DevicePool() {
    int current = 0;
    cudaGetDevice(&current);
    cudaSetDevice(device_);
    for (void* p : all_) cudaFree(p);
    cudaSetDevice(current);
}

void* DevicePool::get(size_t bytes) {
    bytes = (bytes + 255) / 256 * 256;
    auto it = free_.find(bytes);
    if (it != free_.end() && !it->second.empty()) {
        void* p = it->second.back();
        it->second.pop_back();
        return p;
    }
    void* p = nullptr;
    ck(cudaMalloc(&p, bytes), "device pool allocation");
    all_.push_back(p);
    reserved_ += bytes;
    return p;
}

void DevicePool::put(void* p, size_t bytes) {
    bytes = (bytes + 255) / 256 * 256;
    free_[bytes].push_back(p);
}

Tensor Tensor::channels(int c0, int c) const {
    if (c0 < 0 || c0 + c > a.c || (c0 % 16)) throw std::invalid_argument("invalid channel view");
    Tensor t = *this;
    t.a.base = a.base + c0;
    t.a.c = c;
    return t;
}

Tensor Tensor::crop(int h, int w) const {
    if (h > a.h || w > a.w) throw std::invalid_argument("invalid crop");
    Tensor t = *this;
    t.a.h = h;
    t.a.w = w;
    return t;
}

Pinned::~Pinned() {
    if (p_) cudaFreeHost(p_);
}

void* Pinned::get(size_t bytes) {
    if (bytes > n_) {
        if (p_) cudaFreeHost(p_);
        p_ = nullptr;
        n_ = 0;
        ck(cudaMallocHost(&p_, bytes), "pinned allocation");
        n_ = bytes;
    }
    return p_;
}

EngineStats::~EngineStats() {
    for (auto& e : pending) {
        cudaEventDestroy(e.start);
        cudaEventDestroy(e.stop);
    }
    for (auto e : spare) cudaEventDestroy(e);
}

cudaEvent_t EngineStats::take_event() {
    cudaEvent_t ev = nullptr;
    if (!spare.empty()) {
        ev = spare.back();
        spare.pop_back();
    } else {
        ck(cudaEventCreate(&ev), "event");
    }
    return ev;
}

void EngineStats::collect() {
    for (auto& e : pending) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, e.start, e.stop) == cudaSuccess) {
            if (e.tensor_core) conv_ms += ms;
            shapes[e.shape].ms += ms;
        }
        spare.push_back(e.start);
        spare.push_back(e.stop);
    }
    pending.clear();
}

void EngineStats::reset() {
    launches = conv_launches = 0;
    conv_int16_macs = conv_ms = 0;
    shapes.clear();
}

// ----------------------------------------------------------------- model ----

Model::Model(int device, const std::string& variant, const std::vector<HostTensor>& tensors)
    : device_(device), variant_(variant) {
    if (variant != "image" && variant != "hts" && variant != "htl" && variant != "ld")
        throw std::invalid_argument("Unsupported UF integer model variant");
    ck(cudaSetDevice(device), "cudaSetDevice");
    auto upload = [&](const void* host, size_t bytes) -> void* {
        void* d = nullptr;
        ck(cudaMalloc(&d, bytes), "model upload allocation");
        allocations_.push_back(d);
        ck(cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice), "model upload");
        return d;
    };
    const HostTensor *zc = nullptr, *zl = nullptr, *yc = nullptr, *yl = nullptr;
    std::map<std::string, bool> signed_ok;  // every weight <= 32639: signed byte split allowed
    std::map<std::string, bool> narrow_ok;  // narrow tensor-core recombination allowed (tc_narrow_ok)
    std::map<std::string, const int16_t*> host_w, host_b;  // host data of each layer's weight and bias
    for (const auto& t : tensors) {
        names_.insert(t.name);
        size_t numel = 1;
        for (auto d : t.shape) numel *= static_cast<size_t>(d);
        if (ends(t.name, ".weight")) {
            if (t.dtype != 0 || t.shape.size() != 4) throw std::invalid_argument("weight must be int16 4-D: " + t.name);
            ConvLayer& L = convs_[t.name.substr(0, t.name.size() - 7)];
            L.co = static_cast<int>(t.shape[0]);
            L.ci = static_cast<int>(t.shape[1]);
            L.kh = static_cast<int>(t.shape[2]);
            L.kw = static_cast<int>(t.shape[3]);
            L.weights16 = static_cast<int16_t*>(upload(t.data, numel * 2));
            host_w[t.name.substr(0, t.name.size() - 7)] = static_cast<const int16_t*>(t.data);
            const bool sgn = tc_signed_split_ok(static_cast<const int16_t*>(t.data), numel);
            signed_ok[t.name.substr(0, t.name.size() - 7)] = sgn;
            narrow_ok[t.name.substr(0, t.name.size() - 7)] =
                tc_narrow_ok(static_cast<const int16_t*>(t.data), L.co, L.ci, L.kh, L.kw, sgn);
        } else if (ends(t.name, ".bias")) {
            if (t.dtype != 0 || t.shape.size() != 1) throw std::invalid_argument("bias must be int16 1-D: " + t.name);
            convs_[t.name.substr(0, t.name.size() - 5)].bias = static_cast<int16_t*>(upload(t.data, numel * 2));
            host_b[t.name.substr(0, t.name.size() - 5)] = static_cast<const int16_t*>(t.data);
        } else if (begins(t.name, "q_")) {
            if (t.dtype != 0 || t.shape.size() != 2) throw std::invalid_argument("QP table must be int16 2-D: " + t.name);
            ParamTable& p = params_[t.name];
            p.rows = static_cast<int>(t.shape[0]);
            p.cols = static_cast<int>(t.shape[1]);
            p.data = static_cast<int16_t*>(upload(t.data, numel * 2));
        } else if (t.name == "tables.wsilu") {
            if (t.dtype != 0 || numel != 65536) throw std::invalid_argument("invalid WSiLU table");
            wsilu_ = static_cast<int16_t*>(upload(t.data, numel * 2));
            tc_lut_window(static_cast<const int16_t*>(t.data), wsilu_start_, wsilu_n_, wsilu_hi_);
        } else if (t.name == "tables.scale_index") {
            if (t.dtype != 1 || numel != 65536) throw std::invalid_argument("invalid scale-index table");
            scale_index_ = static_cast<uint8_t*>(upload(t.data, numel));
        } else if (t.name == "tables.z_cdf") {
            zc = &t;
        } else if (t.name == "tables.z_lengths") {
            zl = &t;
        } else if (t.name == "tables.y_cdf") {
            yc = &t;
        } else if (t.name == "tables.y_lengths") {
            yl = &t;
        }
    }
    if (!zc || !zl || !yc || !yl) throw std::runtime_error("Missing prepared UF tensor: tables CDF");
    auto set_table = [](RansTables& tab, const HostTensor* cdf, const HostTensor* len) {
        if (cdf->dtype != 2 || len->dtype != 2 || cdf->shape.size() != 2 || len->shape.size() != 1 ||
            cdf->shape[0] != len->shape[0])
            throw std::runtime_error("Prepared UF CDF is not INT32");
        tab.set(static_cast<const int32_t*>(cdf->data), static_cast<int>(cdf->shape[0]),
                static_cast<int>(cdf->shape[1]), static_cast<const int32_t*>(len->data));
    };
    set_table(z_table_, zc, zl);
    set_table(y_table_, yc, yl);
    // tensor-core weight planes for every layer that can use them
    for (auto& kv : convs_) {
        ConvLayer& L = kv.second;
        if (!L.weights16) throw std::runtime_error("Missing prepared UF tensor: " + kv.first + ".weight");
        L.depthwise = L.ci == 1 && L.co > 1;
        if (L.depthwise && L.kh == 3 && L.kw == 3) {
            auto b = host_b.find(kv.first);
            L.dw_narrow = dw_narrow_ok(host_w[kv.first], b == host_b.end() ? nullptr : b->second, L.co);
        }
        if (L.depthwise || static_cast<long long>(L.ci) * L.kh * L.kw > kTcMaxReduction) continue;
        const bool sgn = signed_ok[kv.first];
        const int bn = tc_choose_bn(L.ci, L.kh, L.kw, sgn);
        void* planes = nullptr;
        ck(cudaMalloc(&planes, tc_weight_bytes(L.co, L.ci, L.kh, L.kw, bn)), "weight planes");
        allocations_.push_back(planes);
        std::string err;
        if (!tc_prepare(L.tc, L.weights16, L.co, L.ci, L.kh, L.kw, sgn, bn, static_cast<uint8_t*>(planes), nullptr,
                        err))
            throw std::runtime_error(err);
        L.tc.narrow = narrow_ok[kv.first];
    }
    ck(cudaDeviceSynchronize(), "model upload");
}

Model::~Model() {
    int current = 0;
    cudaGetDevice(&current);
    cudaSetDevice(device_);
    for (void* p : allocations_) cudaFree(p);
    cudaSetDevice(current);
}

const ConvLayer* Model::conv(const std::string& name) const {
    auto it = convs_.find(name);
    return it == convs_.end() ? nullptr : &it->second;
}

const ParamTable* Model::param(const std::string& name) const {
    auto it = params_.find(name);
    return it == params_.end() ? nullptr : &it->second;
}

bool Model::has_child(const std::string& prefix) const {
    const std::string p = prefix + ".";
    auto it = names_.lower_bound(p);
    return it != names_.end() && begins(*it, p);
}

// ---------------------------------------------------------------- runner ----

Tensor Runner::alloc(int n, int h, int w, int c) {
    const int pitch = pitch_for(c);
    const size_t bytes = static_cast<size_t>(n) * h * w * 2 * pitch;
    Tensor t;
    void* p = pool_.get(bytes);
    t.mem = std::shared_ptr<Block>(new Block{&pool_, p, bytes});
    t.a = make_act(static_cast<uint8_t*>(p), n, h, w, c, pitch);
    return t;
}

bool Runner::residual_shortcut() const {
    // Only ResidualBlockUpsample/WithStride2 set DepthConvBlock.shortcut for
    // the image and HT-L variants (src/layers.cpp:84-89).
    return m_.variant() == "image" || m_.variant() == "htl";
}

// Layers::run_conv (src/layers.cpp:74-82): padding 1 for 3x3 kernels, stride
// 2 for encoder.down / enc.enc_2.6, depthwise when the weight has one input
// channel per group and as many outputs as the input has channels.
Tensor Runner::conv(const std::string& name, const Tensor& in, const Fuse& f, const Tensor* out_view) {
    const ConvLayer* L = m_.conv(name);
    if (!L) throw std::runtime_error("Missing prepared UF tensor: " + name + ".weight");
    const int pad = L->kh == 3 ? 1 : 0;
    const int stride = name == "encoder.down" || name == "enc.enc_2.6" ? 2 : 1;
    const bool grouped = L->ci == 1 && L->co == in.a.c;
    const int oh = (in.a.h + 2 * pad - L->kh) / stride + 1, ow = (in.a.w + 2 * pad - L->kw) / stride + 1;
    if (!grouped && L->ci != in.a.c) throw std::invalid_argument("channel mismatch in " + name);
    int out_c = f.wsilu4 ? L->co / 4 : (f.shuffle2 ? L->co / 4 : L->co);
    int out_h = f.shuffle2 ? 2 * oh : oh, out_w = f.shuffle2 ? 2 * ow : ow;
    Tensor out = out_view ? *out_view : alloc(in.a.n, out_h, out_w, out_c);
    if (out.a.c != out_c || out.a.h != out_h || out.a.w != out_w || out.a.n != in.a.n)
        throw std::invalid_argument("output view does not match " + name);
    if (grouped) {
        if (L->kh != 3 || L->kw != 3 || stride != 1 || f.lut || f.wsilu4 || f.shuffle2 || f.res1 || f.mulq)
            throw std::invalid_argument("unsupported depthwise configuration in " + name);
        cudaEvent_t ev0 = nullptr;
        if (stats_ && stats_->profile) {
            ev0 = stats_->take_event();
            ck(cudaEventRecord(ev0, s_), "event");
        }
        ck(dwconv3x3(in.a, out.a, L->weights16, L->bias, status_, s_, L->dw_narrow), "depthwise conv");
        if (ev0) {
            cudaEvent_t ev1 = stats_->take_event();
            ck(cudaEventRecord(ev1, s_), "event");
            char key[96];
            const long long px = static_cast<long long>(in.a.n) * oh * ow;
            snprintf(key, sizeof(key), "depthwise %d 3x3 @ %lld", L->co, px);
            stats_->pending.push_back({ev0, ev1, key, false});
            auto& sh = stats_->shapes[key];
            ++sh.launches;
            sh.int16_macs += static_cast<double>(px) * L->co * 9;
            sh.hbm_bytes += 2.0 * (static_cast<double>(in.a.pixels()) * in.a.c + static_cast<double>(px) * L->co +
                                   9.0 * L->co);
        }
        count();
        return out;
    }
    if ((f.lut || f.wsilu4) && (!L->tc.planes || !tc_table_window_fits(L->tc, m_.wsilu_n()))) {
        // a table without a shared-memory window (not WSiLU-shaped): the plain
        // convolution, then the table step as its own pass
        Fuse plain;
        const Tensor t = conv(name, in, plain);
        ck(lut_split(t.a, m_.wsilu(), f.wsilu4 ? 4 : 1, out.a, s_), "table step");
        count();
        return out;
    }
    if (L->tc.planes && (stride == 1 || !(f.lut || f.wsilu4 || f.shuffle2 || f.res1 || f.mulq))) {
        Epilogue e{};
        e.bias = L->bias;
        e.bias32 = 0;
        e.lut = (f.lut || f.wsilu4) ? m_.wsilu() : nullptr;
        e.lut_start = m_.wsilu_start();
        e.lut_n = m_.wsilu_n();
        e.lut_hi = m_.wsilu_hi();
        e.wsilu4 = f.wsilu4;
        e.shuffle2 = f.shuffle2;
        if (f.res1) e.res1 = f.res1->a;
        if (f.res2) e.res2 = f.res2->a;
        e.mulq = f.mulq;
        std::string err;
        const double macs = static_cast<double>(in.a.n) * oh * ow * L->co * L->ci * L->kh * L->kw;
        cudaEvent_t ev0 = nullptr;
        if (stats_ && stats_->profile) {
            ev0 = stats_->take_event();
            ck(cudaEventRecord(ev0, s_), "event");
        }
        if (conv_tc_run(L->tc, in.a, out.a, e, pad, pad, s_, status_, err, stride) != 0)
            throw std::runtime_error(name + ": " + err);
        if (ev0) {
            cudaEvent_t ev1 = stats_->take_event();
            ck(cudaEventRecord(ev1, s_), "event");
            char key[128];
            const char* epi = f.wsilu4 ? " +wsilu4" : f.lut ? " +lut" : f.shuffle2 ? " +shuffle2" : "";
            snprintf(key, sizeof(key), "conv %d>%d %dx%d%s%s%s%s%s @ %lld", L->ci, L->co, L->kh, L->kw,
                     stride == 2 ? "/2" : "", epi, f.res1 ? " +res" : "", f.res2 ? " +res" : "",
                     f.mulq ? " +mulq" : "", static_cast<long long>(in.a.n) * oh * ow);
            stats_->pending.push_back({ev0, ev1, key, true});
            auto& sh = stats_->shapes[key];
            ++sh.launches;
            sh.int16_macs += macs;
            const double out_values = static_cast<double>(out.a.pixels()) * out.a.c;
            sh.hbm_bytes += 2.0 * (static_cast<double>(in.a.pixels()) * in.a.c + out_values *
                                   (1 + (f.res1 ? 1 : 0) + (f.res2 ? 1 : 0)) +
                                   static_cast<double>(L->co) * L->ci * L->kh * L->kw);
        }
        if (stats_) {
            ++stats_->launches;
            ++stats_->conv_launches;
            stats_->conv_int16_macs += macs;
        }
        return out;
    }
    // Strided convolution whose reduction exceeds the tensor-core bound: direct
    // int64 kernel on NCHW copies (encode only; the HT-L and image strided
    // layers, encoder.down and enc.enc_2.6, run on the tensor cores above).
    if (f.lut || f.wsilu4 || f.shuffle2 || f.res1 || f.mulq) throw std::invalid_argument("unsupported fusion for " + name);
    const size_t in_el = static_cast<size_t>(in.a.n) * in.a.c * in.a.h * in.a.w;
    const size_t out_el = static_cast<size_t>(in.a.n) * L->co * oh * ow;
    void* xin = pool_.get(in_el * 2);
    void* xout = pool_.get(out_el * 2);
    ck(split_to_nchw(in.a, 1, static_cast<int16_t*>(xin), s_), "strided conv layout");
    ck(conv_direct(static_cast<int16_t*>(xout), static_cast<int16_t*>(xin), L->weights16, L->bias, 0, in.a.n, in.a.c,
                   L->co, in.a.h, in.a.w, oh, ow, L->kh, L->kw, stride, stride, pad, pad, 1, s_),
       "strided conv");
    ck(nchw_to_split(static_cast<int16_t*>(xout), in.a.n, L->co, oh, ow, 1, out.a, s_), "strided conv layout");
    count(3);
    pool_.put(xin, in_el * 2);
    pool_.put(xout, out_el * 2);
    return out;
}

// Layers::run_depth (src/layers.cpp:91-104) with each elementwise step fused
// into the epilogue of the convolution that produces its input:
//   dc.0 -> lookup(wsilu), dc.3 -> add(x), ffn.0 -> wsilu4, ffn.2 -> add(out)[, add(x)].
Tensor Runner::depth(const std::string& name, const Tensor& in, bool shortcut, const Tensor* out_view) {
    const Tensor x = m_.has(name + ".adaptor.weight") ? conv(name + ".adaptor", in) : in;
    Fuse f0;
    f0.lut = true;
    const Tensor t1 = conv(name + ".dc.0", x, f0);
    const Tensor t2 = conv(name + ".dc.2", t1);
    Fuse f3;
    f3.res1 = &x;
    const Tensor o1 = conv(name + ".dc.3", t2, f3);
    Fuse f4;
    f4.wsilu4 = true;
    const Tensor t3 = conv(name + ".ffn.0", o1, f4);
    Fuse f5;
    f5.res1 = &o1;
    f5.res2 = shortcut ? &x : nullptr;
    return conv(name + ".ffn.2", t3, f5, out_view);
}

// Layers::run_simple (src/layers.cpp:106-130).
Tensor Runner::simple(const std::string& name, const Tensor& in, bool shortcut) {
    if (m_.has(name + ".weight")) return conv(name, in);
    if (m_.has(name + ".dc.0.weight")) return depth(name, in, shortcut);
    if (m_.has(name + ".up.conv.0.weight") && m_.has(name + ".conv.dc.0.weight")) {
        Fuse f;
        f.shuffle2 = true;
        const Tensor up = conv(name + ".up.conv.0", in, f);
        return depth(name + ".conv", up, residual_shortcut());
    }
    if (m_.has(name + ".down.weight") && m_.has(name + ".conv.dc.0.weight")) {
        const Tensor down = conv(name + ".down", unshuffle2(in, nullptr));
        return depth(name + ".conv", down, residual_shortcut());
    }
    if (m_.has(name + ".conv.0.weight") && !m_.has(name + ".conv.1.weight")) {
        Fuse f;
        f.shuffle2 = true;
        return conv(name + ".conv.0", in, f);
    }
    if (m_.has_child(name + ".0")) {
        Tensor v = in;
        for (int i = 0; m_.has_child(name + "." + std::to_string(i)); ++i) v = simple(name + "." + std::to_string(i), v);
        return v;
    }
    throw std::runtime_error("Unsupported UF module path: " + name);
}

Tensor Runner::cat(const std::vector<Tensor>& parts) {
    int c = 0;
    for (const auto& p : parts) c += p.a.c;
    const Tensor& x = parts.at(0);
    Tensor out = alloc(x.a.n, x.a.h, x.a.w, c);
    int off = 0;
    for (const auto& p : parts) {
        if (p.a.n != x.a.n || p.a.h != x.a.h || p.a.w != x.a.w) throw std::invalid_argument("cat shape mismatch");
        if (off % 16) throw std::invalid_argument("cat needs channel counts that are multiples of 16");
        ck(copy_channels(p.a, out.channels(off, p.a.c).a, s_), "cat");
        count();
        off += p.a.c;
    }
    return out;
}

Tensor Runner::multiply(const Tensor& x, const int16_t* q) {
    Tensor out = alloc(x.a.n, x.a.h, x.a.w, x.a.c);
    ck(mul_channels(x.a, q, out.a, s_), "multiply");
    count();
    return out;
}

Tensor Runner::unshuffle2(const Tensor& x, const int16_t* q) {
    if (x.a.h % 2 || x.a.w % 2) throw std::invalid_argument("pixel_unshuffle(2) needs even extents");
    Tensor out = alloc(x.a.n, x.a.h / 2, x.a.w / 2, x.a.c * 4);
    ck(mul_unshuffle2(x.a, q, out.a, s_), "pixel_unshuffle");
    count();
    return out;
}

// Layers::run (src/layers.cpp:132-184).  Inputs of "enc" / "encoder" are the
// already pixel-unshuffled frames (the unshuffle is fused into their upload).
Tensor Runner::run(const std::string& module, const std::vector<Tensor>& args, const int16_t* q) {
    if (args.empty()) throw std::invalid_argument("UF integer layer requires an INT16 input");
    const Tensor& x = args[0];
    const bool image = m_.variant() == "image";
    if (module == "enc" && image) {
        if (!q) throw std::invalid_argument("Image encoder needs its QP parameter");
        const Tensor first = simple("enc.enc_1", x);
        return simple("enc.enc_2", multiply(first, q));
    }
    if (module == "dec" && image) {
        if (!q) throw std::invalid_argument("Image decoder needs its QP parameter");
        const Tensor first = simple("dec.dec_1", x);
        return simple("dec.dec_2", multiply(first, q));
    }
    if (module == "encoder") {
        if (args.size() != 2 || !q) throw std::invalid_argument("Video encoder needs context and QP");
        Tensor out = simple("encoder.conv1", cat({x, args[1]}));
        if (m_.has_child("encoder.conv2")) out = simple("encoder.conv2", out);
        return conv("encoder.down", multiply(out, q));
    }
    if (module == "decoder") {
        if (args.size() != 2 || !q) throw std::invalid_argument("Video decoder needs context and QP");
        const Tensor up = simple("decoder.up", x);
        Tensor out = simple("decoder.conv1", cat({up, args[1]}));
        if (m_.has("decoder.conv2.weight")) out = conv("decoder.conv2", out);
        return multiply(out, q);
    }
    if (module == "feature_adaptor_m") return simple(module + ".conv", args.size() > 1 ? cat(args) : x);
    if (module == "temporal_prior_encoder") {
        const std::string name = module + ".conv";
        if (q && m_.has(name + ".down.weight") && m_.has(name + ".conv.dc.0.weight")) {
            // multiply by the QP row fused into the down block's pixel_unshuffle(2)
            const Tensor down = conv(name + ".down", unshuffle2(x, q));
            return depth(name + ".conv", down, residual_shortcut());
        }
        return simple(name, q ? multiply(x, q) : x);
    }
    if (module == "y_prior_fusion" && !image && args.size() > 1) {
        const Tensor other = q ? multiply(args[1], q) : args[1];
        return simple(module + ".conv", cat({x, other}));
    }
    if (begins(module, "y_spatial_prior_adaptor_") && args.size() == 2) return depth(module, cat(args), false);
    if (module == "y_spatial_prior" && args.size() == 2) return simple(module + ".conv", cat(args));
    if (module == "hyper_enc" || module == "hyper_dec" || module == "hyper_encoder" || module == "hyper_decoder" ||
        module == "feature_adaptor_i" || module == "feature_extractor" || module == "y_spatial_prior" ||
        module == "y_prior_fusion")
        return simple(module + ".conv", args.size() > 1 ? cat(args) : x);
    return simple(module, x);
}

// Layers::reconstruct for HT-L (src/layers.cpp:209-215): recon heads without
// the final pixel_shuffle(8) (the output stage applies it).
std::vector<Tensor> Runner::reconstruct(const Tensor& feature, bool for_reset) {
    if (m_.variant() != "htl") throw std::invalid_argument("reconstruct is implemented for the HT-L variant");
    std::vector<Tensor> frames;
    for (int index = for_reset ? 7 : 0; index < 8; ++index)
        frames.push_back(simple("recon_head.conv." + std::to_string(index), feature));
    return frames;
}

// ----------------------------------------------------------------- codec ----

Codec::Codec(const Model& model, int batch) : m_(model), batch_(batch), pool_(model.device()) {
    if (batch <= 0) throw std::invalid_argument("batch must be positive");
    ck(cudaSetDevice(model.device()), "cudaSetDevice");
    ck(cudaStreamCreateWithFlags(&own_, cudaStreamNonBlocking), "stream");
    s_ = own_;
    ck(cudaMalloc(&status_, sizeof(int)), "status");
    ck(cudaMemset(status_, 0, sizeof(int)), "status");
    decoders_.resize(batch);
}

Codec::~Codec() {
    if (s_) cudaStreamSynchronize(s_);
    reference_ = memory_ = context_ = Tensor();
    last_frames_.clear();
    if (own_) {
        cudaStreamSynchronize(own_);
        cudaStreamDestroy(own_);
    }
    if (status_) cudaFree(status_);
}

void Codec::set_stream(cudaStream_t s) {
    // all pooled blocks are reused in stream order, so drain the old stream first
    ck(cudaStreamSynchronize(s_), "codec stream");
    s_ = s ? s : own_;
}

void Codec::set_skip_threshold(double threshold) {
    // IntegerModel::set_skip_threshold (src/integer_model.cpp:116-126)
    const volatile double scaled = threshold * kFeatureScale;
    const double rounded = std::trunc(scaled + 0.5);
    if (!std::isfinite(rounded) || rounded < 0 || rounded > 32767)
        throw std::invalid_argument("UF skip threshold is outside the INT16 feature range");
    skip_threshold_ = static_cast<int>(rounded);
}

void Codec::clear_dpb() {
    DeviceGuard device(m_.device());
    reference_ = memory_ = context_ = Tensor();
}

void Codec::sync_and_check() {
    ck(cudaStreamSynchronize(s_), "codec stream");
    stats_.collect();
    int st = 0;
    ck(cudaMemcpy(&st, status_, sizeof(int), cudaMemcpyDeviceToHost), "status read");
    if (st != 0) {
        cudaMemset(status_, 0, sizeof(int));
        throw std::runtime_error("kernel pipeline timeout (status " + std::to_string(st) + ")");
    }
}

template <class F>
void Codec::parallel_streams(F&& fn) {
    const auto t0 = std::chrono::steady_clock::now();
    const int hw = std::max(1u, std::thread::hardware_concurrency());
    const int workers = std::min(batch_, hw);
    if (workers <= 1) {
        for (int b = 0; b < batch_; ++b) fn(b);
    } else {
        std::vector<std::thread> pool;
        std::vector<std::exception_ptr> errors(workers);
        for (int w = 0; w < workers; ++w)
            pool.emplace_back([&, w] {
                try {
                    for (int b = w; b < batch_; b += workers) fn(b);
                } catch (...) {
                    errors[w] = std::current_exception();
                }
            });
        for (auto& t : pool) t.join();
        for (auto& e : errors)
            if (e) std::rethrow_exception(e);
    }
    host_seconds_ += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void Codec::add_ref_frames(const int16_t* frames, int h, int w) {
    DeviceGuard device(m_.device());
    // IntegerModel::add_ref_feature_from_frame: clear the DPB, reference =
    // pixel_unshuffle(frame, 8) (src/integer_model.cpp:107-114).
    if (h % 8 || w % 8) throw std::invalid_argument("reference frame extents must be multiples of 8");
    clear_dpb();
    Runner r(m_, pool_, s_, status_, &stats_);
    const size_t bytes = static_cast<size_t>(batch_) * 3 * h * w * 2;
    void* d = pool_.get(bytes);
    ck(cudaMemcpyAsync(d, frames, bytes, cudaMemcpyHostToDevice, s_), "reference upload");
    reference_ = r.alloc(batch_, h / 8, w / 8, 192);
    ck(nchw_to_split(static_cast<int16_t*>(d), batch_, 3, h, w, 8, reference_.a, s_), "reference unshuffle");
    stats_.launches += 1;
    sync_and_check();
    pool_.put(d, bytes);
}

void Codec::set_reference_from(const Codec& image) {
    DeviceGuard device(m_.device());
    if (image.last_frames_.empty()) throw std::runtime_error("image codec has no reconstruction");
    const Tensor& f = image.last_frames_.back();
    if (f.a.n != batch_ || f.a.c != 192) throw std::invalid_argument("reference batch or channels differ");
    clear_dpb();
    reference_ = f;  // shared device storage; the image codec's next call allocates new tensors
}

void Codec::update_context(Runner& r) {
    // src/integer_model.cpp:128-134
    if (!reference_.defined()) throw std::runtime_error("UF P-frame has no reference");
    memory_ = memory_.defined() ? r.run("feature_adaptor_m", {memory_, reference_})
                                : r.run("feature_adaptor_i", {reference_});
    context_ = r.run("feature_extractor", {memory_});
}

Tensor Codec::params(Runner& r, const Tensor& z, int qp, int y_h, int y_w) {
    // src/integer_model.cpp:184-200
    if (m_.variant() == "image") {
        const Tensor hyper = r.run("hyper_dec", {z});
        return r.run("y_prior_fusion", {hyper}).crop(y_h, y_w);
    }
    const Tensor hyper = r.run("hyper_decoder", {z}).crop(y_h, y_w);
    const ParamTable* q = m_.param("q_feature");
    if (!q) throw std::runtime_error("Missing prepared UF tensor: q_feature");
    const Tensor temporal = r.run("temporal_prior_encoder", {memory_}, q->data + static_cast<size_t>(qp) * q->cols);
    return r.run("y_prior_fusion", {hyper, temporal});
}

// IntegerModel::prior (src/integer_model.cpp:202-293).
Tensor Codec::prior(Runner& r, const Tensor* y, const Tensor& params, int qp, bool encode,
                    std::vector<std::vector<std::vector<int16_t>>>* packed_parts) {
    const bool image = m_.variant() == "image";
    const int C = 256;
    const int n = params.a.n, h = params.a.h, w = params.a.w;
    Tensor scales = params.channels(image ? 0 : 256, C);
    Tensor means = params.channels(image ? 256 : 512, C);
    const Tensor qraw = image ? Tensor() : params.channels(0, C);
    const int16_t* qrow = nullptr;
    if (image) {
        const ParamTable* q = m_.param(encode ? "q_scale_y_enc" : "q_scale_y_dec");
        if (!q) throw std::runtime_error("Missing prepared UF tensor: q_scale_y_*");
        qrow = q->data + static_cast<size_t>(qp) * q->cols;
    }
    Tensor yenc;
    if (encode) {
        yenc = r.alloc(n, h, w, C);
        if (image) {
            ck(mul_channels(y->a, qrow, yenc.a, r.stream()), "encode multiply");
            stats_.launches += 1;
        } else {
            // q_enc = reciprocal(max(q_raw, 256)); encoded_y = multiply(y, q_enc)
            Tensor qenc = r.alloc(n, h, w, C);
            ck(reciprocal_q(qraw.a, qenc.a, r.stream()), "reciprocal");
            stats_.launches += 1;
            ck(mul_elementwise(y->a, qenc.a, yenc.a, r.stream()), "encode multiply");
            stats_.launches += 1;
        }
    }
    // cat(restored, reduction) lives in one buffer so the adaptors read it in place
    Tensor rr = r.alloc(n, h, w, 2 * C);
    Tensor restored = rr.channels(0, C);
    Tensor reduction_view = rr.channels(C, C);
    r.conv("y_spatial_prior_reduction", params, Fuse(), &reduction_view);
    ck(fill_zero(restored.a, r.stream()), "restored clear");
    stats_.launches += 1;

    const long long cap = static_cast<long long>(C) * h * w;
    const int bps = prior_blocks_per_stream(C, h, w);
    int* d_counts = static_cast<int*>(pool_.get(sizeof(int) * (static_cast<size_t>(bps) * n + n)));
    int* d_totals = d_counts + static_cast<size_t>(bps) * n;
    void* d_buf = pool_.get(static_cast<size_t>(cap) * n * 2);
    int* h_totals = static_cast<int*>(pin_a_.get(sizeof(int) * n));
    uint8_t* h_buf = static_cast<uint8_t*>(pin_b_.get(static_cast<size_t>(cap) * n * 2));
    int8_t* h_sym = static_cast<int8_t*>(pin_c_.get(static_cast<size_t>(cap) * n));
    Tensor next;
    if (packed_parts) packed_parts->assign(n, std::vector<std::vector<int16_t>>(4));
    for (int part = 0; part < 4; ++part) {
        if (part) {
            const Tensor adapted = r.run("y_spatial_prior_adaptor_" + std::to_string(part), {rr});
            next = r.run("y_spatial_prior", {adapted});
            scales = next.channels(0, C);
            means = next.channels(C, C);
        }
        ck(prior_scan(C, h, w, n, part, scales.a, skip_threshold_, d_counts, d_totals, r.stream()), "prior scan");
    stats_.launches += 2;
        ck(cudaMemcpyAsync(h_totals, d_totals, sizeof(int) * n, cudaMemcpyDeviceToHost, r.stream()), "totals");
        if (!encode) {
            ck(prior_indexes(C, h, w, n, part, scales.a, skip_threshold_, d_counts, m_.scale_index(),
                             static_cast<uint8_t*>(d_buf), cap, r.stream()),
               "prior indexes");
            stats_.launches += 1;
            sync_and_check();
            for (int b = 0; b < n; ++b)
                if (h_totals[b])
                    ck(cudaMemcpyAsync(h_buf + b * cap, static_cast<uint8_t*>(d_buf) + b * cap, h_totals[b],
                                       cudaMemcpyDeviceToHost, r.stream()),
                       "indexes");
            ck(cudaStreamSynchronize(r.stream()), "indexes");
            parallel_streams([&](int b) {
                decoders_[b].decode_y(m_.y_table(), h_buf + b * cap, static_cast<size_t>(h_totals[b]),
                                      h_sym + b * cap);
            });
            int8_t* d_sym = static_cast<int8_t*>(d_buf);  // indexes are consumed; reuse the buffer
            for (int b = 0; b < n; ++b)
                if (h_totals[b])
                    ck(cudaMemcpyAsync(d_sym + b * cap, h_sym + b * cap, h_totals[b], cudaMemcpyHostToDevice,
                                       r.stream()),
                       "symbols");
            ck(prior_restore(C, h, w, n, part, scales.a, means.a, skip_threshold_, d_counts, d_sym, cap, restored.a,
                             r.stream()),
               "prior restore");
            stats_.launches += 1;
            // the host buffers are reused by the next part: wait for the uploads
            ck(cudaStreamSynchronize(r.stream()), "symbols");
        } else {
            ck(prior_encode(C, h, w, n, part, scales.a, means.a, yenc.a, skip_threshold_, d_counts, m_.scale_index(),
                            static_cast<int16_t*>(d_buf), cap, restored.a, r.stream()),
               "prior encode");
            stats_.launches += 1;
            sync_and_check();
            int16_t* hp = reinterpret_cast<int16_t*>(h_buf);
            for (int b = 0; b < n; ++b)
                if (h_totals[b])
                    ck(cudaMemcpyAsync(hp + b * cap, static_cast<int16_t*>(d_buf) + b * cap,
                                       sizeof(int16_t) * h_totals[b], cudaMemcpyDeviceToHost, r.stream()),
                       "packed");
            ck(cudaStreamSynchronize(r.stream()), "packed");
            for (int b = 0; b < n; ++b)
                (*packed_parts)[b][part].assign(hp + b * cap, hp + b * cap + h_totals[b]);
        }
    }
    pool_.put(d_buf, static_cast<size_t>(cap) * n * 2);
    pool_.put(d_counts, sizeof(int) * (static_cast<size_t>(bps) * n + n));
    Tensor yhat_t = r.alloc(n, h, w, C);
    if (image) {
        const ParamTable* q = m_.param("q_scale_y_dec");
        ck(mul_channels(restored.a, q->data + static_cast<size_t>(qp) * q->cols, yhat_t.a, r.stream()), "y_hat");
        stats_.launches += 1;
    } else {
        ck(yhat(restored.a, qraw.a, yhat_t.a, r.stream()), "y_hat");
        stats_.launches += 1;
    }
    return yhat_t;
}

// IntegerModel::reconstruct (src/integer_model.cpp:295-310).
std::vector<Tensor> Codec::reconstruct(Runner& r, const Tensor& y, int qp, bool reset, bool output_pixels) {
    if (m_.variant() == "image") {
        const ParamTable* q = m_.param("q_scale_dec");
        return {r.run("dec", {y}, q->data + static_cast<size_t>(qp) * q->cols)};
    }
    const ParamTable* q = m_.param("q_decoder");
    if (!q) throw std::runtime_error("Missing prepared UF tensor: q_decoder");
    const Tensor feature = r.run("decoder", {y, context_}, q->data + static_cast<size_t>(qp) * q->cols);
    std::vector<Tensor> frames;
    if (output_pixels) frames = r.reconstruct(feature, false);
    reference_ = feature;
    if (reset) {
        // the reset reference is recon head 7 before its pixel shuffle; when
        // the frames were produced it is the last one and is reused as is
        const Tensor head7 = output_pixels ? frames.back() : r.reconstruct(feature, true).at(0);
        clear_dpb();
        reference_ = head7;
    }
    return frames;
}

void Codec::emit_frames(const std::vector<Tensor>& frames, uint32_t width, uint32_t height, int16_t* frames_out,
                        uint8_t* yuv_out) {
    const int F = static_cast<int>(frames.size());
    if (!F) return;
    const int hp = frames[0].a.h * 8, wp = frames[0].a.w * 8;
    const size_t per_frame = static_cast<size_t>(3) * hp * wp;
    const size_t yuv_frame = static_cast<size_t>(width) * height * 3 / 2;
    if (frames_out) {
        const size_t bytes = per_frame * 2 * F * batch_;
        int16_t* d = static_cast<int16_t*>(pool_.get(bytes));
        for (int f = 0; f < F; ++f) {
            // batch-major output [b][f][3][hp][wp]: one shuffle per (b, f)
            for (int b = 0; b < batch_; ++b) {
                Act one = frames[f].a;
                one.base = frames[f].a.base + static_cast<long long>(b) * frames[f].a.img_px * 2 * frames[f].a.pitch;
                one.n = 1;
                ck(split_to_nchw(one, 8, d + (static_cast<size_t>(b) * F + f) * per_frame, s_), "frame shuffle");
                stats_.launches += 1;
            }
        }
        ck(cudaMemcpyAsync(frames_out, d, bytes, cudaMemcpyDeviceToHost, s_), "frames download");
        sync_and_check();
        pool_.put(d, bytes);
    }
    if (yuv_out) {
        const size_t bytes = yuv_frame * F * batch_;
        uint8_t* d = static_cast<uint8_t*>(pool_.get(bytes));
        for (int f = 0; f < F; ++f) {
            // every stream's frame f in one launch: stream b lands at (b * F + f) * yuv_frame
            ck(raw_frame(frames[f].a, static_cast<int>(height), static_cast<int>(width), d + f * yuv_frame,
                         static_cast<long long>(F) * yuv_frame, s_),
               "raw frame");
            stats_.launches += 1;
        }
        ck(cudaMemcpyAsync(yuv_out, d, bytes, cudaMemcpyDeviceToHost, s_), "yuv download");
        sync_and_check();
        pool_.put(d, bytes);
    }
}

// IntegerModel::decompress (src/integer_model.cpp:336-359).
int Codec::decompress(const uint8_t* const* payloads, const size_t* lengths, uint32_t width, uint32_t height, int qp,
                      bool reset, int16_t* frames_out, uint8_t* yuv_out) {
    check_interrupt();
    DeviceGuard device(m_.device());
    if (qp < 0 || qp >= 64 || !width || !height) throw std::invalid_argument("Unsupported UF integer packet parameters");
    host_seconds_ = 0;
    Runner r(m_, pool_, s_, status_, &stats_);
    const bool image = m_.variant() == "image";
    if (!image) update_context(r);  // queued on the GPU while the host decodes z
    const int y_h = static_cast<int>((height + 15) / 16), y_w = static_cast<int>((width + 15) / 16);
    const int z_h = (y_h + 3) / 4, z_w = (y_w + 3) / 4;
    const int zc = 128;
    const size_t zn = static_cast<size_t>(z_h) * z_w * zc;
    int8_t* hz = static_cast<int8_t*>(pin_c_.get(zn * batch_));
    parallel_streams([&](int b) {
        decoders_[b].set_stream(payloads[b], lengths[b]);
        decoders_[b].decode_z(m_.z_table(), zn, qp * zc, zc, hz + b * zn);
    });
    int8_t* dz = static_cast<int8_t*>(pool_.get(zn * batch_));
    ck(cudaMemcpyAsync(dz, hz, zn * batch_, cudaMemcpyHostToDevice, s_), "z upload");
    Tensor z = r.alloc(batch_, z_h, z_w, zc);
    ck(symbols_to_split(dz, z.a, s_), "from_symbols");
    stats_.launches += 1;
    const Tensor p = params(r, z, qp, y_h, y_w);
    const Tensor y_hat = prior(r, nullptr, p, qp, false, nullptr);
    pool_.put(dz, zn * batch_);
    const std::vector<Tensor> frames = reconstruct(r, y_hat, qp, reset, true);
    last_frames_ = frames;
    emit_frames(frames, width, height, frames_out, yuv_out);
    sync_and_check();
    return static_cast<int>(frames.size());
}

// IntegerModel::compress (src/integer_model.cpp:312-334).
int Codec::compress(const uint8_t* frames, int channels, int h, int w, int qp, bool reset,
                    std::vector<std::vector<uint8_t>>& payloads, int16_t* frames_out) {
    check_interrupt();
    DeviceGuard device(m_.device());
    if (qp < 0 || qp >= 64) throw std::invalid_argument("UF QP must be between 0 and 63");
    host_seconds_ = 0;
    Runner r(m_, pool_, s_, status_, &stats_);
    const bool image = m_.variant() == "image";
    const int hp = (h + 15) / 16 * 16, wp = (w + 15) / 16 * 16;  // pad_right_bottom(x, 16)
    const size_t in_bytes = static_cast<size_t>(batch_) * channels * h * w;
    uint8_t* d_in = static_cast<uint8_t*>(pool_.get(in_bytes));
    ck(cudaMemcpyAsync(d_in, frames, in_bytes, cudaMemcpyHostToDevice, s_), "frame upload");
    Tensor y;
    if (image) {
        if (channels != 3) throw std::invalid_argument("image model takes one frame");
        Tensor x = r.alloc(batch_, hp / 8, wp / 8, 192);
        ck(bytes_to_split_padded(d_in, batch_, channels, h, w, hp, wp, 8, x.a, s_), "frame unshuffle");
        stats_.launches += 1;
        const ParamTable* q = m_.param("q_scale_enc");
        y = r.run("enc", {x}, q->data + static_cast<size_t>(qp) * q->cols);
    } else {
        update_context(r);
        // cat(pixel_unshuffle(x, 8), context) built in place
        Tensor xin = r.alloc(batch_, hp / 8, wp / 8, channels * 64 + context_.a.c);
        Tensor xv = xin.channels(0, channels * 64);
        ck(bytes_to_split_padded(d_in, batch_, channels, h, w, hp, wp, 8, xv.a, s_), "frame unshuffle");
        stats_.launches += 1;
        Tensor cv = xin.channels(channels * 64, context_.a.c);
        ck(copy_channels(context_.a, cv.a, s_), "context cat");
        stats_.launches += 1;
        const ParamTable* q = m_.param("q_encoder");
        Tensor out = r.simple("encoder.conv1", xin);
        if (m_.has_child("encoder.conv2")) out = r.simple("encoder.conv2", out);
        y = r.conv("encoder.down", r.multiply(out, q->data + static_cast<size_t>(qp) * q->cols));
    }
    pool_.put(d_in, in_bytes);
    const int y_h = y.a.h, y_w = y.a.w;
    // z = symbols(hyper_encoder(pad_right_bottom(y, 4)))
    const int yph = (y_h + 3) / 4 * 4, ypw = (y_w + 3) / 4 * 4;
    Tensor ypad = r.alloc(batch_, yph, ypw, y.a.c);
    ck(pad_replicate(y.a, ypad.a, s_), "pad_right_bottom");
    stats_.launches += 1;
    const Tensor zf = r.run(image ? "hyper_enc" : "hyper_encoder", {ypad});
    const int z_h = zf.a.h, z_w = zf.a.w, zc = zf.a.c;
    const size_t zn = static_cast<size_t>(z_h) * z_w * zc;
    int8_t* dz = static_cast<int8_t*>(pool_.get(zn * batch_));
    ck(split_to_symbols(zf.a, dz, s_), "symbols");
    stats_.launches += 1;
    Tensor z = r.alloc(batch_, z_h, z_w, zc);
    ck(symbols_to_split(dz, z.a, s_), "from_symbols");
    stats_.launches += 1;
    int8_t* hz = static_cast<int8_t*>(pin_c_.get(zn * batch_));
    ck(cudaMemcpyAsync(hz, dz, zn * batch_, cudaMemcpyDeviceToHost, s_), "z download");
    std::vector<int8_t> zhost;
    sync_and_check();
    zhost.assign(hz, hz + zn * batch_);
    pool_.put(dz, zn * batch_);
    const Tensor p = params(r, z, qp, y_h, y_w);
    std::vector<std::vector<std::vector<int16_t>>> parts;
    const Tensor y_hat = prior(r, &y, p, qp, true, &parts);
    payloads.assign(batch_, {});
    parallel_streams([&](int b) {
        RansEncoder enc;
        enc.reset();
        for (int part = 3; part >= 0; --part)
            if (!parts[b][part].empty()) enc.encode_y(m_.y_table(), parts[b][part].data(), parts[b][part].size());
        enc.encode_z(m_.z_table(), zhost.data() + b * zn, zn, qp * zc, zc);
        payloads[b] = enc.flush();
    });
    const std::vector<Tensor> rec = reconstruct(r, y_hat, qp, reset, frames_out != nullptr || image);
    last_frames_ = rec;
    if (frames_out) {
        emit_frames(rec, static_cast<uint32_t>(wp), static_cast<uint32_t>(hp), frames_out, nullptr);
    }
    sync_and_check();
    return static_cast<int>(rec.size());
}

bool Codec::state_shape(int which, int64_t* shape4) const {
    const Tensor& t = which == 0 ? reference_ : which == 1 ? memory_ : context_;
    if (!t.defined()) return false;
    shape4[0] = t.a.n;
    shape4[1] = t.a.c;
    shape4[2] = t.a.h;
    shape4[3] = t.a.w;
    return true;
}

bool Codec::state(int which, int16_t* out, size_t capacity, int64_t* shape4) {
    DeviceGuard device(m_.device());
    const Tensor& t = which == 0 ? reference_ : which == 1 ? memory_ : context_;
    if (!t.defined()) return false;
    const size_t n = static_cast<size_t>(t.a.n) * t.a.c * t.a.h * t.a.w;
    if (capacity < n) throw std::length_error("state buffer too small");
    int16_t* d = static_cast<int16_t*>(pool_.get(n * 2));
    ck(split_to_nchw(t.a, 1, d, s_), "state layout");
    ck(cudaMemcpyAsync(out, d, n * 2, cudaMemcpyDeviceToHost, s_), "state download");
    sync_and_check();
    pool_.put(d, n * 2);
    shape4[0] = t.a.n;
    shape4[1] = t.a.c;
    shape4[2] = t.a.h;
    shape4[3] = t.a.w;
    return true;
}

}  // namespace ufb
