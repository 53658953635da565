// Model-level engine: prepared-model upload, the module-graph runner
// (counterpart of the reference's uf::Layers, src/layers.cpp) and the
// per-stream codec state machine (counterpart of uf::IntegerModel,
// src/integer_model.cpp), all on split-NHWC device tensors.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "conv_tc.h"
#include "rans.h"
#include "uf_common.cuh"

namespace ufb {

// A failing CUDA runtime call inside the engine (maps to UFB_ECUDA).
struct CudaFailure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Stream-ordered device memory reuse: every tensor of one engine lives on one
// CUDA stream, so a block returned to the pool may be handed out again at
// once -- later work on the same stream runs after earlier readers finish.
class DevicePool {
public:
    explicit DevicePool(int device) : device_(device) {}
    ~DevicePool();
    DevicePool(const DevicePool&) = delete;
    DevicePool& operator=(const DevicePool&) = delete;
    void* get(size_t bytes);
    void put(void* p, size_t bytes);
    size_t reserved() const { return reserved_; }

private:
    int device_;
    std::map<size_t, std::vector<void*>> free_;
    std::vector<void*> all_;
    size_t reserved_ = 0;
};

struct Block {
    DevicePool* pool;
    void* ptr;
    size_t bytes;
    ~Block() { pool->put(ptr, bytes); }
};

// Split-NHWC tensor: shared ownership of a device block plus a view.
struct Tensor {
    std::shared_ptr<Block> mem;
    Act a{};
    bool defined() const { return static_cast<bool>(mem); }
    Tensor channels(int c0, int c) const;
    Tensor crop(int h, int w) const;
};

struct ConvLayer {
    int co = 0, ci = 0, kh = 0, kw = 0;
    bool depthwise = false;
    bool dw_narrow = false;       // depthwise sums fit one int32 (dw_narrow_ok)
    TcWeights tc;                 // groups == 1 layers
    int16_t* weights16 = nullptr; // original int16 weights (depthwise, strided, direct paths)
    int16_t* bias = nullptr;      // int16 [co] or null
};

struct ParamTable {
    int rows = 0, cols = 0;
    int16_t* data = nullptr;      // [rows][cols] on the device
};

struct HostTensor {
    std::string name;
    int dtype;                    // 0 int16, 1 uint8, 2 int32, 3 int8, 4 int64
    std::vector<int64_t> shape;
    const void* data;
};

class Model {
public:
    Model(int device, const std::string& variant, const std::vector<HostTensor>& tensors);
    ~Model();
    Model(const Model&) = delete;
    Model& operator=(const Model&) = delete;

    const std::string& variant() const { return variant_; }
    int device() const { return device_; }
    const ConvLayer* conv(const std::string& name) const;
    const ParamTable* param(const std::string& name) const;
    bool has(const std::string& name) const { return names_.count(name) != 0; }
    bool has_child(const std::string& prefix) const;
    const int16_t* wsilu() const { return wsilu_; }
    // shared-memory window of the WSiLU table (Epilogue::lut_start / lut_n / lut_hi)
    int wsilu_start() const { return wsilu_start_; }
    int wsilu_n() const { return wsilu_n_; }
    int wsilu_hi() const { return wsilu_hi_; }
    const uint8_t* scale_index() const { return scale_index_; }
    const RansTables& z_table() const { return z_table_; }
    const RansTables& y_table() const { return y_table_; }

private:
    int device_;
    std::string variant_;
    std::set<std::string> names_;
    std::map<std::string, ConvLayer> convs_;
    std::map<std::string, ParamTable> params_;
    std::vector<void*> allocations_;
    int16_t* wsilu_ = nullptr;
    int wsilu_start_ = 0, wsilu_n_ = 0, wsilu_hi_ = 0;
    uint8_t* scale_index_ = nullptr;
    RansTables z_table_, y_table_;
};

// Launch accounting of one engine (all kernels) and, when profiling is on,
// CUDA-event timing of the tensor-core convolution launches.
// Makes `device` current in the calling thread for the guard's lifetime (the
// engine's objects may be driven from any host thread, each of which starts
// on device 0) and restores the previous device.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        if (prev_ != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_ = -1;
};

struct EngineStats {
    long long launches = 0;        // kernels launched
    long long conv_launches = 0;   // tensor-core convolution launches
    double conv_int16_macs = 0;    // algorithmic int16 MACs of those launches
    double conv_ms = 0;            // summed event time of those launches (profiling on)
    bool profile = false;
    // per launch shape and epilogue ("conv ci>co kh x kw +epilogue @ pixels",
    // "depthwise c 3x3 @ pixels"), filled while profiling is on; hbm_bytes is
    // the launch's algorithmic DRAM traffic (input and residuals read once,
    // output written once, weights)
    struct Shape {
        long long launches = 0;
        double int16_macs = 0;
        double ms = 0;
        double hbm_bytes = 0;
    };
    std::map<std::string, Shape> shapes;
    struct Pending {
        cudaEvent_t start, stop;
        std::string shape;
        bool tensor_core;
    };
    std::vector<Pending> pending;
    std::vector<cudaEvent_t> spare;
    cudaEvent_t take_event();
    void collect();                // adds the elapsed time of completed launches
    void reset();
    ~EngineStats();
};

// Epilogue options of one convolution call.
struct Fuse {
    bool lut = false;
    bool wsilu4 = false;
    bool shuffle2 = false;
    const Tensor* res1 = nullptr;
    const Tensor* res2 = nullptr;
    const int16_t* mulq = nullptr;
};

// Executes module paths by parameter name, mirroring src/layers.cpp:74-216.
class Runner {
public:
    Runner(const Model& m, DevicePool& pool, cudaStream_t s, int* status, EngineStats* stats = nullptr)
        : m_(m), pool_(pool), s_(s), status_(status), stats_(stats) {}
    void count(int n = 1) {
        if (stats_) stats_->launches += n;
    }
    Tensor alloc(int n, int h, int w, int c);
    Tensor conv(const std::string& name, const Tensor& in, const Fuse& f = Fuse(), const Tensor* out = nullptr);
    Tensor depth(const std::string& name, const Tensor& in, bool shortcut, const Tensor* out = nullptr);
    Tensor simple(const std::string& name, const Tensor& in, bool shortcut = false);
    // Layers::run for one module; q_row: device row of the module's QP table
    // (multiply argument) or null.
    Tensor run(const std::string& module, const std::vector<Tensor>& args, const int16_t* q_row = nullptr);
    std::vector<Tensor> reconstruct(const Tensor& feature, bool for_reset);
    Tensor cat(const std::vector<Tensor>& parts);
    Tensor multiply(const Tensor& x, const int16_t* q_row);
    Tensor unshuffle2(const Tensor& x, const int16_t* q_row);
    cudaStream_t stream() const { return s_; }
    const Model& model() const { return m_; }
    DevicePool& pool() { return pool_; }
    int* status() const { return status_; }

private:
    bool residual_shortcut() const;
    const Model& m_;
    DevicePool& pool_;
    cudaStream_t s_;
    int* status_;
    EngineStats* stats_;
};

// Host buffers pinned for transfers, grown on demand.
class Pinned {
public:
    ~Pinned();
    void* get(size_t bytes);

private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

// Per-stream-batch codec state (uf::IntegerModel).  `batch` independent video
// streams are processed together as the N dimension of every tensor; they share
// the model, QP and reset flag, and each has its own entropy-coded payload.
class Codec {
public:
    Codec(const Model& model, int batch);
    ~Codec();
    int batch() const { return batch_; }
    void set_skip_threshold(double t);
    void clear_dpb();
    // frames: host int16 [batch][3][h][w] (IntegerModel::add_ref_feature_from_frame)
    void add_ref_frames(const int16_t* frames, int h, int w);
    // IntegerModel::decompress for every stream of the batch.  frames_out:
    // host int16 [batch][F][3][Hp][Wp] or null; yuv_out: host u8
    // [batch][F][w*h*3/2] (IntegerCodec::raw_frame) or null.
    int decompress(const uint8_t* const* payloads, const size_t* lengths, uint32_t width, uint32_t height, int qp,
                   bool reset, int16_t* frames_out, uint8_t* yuv_out);
    // IntegerModel::compress: frames host uint8 YUV444 [batch][3F][h][w]
    // (from_bytes applied on the device).  Payloads are returned per stream.
    int compress(const uint8_t* frames, int channels, int h, int w, int qp, bool reset,
                 std::vector<std::vector<uint8_t>>& payloads, int16_t* frames_out);
    // state: 0 reference, 1 memory, 2 context; copies NCHW int16 to host.
    // Returns false when the state is undefined.
    bool state(int which, int16_t* out, size_t capacity, int64_t* shape4);
    // NCHW shape of a state (false when undefined)
    bool state_shape(int which, int64_t* shape4) const;
    int frames_per_packet() const { return m_.variant() == "image" ? 1 : 8; }
    double last_host_seconds() const { return host_seconds_; }
    // reference = another codec's last reconstruction (device to device): the
    // image model's output is pixel_unshuffle(frame, 8) of the I frame, which
    // is what add_ref_feature_from_frame stores (src/integer_model.cpp:107-114)
    void set_reference_from(const Codec& image);
    EngineStats& stats() { return stats_; }
    // run on a caller-owned CUDA stream from now on (null: back to our own)
    void set_stream(cudaStream_t s);

private:
    void update_context(Runner& r);
    Tensor params(Runner& r, const Tensor& z, int qp, int y_h, int y_w);
    Tensor prior(Runner& r, const Tensor* y, const Tensor& params, int qp, bool encode,
                 std::vector<std::vector<std::vector<int16_t>>>* packed_parts);
    std::vector<Tensor> reconstruct(Runner& r, const Tensor& y, int qp, bool reset, bool output_pixels);
    void emit_frames(const std::vector<Tensor>& frames, uint32_t width, uint32_t height, int16_t* frames_out,
                     uint8_t* yuv_out);
    void sync_and_check();
    template <class F>
    void parallel_streams(F&& fn);

    const Model& m_;
    int batch_;
    DevicePool pool_;
    cudaStream_t s_ = nullptr;
    cudaStream_t own_ = nullptr;
    int* status_ = nullptr;
    int skip_threshold_ = 0;
    Tensor reference_, memory_, context_;
    std::vector<RansDecoder> decoders_;
    Pinned pin_a_, pin_b_, pin_c_;
    double host_seconds_ = 0;
    std::vector<Tensor> last_frames_;  // last reconstruction (head outputs, 192 ch)
    EngineStats stats_;
};

}  // namespace ufb
