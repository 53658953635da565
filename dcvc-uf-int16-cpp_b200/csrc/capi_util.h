// Error reporting and stream-ordered scratch buffers shared by the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace ufb {

// Thread-local last error (message + code) reported by ufb_last_error().
void clear_error();
bool fail(int code, const std::string& message);  // records, returns false
inline int err(int code, const std::string& message) {
    fail(code, message);
    return code;
}
int last_code();
const char* last_message();
bool cuda_ok(cudaError_t e, const char* what);     // records UFB_ECUDA on failure

// Per-device kernel status word (pipeline timeouts): a device variable of the
// library resolved on first use (status.cu); null with the error recorded when
// the address cannot be resolved.
int* device_status(int device);

// Argument checks of uf_conv (src/cuda/conv.cu:65-83) shared by every
// convolution entry point; fills the output extent.
bool check_conv(const int16_t* x, int n, int ci, int h, int w, const int16_t* weight, int co, int kh, int kw,
                int bias_bits, int sh, int sw, int ph, int pw, int groups, const int16_t* out, int& oh, int& ow);

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Scratch memory allocated and released in stream order (cudaMallocAsync /
// cudaFreeAsync), so concurrent calls on different streams never share it.
class StreamBuffer {
public:
    StreamBuffer(size_t bytes, cudaStream_t stream) : stream_(stream) {
        if (bytes == 0) bytes = 256;
        ok_ = cudaMallocAsync(&ptr_, bytes, stream) == cudaSuccess;
        if (!ok_) ptr_ = nullptr;
    }
    ~StreamBuffer() {
        if (ptr_) cudaFreeAsync(ptr_, stream_);
    }
    StreamBuffer(const StreamBuffer&) = delete;
    StreamBuffer& operator=(const StreamBuffer&) = delete;
    bool ok() const { return ok_; }
    template <class T>
    T* get() const {
        return static_cast<T*>(ptr_);
    }

private:
    void* ptr_ = nullptr;
    cudaStream_t stream_;
    bool ok_ = false;
};

}  // namespace ufb
