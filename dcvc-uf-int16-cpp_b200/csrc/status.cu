// Per-device kernel status word: pipeline kernels record a bounded-wait
// timeout here (a nonzero code) instead of hanging; ufb_device_status reads
// and clears it.  The word is a file-scope device variable, so every GPU that
// loads the library has its own copy from module load on, already zero, and
// no call ever allocates device memory for it.
#include "capi_util.h"

#include "uf_b200.h"

#include <mutex>
#include <vector>

namespace ufb {

namespace {

static __device__ __align__(16) int g_status_word;

std::mutex g_status_mutex;
std::vector<int*> g_status;  // device address per ordinal, null until resolved

}  // namespace

int* device_status(int device) {
    std::lock_guard<std::mutex> lock(g_status_mutex);
    if (device < 0) {
        fail(UFB_EINVAL, "invalid device");
        return nullptr;
    }
    if (static_cast<size_t>(device) >= g_status.size()) g_status.resize(device + 1, nullptr);
    if (!g_status[device]) {
        // host code names only the host shadow of g_status_word: resolve the
        // device address with that device current
        int current = 0;
        if (!cuda_ok(cudaGetDevice(&current), "cudaGetDevice")) return nullptr;
        if (current != device && !cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return nullptr;
        void* p = nullptr;
        const bool ok = cuda_ok(cudaGetSymbolAddress(&p, g_status_word), "cudaGetSymbolAddress(status)");
        if (current != device) cudaSetDevice(current);
        if (!ok) return nullptr;
        g_status[device] = static_cast<int*>(p);
    }
    return g_status[device];
}

}  // namespace ufb
