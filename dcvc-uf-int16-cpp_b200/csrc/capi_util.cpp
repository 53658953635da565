#include "capi_util.h"

#include "uf_b200.h"

#include <mutex>
#include <vector>

namespace ufb {

namespace {
thread_local std::string g_message;
thread_local int g_code = 0;
std::mutex g_status_mutex;
std::vector<int*> g_status;
}  // namespace

void clear_error() {
    g_message.clear();
    g_code = 0;
}

bool fail(int code, const std::string& message) {
    g_code = code;
    g_message = message;
    return false;
}

int last_code() { return g_code ? g_code : UFB_ECUDA; }

const char* last_message() { return g_message.c_str(); }

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    return fail(UFB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int* device_status(int device) {
    std::lock_guard<std::mutex> lock(g_status_mutex);
    if (device < 0) {
        fail(UFB_EINVAL, "invalid device");
        return nullptr;
    }
    if (static_cast<size_t>(device) >= g_status.size()) g_status.resize(device + 1, nullptr);
    if (!g_status[device]) {
        int current = 0;
        cudaGetDevice(&current);
        if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return nullptr;
        int* p = nullptr;
        const bool ok = cuda_ok(cudaMalloc(&p, sizeof(int)), "status allocation") &&
                        cuda_ok(cudaMemset(p, 0, sizeof(int)), "status clear");
        cudaSetDevice(current);
        if (!ok) return nullptr;
        g_status[device] = p;
    }
    return g_status[device];
}

}  // namespace ufb
