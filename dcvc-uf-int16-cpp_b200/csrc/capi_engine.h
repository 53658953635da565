// Handles and error translation shared by the engine-level C ABI files
// (capi_engine.cpp, capi_stream.cpp).
#pragma once

#include "uf_b200.h"

#include "capi_util.h"
#include "engine.h"
#include "interrupt.h"
#include "rans.h"

#include <memory>
#include <new>
#include <stdexcept>
#include <string>

struct ufb_model {
    std::unique_ptr<ufb::Model> m;
    ufb::DevicePool pool;
    cudaStream_t s = nullptr;
    int* status = nullptr;
    explicit ufb_model(int device) : pool(device) {}
};

struct ufb_codec {
    std::unique_ptr<ufb::Codec> c;
};

namespace ufb {

// Runs fn, mapping exceptions to UFB_E* codes and the thread-local message.
template <class F>
inline int guarded(F&& fn) {
    clear_error();
    try {
        return fn();
    } catch (const Interrupted& e) {
        return err(UFB_EINTR, e.what());
    } catch (const StreamError& e) {
        return err(UFB_ESTREAM, e.what());
    } catch (const CudaFailure& e) {
        return err(UFB_ECUDA, e.what());
    } catch (const std::invalid_argument& e) {
        return err(UFB_EINVAL, e.what());
    } catch (const std::length_error& e) {
        return err(UFB_ERANGE, e.what());
    } catch (const std::overflow_error& e) {
        return err(UFB_ERANGE, e.what());
    } catch (const std::out_of_range& e) {
        return err(UFB_ERANGE, e.what());
    } catch (const std::bad_alloc&) {
        return err(UFB_ECUDA, "host allocation failed");
    } catch (const std::exception& e) {
        return err(UFB_ESTATE, e.what());
    }
}

inline void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace ufb
