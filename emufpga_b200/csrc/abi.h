// Shared by the translation units that implement C ABI entry points: every
// entry point runs its body under guarded(), which turns a thrown Error into
// its status code and the thread's spm_last_error() message.
#pragma once
#include <cuda_runtime_api.h>

#include <exception>
#include <new>
#include <string>

#include "common.h"

#define CUDA_OK(expr)                                                                        \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess) spm::fail(SPM_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

namespace spm {

template <class F>
spm_status guarded(F&& f) {
    try {
        f();
        return SPM_OK;
    } catch (const Error& e) {
        set_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc&) {
        set_error("host allocation failed");
        return SPM_E_ARG;
    } catch (const std::exception& e) {
        set_error(e.what());
        return SPM_E_ARG;
    }
}

struct DeviceBuf {
    void* p = nullptr;
    DeviceBuf() = default;
    DeviceBuf(const DeviceBuf&) = delete;
    DeviceBuf& operator=(const DeviceBuf&) = delete;
    ~DeviceBuf() { if (p) cudaFree(p); }
};

}  // namespace spm
