// Host plumbing shared by the library's C ABI entry points: the error types
// that map to its status codes, the CUDA check, device buffers, and the
// guard every extern "C" function runs its body in.
#pragma once

#include "../../include/wsp_decoder.h"

#include <cuda_runtime.h>

#include <new>
#include <stdexcept>
#include <string>

namespace wsp {

// -------------------------------------------------------------- errors

struct ModelError : std::runtime_error { using std::runtime_error::runtime_error; };
struct LogicError : std::logic_error { using std::logic_error::logic_error; };
struct InvalidArgument : std::invalid_argument { using std::invalid_argument::invalid_argument; };
struct CudaFailure : std::runtime_error {
    bool out_of_memory;
    CudaFailure(const std::string& what, bool oom) : std::runtime_error(what), out_of_memory(oom) {}
};

// The text of the calling thread's last failed call (wsp_last_error).
std::string& last_error_text();

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(e), e == cudaErrorMemoryAllocation);
}
#define CUDA_CHECK(x) cuda_check((x), #x)

// ------------------------------------------------------- device memory

// Host-side memsets and pageable copies run on the legacy default stream,
// and may still be in flight when the call returns (a pageable copy returns
// once the data is staged; a memset of device memory once it is queued).
// The decoder launches on a non-blocking stream, which does not wait for
// the legacy one -- and a cooperative launch that holds every SM can keep
// a queued memset from running until after it.  So every such call is
// followed by this wait before anything the decoder launches can read the
// memory.
inline void settle_legacy_stream() { CUDA_CHECK(cudaStreamSynchronize(cudaStreamLegacy)); }

class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { release(); }

    void allocate(size_t bytes) {
        release();
        if (bytes == 0) bytes = 16;
        CUDA_CHECK(cudaMalloc(&ptr_, bytes));
        CUDA_CHECK(cudaMemset(ptr_, 0, bytes));
        settle_legacy_stream();
        bytes_ = bytes;
    }
    void release() {
        if (ptr_) cudaFree(ptr_);
        ptr_ = nullptr;
        bytes_ = 0;
    }
    template <typename T = void> T* get() const { return static_cast<T*>(ptr_); }
    size_t bytes() const { return bytes_; }

private:
    void* ptr_ = nullptr;
    size_t bytes_ = 0;
};


// Runs an entry point's body: its exceptions become status codes, their
// text the thread's last error.
template <typename F>
int guarded(F&& f) {
    try {
        f();
        last_error_text().clear();
        return WSP_OK;
    } catch (const ModelError& e) {
        last_error_text() = e.what();
        return WSP_MODEL_ERROR;
    } catch (const InvalidArgument& e) {
        last_error_text() = e.what();
        return WSP_INVALID_ARGUMENT;
    } catch (const LogicError& e) {
        last_error_text() = e.what();
        return WSP_LOGIC_ERROR;
    } catch (const CudaFailure& e) {
        last_error_text() = e.what();
        return e.out_of_memory ? WSP_OUT_OF_MEMORY : WSP_CUDA_ERROR;
    } catch (const std::bad_alloc&) {
        last_error_text() = "host allocation failed";
        return WSP_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        last_error_text() = e.what();
        return WSP_LOGIC_ERROR;
    }
}


}  // namespace wsp
