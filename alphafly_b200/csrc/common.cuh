// Shared helpers of the alphafly_b200 CUDA library: error reporting, device buffers, launch checks.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/afb.h"

namespace afb {

// Status-carrying exception used inside the library; the C ABI converts it to a return code and
// stores the message for afb_last_error().
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string &msg);

#define AFB_CUDA(call)                                                                          \
    do {                                                                                        \
        cudaError_t err_ = (call);                                                              \
        if (err_ != cudaSuccess)                                                                \
            throw ::afb::Error(AFB_ECUDA, std::string(#call) + ": " + cudaGetErrorString(err_)); \
    } while (0)

#define AFB_CHECK(cond, msg)                                                  \
    do {                                                                      \
        if (!(cond)) throw ::afb::Error(AFB_EINVAL, std::string(msg));        \
    } while (0)

#define AFB_LAUNCHED() AFB_CUDA(cudaGetLastError())

// Runs `body`, translating exceptions into an AFB status code.
template <typename F>
int guarded(F &&body) {
    try {
        body();
        return AFB_OK;
    } catch (const Error &e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc &) {
        set_last_error("host allocation failed");
        return AFB_ECUDA;
    } catch (const std::exception &e) {
        set_last_error(e.what());
        return AFB_ECUDA;
    }
}

// Owning device buffer (cudaMalloc / cudaFree); used only by set-up paths, never per forward call.
template <typename T>
struct DevBuf {
    T *p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    explicit DevBuf(size_t count) { alloc(count); }
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : p(o.p), n(o.n) { o.p = nullptr; o.n = 0; }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) { release(); p = o.p; n = o.n; o.p = nullptr; o.n = 0; }
        return *this;
    }
    ~DevBuf() { release(); }
    void alloc(size_t count) {
        release();
        n = count;
        if (count) AFB_CUDA(cudaMalloc(&p, count * sizeof(T)));
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    T *get() const { return p; }
};

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline int grid_for(int64_t n, int block, int cap = 148 * 32) {
    int64_t g = (n + block - 1) / block;
    if (g < 1) g = 1;
    return (int)(g < cap ? g : cap);
}

template <typename T>
std::vector<T> to_host(const T *d, size_t n, cudaStream_t s) {
    std::vector<T> h(n);
    if (n) {
        AFB_CUDA(cudaMemcpyAsync(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost, s));
        AFB_CUDA(cudaStreamSynchronize(s));
    }
    return h;
}

template <typename T>
void to_device(T *d, const std::vector<T> &h, cudaStream_t s) {
    if (!h.empty()) {
        AFB_CUDA(cudaMemcpyAsync(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice, s));
        AFB_CUDA(cudaStreamSynchronize(s));
    }
}

inline void check_aligned(const void *p, size_t a, const char *what) {
    AFB_CHECK((reinterpret_cast<uintptr_t>(p) % a) == 0, std::string(what) + " must be " + std::to_string(a) + "-byte aligned");
}

}  // namespace afb
