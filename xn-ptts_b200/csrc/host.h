// Host-side helpers shared by the C ABI translation units: error plumbing (status codes plus a
// thread-local message; no exception crosses the ABI), device scope, grow-only device buffers
// and pinned staging for small uploads.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>

#include "ptts_b200.h"

namespace ptts {
namespace host {

// This thread's last error message (ptts_b200_last_error).
inline thread_local std::string g_last_error;

struct Error {
    int code;
    std::string msg;
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error{code, msg}; }

#define CK(call)                                                                             \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) fail(PTTS_B200_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

template <class F>
int guarded(F&& f) {
    try {
        f();
        return PTTS_B200_OK;
    } catch (const Error& e) {
        g_last_error = e.msg;
        return e.code;
    } catch (const std::exception& e) {
        g_last_error = std::string("internal error: ") + e.what();
        return PTTS_B200_ERR_STATE;
    } catch (...) {
        g_last_error = "internal error: unknown exception";
        return PTTS_B200_ERR_STATE;
    }
}

// Checks that run per stream build their message only on failure (`if (!ok) fail(...)`): a
// message assembled before the test costs an allocation per stream per call.
inline void require(bool ok, int code, const char* msg) {
    if (!ok) fail(code, msg);
}
inline void require(bool ok, int code, const std::string& msg) {
    if (!ok) fail(code, msg);
}

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev) {
        CK(cudaGetDevice(&prev));
        if (prev != dev) CK(cudaSetDevice(dev));
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Grow-only device buffer.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    void* need(size_t n) {
        if (n <= bytes) return p;
        if (p) {
            CK(cudaDeviceSynchronize());
            CK(cudaFree(p));
            p = nullptr;
            bytes = 0;
        }
        CK(cudaMalloc(&p, n));
        bytes = n;
        return p;
    }
    // Free the memory (the buffer reads as empty again).
    void release() {
        if (p) {
            CK(cudaDeviceSynchronize());
            CK(cudaFree(p));
        }
        p = nullptr;
        bytes = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
    // Like need(), and zero-filled whenever it is (re)allocated.
    void* need_zeroed(size_t n) {
        if (n <= bytes) return p;
        need(n);
        CK(cudaMemset(p, 0, n));
        return p;
    }
};

// Pinned staging for small host -> device uploads: a ring of slots, each reused only after its
// previous copy has completed, so a call does not wait for the device's earlier work.
struct Staging {
    static constexpr int kSlots = 16;
    void* host[kSlots] = {};
    size_t bytes[kSlots] = {};
    cudaEvent_t done[kSlots] = {};
    int next = 0;
    ~Staging() {
        for (int i = 0; i < kSlots; ++i) {
            if (host[i]) cudaFreeHost(host[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
    }
    void upload(void* dev, const void* src, size_t n, cudaStream_t s) {
        const int i = next;
        next = (next + 1) % kSlots;
        if (!done[i]) CK(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
        CK(cudaEventSynchronize(done[i]));
        if (n > bytes[i]) {
            if (host[i]) CK(cudaFreeHost(host[i]));
            host[i] = nullptr;
            CK(cudaMallocHost(&host[i], n < 4096 ? 4096 : n));
            bytes[i] = n < 4096 ? 4096 : n;
        }
        std::memcpy(host[i], src, n);
        CK(cudaMemcpyAsync(dev, host[i], n, cudaMemcpyHostToDevice, s));
        CK(cudaEventRecord(done[i], s));
    }
};

// f16 bits -> f32 (exact; subnormals, infinities and NaN included).
inline float f16_value(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FFu;
    float v;
    if (exp == 0) v = std::ldexp((float)man, -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = std::ldexp((float)(man | 0x400u), (int)exp - 25);
    uint32_t u;
    std::memcpy(&u, &v, 4);
    u |= sign;
    std::memcpy(&v, &u, 4);
    return v;
}

}  // namespace host
}  // namespace ptts
