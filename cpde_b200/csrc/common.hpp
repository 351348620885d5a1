// Shared host utilities of the cpde_b200 engine: error types, CUDA checks that
// throw instead of exiting, and RAII device buffers.
#pragma once
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace cpde {

// A rejected request (bad handle, shape, value). The engine stays usable.
struct RequestError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// A CUDA runtime/driver failure. The device may no longer be usable.
struct DeviceError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void require(bool ok, const char* message) {
    if (!ok) throw RequestError(message);
}
inline void require(bool ok, const std::string& message) {
    if (!ok) throw RequestError(message);
}

inline void cuda_check(cudaError_t status, const char* what, const char* file, int line) {
    if (status == cudaSuccess) return;
    throw DeviceError(std::string(file) + ":" + std::to_string(line) + ": " + what + " failed: " +
                      cudaGetErrorString(status));
}
#define CPDE_CUDA(expr) ::cpde::cuda_check((expr), #expr, __FILE__, __LINE__)
#define CPDE_LAUNCHED() ::cpde::cuda_check(cudaGetLastError(), "kernel launch", __FILE__, __LINE__)

// Product of positive dimensions that must fit the int32 indexing of the
// protocol's array headers (same rule as cuda/cpde_server.cu:23-25).
inline int checked_size(long long a, long long b, long long c = 1) {
    long long n = a * b * c;
    require(a > 0 && b > 0 && c > 0 && n <= INT_MAX, "invalid or excessive dimensions");
    return int(n);
}

// Owning device allocation; contents undefined until written.
template <class T>
struct DeviceBuffer {
    T* ptr = nullptr;
    size_t count = 0;
    DeviceBuffer() = default;
    explicit DeviceBuffer(size_t n) { resize(n); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& o) noexcept : ptr(o.ptr), count(o.count) { o.ptr = nullptr; o.count = 0; }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
        if (this != &o) { release(); ptr = o.ptr; count = o.count; o.ptr = nullptr; o.count = 0; }
        return *this;
    }
    ~DeviceBuffer() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        count = 0;
    }
    // Grows (never shrinks) to at least n elements; old contents are dropped.
    void reserve(size_t n) {
        if (n <= count) return;
        resize(n);
    }
    void resize(size_t n) {
        release();
        if (n) CPDE_CUDA(cudaMalloc((void**)&ptr, n * sizeof(T)));
        count = n;
    }
    // Copies n elements from host memory, reallocating only when n changes.
    void upload(const T* host, size_t n, cudaStream_t stream = 0) {
        if (n != count) resize(n);
        if (n) CPDE_CUDA(cudaMemcpyAsync(ptr, host, n * sizeof(T), cudaMemcpyHostToDevice, stream));
    }
    void upload(const std::vector<T>& v, cudaStream_t stream = 0) { upload(v.data(), v.size(), stream); }
    size_t bytes() const { return count * sizeof(T); }
};

// Page-locked host staging area for small per-epoch downloads.
template <class T>
struct PinnedBuffer {
    T* ptr = nullptr;
    size_t count = 0;
    PinnedBuffer() = default;
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    ~PinnedBuffer() { if (ptr) cudaFreeHost(ptr); }
    void reserve(size_t n) {
        if (n <= count) return;
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        CPDE_CUDA(cudaHostAlloc((void**)&ptr, n * sizeof(T), cudaHostAllocDefault));
        count = n;
    }
};

}  // namespace cpde
