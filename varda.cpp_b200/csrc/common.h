// Shared host/device helpers of libvarda_b200: error type, CUDA checks, device buffers.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

namespace vb {

// Error classes reported through the C ABI (include/varda_b200.h).
enum ErrorClass : int {
    kOk = 0,
    kInvalidArgument = 1,  // bad pointer, size or option
    kFormat = 2,           // model file / config problem (missing tensor, bad shape, unknown kind)
    kCuda = 3,             // a CUDA runtime error
    kUnsupported = 4,      // a model the kernels do not support
    kInternal = 5,         // anything else (including NCCL errors)
    kTimeout = 6,          // a bounded device-side wait gave up
};

struct Error : std::runtime_error {
    int cls;
    Error(int c, const std::string& m) : std::runtime_error(m), cls(c) {}
};

[[noreturn]] inline void fail(int cls, const std::string& msg) { throw Error(cls, msg); }

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
    if (e != cudaSuccess)
        throw Error(kCuda, std::string(what) + ": " + cudaGetErrorString(e) + " (" + file + ":" +
                               std::to_string(line) + ")");
}
#define VB_CUDA(x) ::vb::cuda_check((x), #x, __FILE__, __LINE__)

// Number of this library's kernel launches issued by the calling process (eager launches and
// launches recorded into a graph capture); read through vb_launch_count().
std::atomic<int64_t>& launch_counter();
#define VB_LAUNCH()                                                                    \
    do {                                                                               \
        ::vb::cuda_check(cudaGetLastError(), "kernel launch", __FILE__, __LINE__);     \
        ++::vb::launch_counter();                                                      \
    } while (0)

inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

// One-time setup per CUDA device, such as a kernel's function attributes (the runtime keeps them per
// device): runs f() on the first call made with the current device (devices 0..63; beyond that, on
// every call), marking the device only once f() has returned. Concurrent first calls may both run
// f(), which must be idempotent.
template <class F> void once_per_device(std::atomic<uint64_t>& done, F&& f) {
    int dev = 0;
    VB_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = dev >= 0 && dev < 64 ? uint64_t(1) << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return;
    f();
    if (bit) done.fetch_or(bit, std::memory_order_release);
}

// SM count of the current device (cached per device).
inline int device_sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    VB_CUDA(cudaGetDevice(&dev));
    int n = dev >= 0 && dev < 64 ? cache[dev].load(std::memory_order_relaxed) : 0;
    if (!n) {
        VB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Owning device allocation (cudaMalloc at load time only; never inside a forward pass).
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(size_t bytes) { alloc(bytes); }
    ~DeviceBuffer() { release(); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr, o.n_ = 0; }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
        if (this != &o) {
            release();
            p_ = o.p_, n_ = o.n_;
            o.p_ = nullptr, o.n_ = 0;
        }
        return *this;
    }
    void alloc(size_t bytes) {
        release();
        if (bytes) VB_CUDA(cudaMalloc(&p_, bytes));
        n_ = bytes;
    }
    void release() {
        if (p_) cudaFree(p_);
        p_ = nullptr;
        n_ = 0;
    }
    void* get() const { return p_; }
    size_t bytes() const { return n_; }
    template <class T> T* as() const { return static_cast<T*>(p_); }

private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

}  // namespace vb
