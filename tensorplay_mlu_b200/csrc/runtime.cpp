// Device and stream management, copies, error surface, and the shape
// bookkeeping shared by the operator families.
//
// tensorplay-mlu keeps one queue per device and orders everything on it
// (tensorplay_mlu/csrc/MLURuntime.cpp:81-93).  Here the "queue" is a CUDA
// stream chosen per calling thread (default: the legacy default stream, the
// one PyTorch starts on), so kernels, copies and allocator reuse keep program
// order, and a host framework can move work to other streams explicitly.

#include <cuda_runtime.h>

#include <cstdlib>

#include <algorithm>
#include <array>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.h"

namespace tpb {

namespace {

constexpr int kMaxDevices = 64;
thread_local std::string g_last_error;
thread_local std::array<cudaStream_t, kMaxDevices> g_streams{};

// One device word per device that kernels with bounded waits write a failure
// code into (see tp_b200_take_device_error).
std::array<std::atomic<int*>, kMaxDevices> g_error_words{};
std::mutex g_error_lock;

std::array<std::atomic<int>, kMaxDevices> g_sms{};
// SMs the persistent GEMM kernels may occupy per device (0: all of them).
std::array<std::atomic<int>, kMaxDevices> g_gemm_sms{};
std::atomic<int64_t> g_launches{0};

}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
bool pdl_enabled() {
    static const bool on = std::getenv("TPB200_NO_PDL") == nullptr;
    return on;
}
void count_launches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void uncount_launches(int64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }

std::string format(const char* fmt, ...) {
    char buf[1024];
    va_list args;
    va_start(args, fmt);
    vsnprintf(buf, sizeof(buf), fmt, args);
    va_end(args);
    return std::string(buf);
}

void set_last_error(const std::string& message) { g_last_error = message; }

const char* dtype_name(int dtype) {
    switch (dtype) {
        case TPB_U8: return "uint8";
        case TPB_I8: return "int8";
        case TPB_I16: return "int16";
        case TPB_I32: return "int32";
        case TPB_I64: return "int64";
        case TPB_F16: return "float16";
        case TPB_F32: return "float32";
        case TPB_BF16: return "bfloat16";
        case TPB_F64: return "float64";
        case TPB_BOOL: return "bool";
        default: return "unknown";
    }
}

int device_of(const void* ptr) {
    cudaPointerAttributes attr;
    if (ptr != nullptr && cudaPointerGetAttributes(&attr, ptr) == cudaSuccess &&
        attr.type == cudaMemoryTypeDevice) {
        return attr.device;
    }
    cudaGetLastError();
    int dev = 0;
    TPB_CUDA(cudaGetDevice(&dev));
    return dev;
}

cudaStream_t resolve_stream(void* stream, int dev) {
    (void)dev;
    // An operator's stream argument is taken as given: NULL is the CUDA
    // default stream, which is also the handle PyTorch reports for its
    // default stream.
    return static_cast<cudaStream_t>(stream);
}

cudaStream_t thread_current_stream(int dev) {
    TPB_CHECK(dev >= 0 && dev < kMaxDevices, "invalid device index %d", dev);
    return g_streams[dev];
}

int num_sms(int dev) {
    int n = g_sms[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        TPB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        g_sms[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

int gemm_sm_budget(int dev) {
    const int all = num_sms(dev);
    const int limit = g_gemm_sms[dev].load(std::memory_order_relaxed);
    return limit > 0 && limit < all ? limit : all;
}

DeviceGuard::DeviceGuard(int dev) : prev_(0), cur_(dev) {
    TPB_CUDA(cudaGetDevice(&prev_));
    if (cur_ != prev_) TPB_CUDA(cudaSetDevice(cur_));
}

DeviceGuard::~DeviceGuard() {
    if (cur_ != prev_) cudaSetDevice(prev_);
}

int* device_error_word(int dev) {
    int* word = g_error_words[dev].load(std::memory_order_acquire);
    if (word != nullptr) return word;
    std::lock_guard<std::mutex> lock(g_error_lock);
    word = g_error_words[dev].load(std::memory_order_relaxed);
    if (word == nullptr) {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaMalloc(&word, sizeof(int)));
        TPB_CUDA(cudaMemset(word, 0, sizeof(int)));
        g_error_words[dev].store(word, std::memory_order_release);
    }
    return word;
}

int64_t numel_of(const tpb_tensor& t) {
    int64_t n = 1;
    for (int i = 0; i < t.ndim; ++i) n *= t.sizes[i];
    return n;
}

void check_tensor(const tpb_tensor* t, const char* what) {
    TPB_CHECK(t != nullptr, "%s: null tensor descriptor", what);
    TPB_CHECK(t->ndim >= 0 && t->ndim <= TPB_MAX_DIMS, "%s: %d dimensions (at most %d)", what,
              t->ndim, TPB_MAX_DIMS);
    dtype_size(t->dtype);
    for (int i = 0; i < t->ndim; ++i) {
        TPB_CHECK(t->sizes[i] >= 0, "%s: negative size %lld", what, (long long)t->sizes[i]);
    }
    TPB_CHECK(t->data != nullptr || numel_of(*t) == 0, "%s: null data pointer", what);
}

bool is_contiguous(const tpb_tensor& t) {
    int64_t expected = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        if (t.sizes[i] == 1) continue;
        if (t.strides[i] != expected) return false;
        expected *= t.sizes[i];
    }
    return true;
}

void broadcast_strides(const tpb_tensor& t, const tpb_tensor& out, int64_t* strides) {
    TPB_CHECK(t.ndim <= out.ndim, "operand has more dimensions (%d) than the result (%d)", t.ndim,
              out.ndim);
    const int off = out.ndim - t.ndim;
    for (int i = 0; i < out.ndim; ++i) {
        if (i < off) {
            strides[i] = 0;
            continue;
        }
        const int64_t s = t.sizes[i - off];
        TPB_CHECK(s == out.sizes[i] || s == 1,
                  "shape mismatch: operand size %lld cannot broadcast to %lld at dimension %d",
                  (long long)s, (long long)out.sizes[i], i);
        strides[i] = (s == 1 && out.sizes[i] != 1) ? 0 : t.strides[i - off];
    }
}

Layout make_layout(const tpb_tensor& out, const tpb_tensor* const* ins, int nins) {
    TPB_CHECK(nins <= 2, "at most two inputs");
    const int nops = nins + 1;
    int64_t st[3][TPB_MAX_DIMS];
    for (int i = 0; i < out.ndim; ++i) st[0][i] = out.strides[i];
    for (int k = 0; k < nins; ++k) broadcast_strides(*ins[k], out, st[k + 1]);
    Layout L;
    L.numel = numel_of(out);
    // Walk from the innermost dimension outwards, merging a dimension into
    // the running one when every operand steps through it contiguously.
    int nd = 0;
    int64_t sizes[TPB_MAX_DIMS];
    int64_t strides[3][TPB_MAX_DIMS];
    for (int i = out.ndim - 1; i >= 0; --i) {
        const int64_t s = out.sizes[i];
        if (s == 1) continue;
        if (nd > 0) {
            bool merge = true;
            for (int k = 0; k < nops; ++k) {
                if (st[k][i] != strides[k][nd - 1] * sizes[nd - 1]) merge = false;
            }
            if (merge) {
                sizes[nd - 1] *= s;
                continue;
            }
        }
        sizes[nd] = s;
        for (int k = 0; k < nops; ++k) strides[k][nd] = st[k][i];
        ++nd;
    }
    // Store outermost first.
    L.ndim = nd;
    for (int i = 0; i < nd; ++i) {
        L.sizes[i] = sizes[nd - 1 - i];
        for (int k = 0; k < 3; ++k) L.strides[k][i] = k < nops ? strides[k][nd - 1 - i] : 0;
    }
    return L;
}

Scratch::Scratch(size_t nbytes, int dev, cudaStream_t stream)
    : nbytes_(nbytes), dev_(dev), stream_(stream) {
    if (nbytes > 0) ptr_ = cache_alloc(nbytes, dev, stream);
}

Scratch::~Scratch() {
    if (ptr_ != nullptr) cache_free(ptr_, dev_, stream_);
}

}  // namespace tpb

using namespace tpb;

extern "C" {

const char* tp_b200_last_error(void) { return g_last_error.c_str(); }

int tp_b200_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return std::min(n, kMaxDevices);
}

int tp_b200_init(void) {
    try {
        const int n = tp_b200_device_count();
        for (int dev = 0; dev < n; ++dev) {
            cudaDeviceProp prop;
            TPB_CUDA(cudaGetDeviceProperties(&prop, dev));
            TPB_CHECK(prop.major == 10, "device %d (%s) is sm_%d%d; this backend is built for sm_100a",
                      dev, prop.name, prop.major, prop.minor);
        }
        return 0;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return 1;
    }
}

int tp_b200_current_device(void) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        set_last_error(cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    return dev;
}

int tp_b200_set_device(int dev) {
    return guarded([&] {
        const int n = tp_b200_device_count();
        TPB_CHECK(dev >= 0 && dev < n, "invalid device index %d (%d device(s) visible)", dev, n);
        TPB_CUDA(cudaSetDevice(dev));
    });
}

int tp_b200_capability(int dev) {
    int major = 0, minor = 0;
    const int status = guarded([&] {
        TPB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        TPB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    });
    return status < 0 ? status : major * 10 + minor;
}

int tp_b200_synchronize(int dev) {
    return guarded([&] {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaDeviceSynchronize());
    });
}

int tp_b200_set_stream(int dev, void* stream) {
    return guarded([&] {
        TPB_CHECK(dev >= 0 && dev < kMaxDevices, "invalid device index %d", dev);
        g_streams[dev] = static_cast<cudaStream_t>(stream);
    });
}

void* tp_b200_get_stream(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    return g_streams[dev];
}

int tp_b200_memcpy(void* dst, const void* src, size_t nbytes, int kind, int dev, int src_dev,
                   void* stream, int blocking) {
    return guarded([&] {
        if (nbytes == 0) return;
        TPB_CHECK(dst != nullptr && src != nullptr, "memcpy: null pointer");
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        switch (kind) {
            case 1: TPB_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice, s)); break;
            case 2: TPB_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost, s)); break;
            case 3:
                if (src_dev != dev && src_dev >= 0) {
                    TPB_CUDA(cudaMemcpyPeerAsync(dst, dev, src, src_dev, nbytes, s));
                } else {
                    TPB_CUDA(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToDevice, s));
                }
                break;
            default: TPB_CHECK(false, "memcpy: unknown copy kind %d", kind);
        }
        if (blocking) TPB_CUDA(cudaStreamSynchronize(s));
    });
}

int tp_b200_mem_get_info(int dev, size_t* free_bytes, size_t* total_bytes) {
    return guarded([&] {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaMemGetInfo(free_bytes, total_bytes));
    });
}

int64_t tp_b200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int tp_b200_set_gemm_sm_limit(int dev, int sms) {
    return guarded([&] {
        TPB_CHECK(dev >= 0 && dev < kMaxDevices, "set_gemm_sm_limit: device %d out of range", dev);
        const int all = num_sms(dev);
        // An even count (the pair kernel runs 2-SM clusters), at least one pair.
        const int v = sms <= 0 || sms >= all ? 0 : std::max(2, sms & ~1);
        g_gemm_sms[dev].store(v, std::memory_order_relaxed);
    });
}

int tp_b200_take_device_error(int dev) {
    int value = 0;
    const int status = guarded([&] {
        int* word = g_error_words[dev].load(std::memory_order_acquire);
        if (word == nullptr) return;
        DeviceGuard guard(dev);
        TPB_CUDA(cudaDeviceSynchronize());
        TPB_CUDA(cudaMemcpy(&value, word, sizeof(int), cudaMemcpyDeviceToHost));
        if (value != 0) TPB_CUDA(cudaMemset(word, 0, sizeof(int)));
    });
    return status < 0 ? status : value;
}

}  // extern "C"
