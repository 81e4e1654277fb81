// Shared host-side helpers of the native library: error reporting across the
// C ABI, dtype facts, stream lookup, and the shape bookkeeping (broadcast,
// dimension coalescing) every operator family does before it launches.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "tpb200.h"

namespace tpb {

// Failure inside the library; the C ABI wrappers turn it into a negative
// status and a thread-local message.
struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

std::string format(const char* fmt, ...);
void set_last_error(const std::string& message);

#define TPB_CHECK(cond, ...)                                  \
    do {                                                      \
        if (!(cond)) throw ::tpb::Error(::tpb::format(__VA_ARGS__)); \
    } while (0)

#define TPB_CUDA(expr)                                                              \
    do {                                                                            \
        const cudaError_t tpb_status_ = (expr);                                     \
        if (tpb_status_ != cudaSuccess) {                                           \
            (void)cudaGetLastError(); /* a later launch check must not see it */    \
            throw ::tpb::Error(::tpb::format("CUDA error: %s (%s) at %s:%d",        \
                                             cudaGetErrorString(tpb_status_), #expr, \
                                             __FILE__, __LINE__));                  \
        }                                                                           \
    } while (0)

// Run `body` and convert any failure into the C ABI status convention.
template <typename F>
int guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return -1;
    } catch (...) {
        set_last_error("unknown failure in the B200 backend");
        return -1;
    }
}

inline size_t dtype_size(int dtype) {
    switch (dtype) {
        case TPB_U8: case TPB_I8: case TPB_BOOL: return 1;
        case TPB_I16: case TPB_F16: case TPB_BF16: return 2;
        case TPB_I32: case TPB_F32: return 4;
        case TPB_I64: case TPB_F64: return 8;
        default: throw Error(format("unknown dtype code %d", dtype));
    }
}

inline bool is_floating(int dtype) {
    return dtype == TPB_F16 || dtype == TPB_F32 || dtype == TPB_BF16 || dtype == TPB_F64;
}

const char* dtype_name(int dtype);

// The device a pointer lives on (the current device for host pointers).
int device_of(const void* ptr);
// The stream an operator runs on: its argument as given (NULL = the CUDA
// default stream).
cudaStream_t resolve_stream(void* stream, int dev);
// The calling thread's current stream of `dev` (tp_b200_set_stream), used by
// the entry points whose reference signature carries no stream (collectives).
cudaStream_t thread_current_stream(int dev);
int num_sms(int dev);
// SMs the persistent tensor-core GEMMs size their grid to on `dev`: all of
// them unless tp_b200_set_gemm_sm_limit lowered it.
int gemm_sm_budget(int dev);
// Per-device word that kernels with bounded waits write a failure code into.
int* device_error_word(int dev);

// Make `dev` current for the guard's lifetime.
class DeviceGuard {
public:
    explicit DeviceGuard(int dev);
    ~DeviceGuard();
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int prev_;
    int cur_;
};

// A tensor's shape and per-operand strides after broadcasting, with size-1
// dimensions dropped and mergeable neighbours merged (Cnnl.cpp:127-149
// coalesce, generalised to any number of operands).  Dimension 0 is the
// outermost.
struct Layout {
    int ndim = 0;
    int64_t sizes[TPB_MAX_DIMS];
    int64_t strides[3][TPB_MAX_DIMS];  // per operand, in elements
    int64_t numel = 1;
};

int64_t numel_of(const tpb_tensor& t);
void check_tensor(const tpb_tensor* t, const char* what);
bool is_contiguous(const tpb_tensor& t);

// Strides of `t` seen with `out`'s shape (right-aligned broadcasting: size-1
// dimensions read with stride 0).  Throws when the shapes do not broadcast.
void broadcast_strides(const tpb_tensor& t, const tpb_tensor& out, int64_t* strides);

// Build the coalesced layout of `nops` operands; operand 0 defines the shape.
Layout make_layout(const tpb_tensor& out, const tpb_tensor* const* ins, int nins);

// Stream-ordered scratch memory from the caching allocator, returned to it
// when the object goes out of scope (the reference's Workspace,
// Cnnl.cpp:94-97).
class Scratch {
public:
    Scratch(size_t nbytes, int dev, cudaStream_t stream);
    ~Scratch();
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    void* get() const { return ptr_; }

private:
    void* ptr_ = nullptr;
    size_t nbytes_ = 0;
    int dev_ = 0;
    cudaStream_t stream_ = nullptr;
};

// The allocator's internal entry points (allocator.cpp).
void* cache_alloc(size_t nbytes, int dev, cudaStream_t stream);
void cache_free(void* ptr, int dev, cudaStream_t stream);

// Recording hooks of the caching allocator (graph.cpp drives them).
void capture_holding(bool on);
void freeze_capture_blocks();
void drop_capture_blocks();
int64_t capture_allocations();
int64_t capture_blocks();

// Kernels launched by this library since load (tp_b200_launch_count).
void count_launch();
void count_launches(int64_t n);
void uncount_launches(int64_t n);

// Launch-time check for the last kernel launch.
inline void check_launch(const char* what) {
    count_launch();
    const cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess) {
        throw Error(format("launching %s failed: %s", what, cudaGetErrorString(status)));
    }
}

}  // namespace tpb
