// The process-wide caching allocator over cudart, and its C ABI
// (tp_b200_malloc / tp_b200_free / memory statistics).  The caching policy
// lives in allocator_core.h.

#include <cuda_runtime.h>

#include "allocator_core.h"
#include "common.h"

namespace tpb {

namespace {

struct CudaApi {
    static void* raw_alloc(size_t bytes, int dev) {
        DeviceGuard guard(dev);
        void* p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return p;
    }
    static void raw_free(void* p, int dev) {
        DeviceGuard guard(dev);
        cudaFree(p);
    }
    static void* event_create(int dev) {
        DeviceGuard guard(dev);
        cudaEvent_t ev = nullptr;
        TPB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        return ev;
    }
    static void event_destroy(void* ev, int dev) {
        DeviceGuard guard(dev);
        cudaEventDestroy(static_cast<cudaEvent_t>(ev));
    }
    static void event_record(void* ev, void* stream, int dev) {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(ev), static_cast<cudaStream_t>(stream)));
    }
    static bool event_done(void* ev, int dev) {
        DeviceGuard guard(dev);
        const cudaError_t status = cudaEventQuery(static_cast<cudaEvent_t>(ev));
        if (status == cudaErrorNotReady) {
            cudaGetLastError();
            return false;
        }
        return status == cudaSuccess;
    }
    static void stream_wait(void* stream, void* ev, int dev) {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream),
                                     static_cast<cudaEvent_t>(ev), 0));
    }
    static void device_sync(int dev) {
        DeviceGuard guard(dev);
        cudaDeviceSynchronize();
    }
};

using Allocator = CachingAllocatorCore<CudaApi>;

Allocator& instance() {
    // Never destroyed: tensors released during interpreter teardown still
    // return their blocks here (MLUAllocator.cpp:216-222 does the same).
    static Allocator* allocator = new Allocator();
    return *allocator;
}

}  // namespace

void* cache_alloc(size_t nbytes, int dev, cudaStream_t stream) {
    void* p = instance().allocate(nbytes, dev, stream);
    if (p == nullptr) {
        const AllocStats s = instance().stats(dev);
        throw Error(format("B200 out of memory allocating %zu bytes on device %d "
                           "(%lld bytes allocated, %lld reserved by the cache)",
                           nbytes, dev, (long long)s.allocated, (long long)s.reserved));
    }
    return p;
}

void cache_free(void* ptr, int dev, cudaStream_t stream) {
    (void)dev;
    instance().release(ptr, stream);
}

void capture_holding(bool on) { instance().set_capture_holding(on); }
void freeze_capture_blocks() { instance().freeze_capture_blocks(); }
void drop_capture_blocks() { instance().drop_capture_blocks(); }
int64_t capture_allocations() { return instance().capture_allocations(); }
int64_t capture_blocks() { return instance().capture_blocks(); }

}  // namespace tpb

using namespace tpb;

extern "C" {

void* tp_b200_malloc(size_t nbytes, int dev, void* stream) {
    void* p = nullptr;
    const int status = guarded([&] { p = cache_alloc(nbytes, dev, static_cast<cudaStream_t>(stream)); });
    return status == 0 ? p : nullptr;
}

void tp_b200_free(void* ptr, size_t nbytes, int dev, void* stream) {
    (void)nbytes;
    guarded([&] {
        TPB_CHECK(instance().release(ptr, stream), "free of a pointer this allocator did not hand out");
    });
}

void tp_b200_memory_stats(int dev, int64_t out[4]) {
    const int status = guarded([&] {
        TPB_CHECK(dev >= 0 && dev < 64, "invalid device index %d", dev);
        const AllocStats s = instance().stats(dev);
        out[0] = s.allocated;
        out[1] = s.reserved;
        out[2] = s.peak_allocated;
        out[3] = s.peak_reserved;
    });
    if (status != 0) out[0] = out[1] = out[2] = out[3] = -1;
}

void tp_b200_reset_peak_memory_stats(int dev) {
    guarded([&] {
        TPB_CHECK(dev >= 0 && dev < 64, "invalid device index %d", dev);
        instance().reset_peak(dev);
    });
}

void tp_b200_empty_cache(void) {
    guarded([&] { instance().empty_cache(); });
}

}  // extern "C"
