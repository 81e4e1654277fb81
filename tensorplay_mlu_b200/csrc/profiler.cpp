// Device time for the profiler (tensorplay-mlu: MLUProfiler.cpp:20-80, the
// DeviceTimerHooks TensorPlay's profiler calls before and after each
// operation).  A timing event is recorded on the device's current library
// stream (the stream the operations run on); two records bracket an
// operation and elapsed_ms reads the time between them once the second has
// completed.
//
// Events are pooled per device: a profiling session records two per
// operation, and creating one is a driver call the dispatch path should not
// pay each time.  The pool is never destroyed (an event must not be
// destroyed while the driver tears down at exit).

#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "common.h"

using namespace tpb;

namespace {

struct PooledEvent {
    cudaEvent_t event;
    int dev;
};

std::mutex g_lock;
std::vector<PooledEvent*>* g_pool = new std::vector<PooledEvent*>();

PooledEvent* take(int dev) {
    {
        std::lock_guard<std::mutex> lock(g_lock);
        for (size_t i = g_pool->size(); i-- > 0;) {
            if ((*g_pool)[i]->dev == dev) {
                PooledEvent* e = (*g_pool)[i];
                (*g_pool)[i] = g_pool->back();
                g_pool->pop_back();
                return e;
            }
        }
    }
    DeviceGuard guard(dev);
    cudaEvent_t ev = nullptr;
    TPB_CUDA(cudaEventCreate(&ev));  // timing enabled
    return new PooledEvent{ev, dev};
}

void give_back(PooledEvent* e) {
    std::lock_guard<std::mutex> lock(g_lock);
    g_pool->push_back(e);
}

}  // namespace

extern "C" {

int tp_b200_timer_current_device(void) {
    int dev = 0;
    return cudaGetDevice(&dev) == cudaSuccess ? dev : 0;
}

// Record a timing event on `dev`'s current stream; null on failure.
void* tp_b200_timer_record(int dev) {
    PooledEvent* e = nullptr;
    const int status = guarded([&] {
        int count = 0;
        TPB_CUDA(cudaGetDeviceCount(&count));
        TPB_CHECK(dev >= 0 && dev < count, "invalid device index %d", dev);
        e = take(dev);
        DeviceGuard guard(dev);
        const cudaError_t r = cudaEventRecord(e->event, thread_current_stream(dev));
        if (r != cudaSuccess) {
            give_back(e);
            e = nullptr;
            TPB_CUDA(r);
        }
    });
    return status == 0 ? e : nullptr;
}

// Milliseconds between two records, waiting for `end`; status 0 on success.
int tp_b200_timer_elapsed_ms(void* start, void* end, float* ms) {
    return guarded([&] {
        TPB_CHECK(start != nullptr && end != nullptr && ms != nullptr, "timer: null event");
        auto* s = static_cast<PooledEvent*>(start);
        auto* e = static_cast<PooledEvent*>(end);
        TPB_CHECK(s->dev == e->dev, "timer: events of different devices");
        DeviceGuard guard(e->dev);
        TPB_CUDA(cudaEventSynchronize(e->event));
        TPB_CUDA(cudaEventElapsedTime(ms, s->event, e->event));
    });
}

// Return an event to the pool.
void tp_b200_timer_release(void* event) {
    if (event != nullptr) give_back(static_cast<PooledEvent*>(event));
}

// Events the pool holds (for tests: a session gives back what it took).
int64_t tp_b200_timer_pooled(void) {
    std::lock_guard<std::mutex> lock(g_lock);
    return static_cast<int64_t>(g_pool->size());
}

}  // extern "C"
