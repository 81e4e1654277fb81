// Test harness: the caching allocator's policy (allocator_core.h) over a fake
// device -- host memory for "device" blocks, counters for events -- so the
// bookkeeping can be checked on a machine without a GPU.  Built by
// tests/test_allocator_core.py with g++.
#include <cstdint>
#include <cstdlib>
#include <map>

#include "allocator_core.h"

namespace {

int64_t g_capacity = 1 << 30;     // bytes the fake device can hold
int64_t g_used = 0;
int64_t g_syncs = 0;
int64_t g_waits = 0;
std::map<void*, int64_t> g_sizes;
// An event is "done" once fake_complete() has been called after its record.
struct FakeEvent { bool done = true; };

struct FakeApi {
    static void* raw_alloc(size_t bytes, int) {
        if (g_used + (int64_t)bytes > g_capacity) return nullptr;
        void* p = std::malloc(bytes);
        g_used += bytes;
        g_sizes[p] = bytes;
        return p;
    }
    static void raw_free(void* p, int) {
        g_used -= g_sizes[p];
        g_sizes.erase(p);
        std::free(p);
    }
    static void* event_create(int) { return new FakeEvent(); }
    static void event_destroy(void* ev, int) { delete static_cast<FakeEvent*>(ev); }
    static void event_record(void* ev, void*, int) { static_cast<FakeEvent*>(ev)->done = false; }
    static bool event_done(void* ev, int) { return static_cast<FakeEvent*>(ev)->done; }
    static void stream_wait(void*, void*, int) { ++g_waits; }
    static void device_sync(int) { ++g_syncs; }
};

tpb::CachingAllocatorCore<FakeApi, 4>* g_alloc = nullptr;
std::map<void*, FakeEvent*> g_events;

}  // namespace

extern "C" {
void fake_reset(int64_t capacity) {
    g_alloc = new tpb::CachingAllocatorCore<FakeApi, 4>();  // leaked per test on purpose
    g_capacity = capacity;
    g_used = 0;
    g_syncs = 0;
    g_waits = 0;
}
void* fake_alloc(size_t n, int dev, void* stream) { return g_alloc->allocate(n, dev, stream); }
int fake_free(void* p, void* stream) { return g_alloc->release(p, stream) ? 0 : -1; }
void fake_stats(int dev, int64_t* out) {
    const tpb::AllocStats s = g_alloc->stats(dev);
    out[0] = s.allocated; out[1] = s.reserved; out[2] = s.peak_allocated; out[3] = s.peak_reserved;
}
void fake_reset_peak(int dev) { g_alloc->reset_peak(dev); }
void fake_empty_cache() { g_alloc->empty_cache(); }
int64_t fake_raw_allocs() { return g_alloc->raw_allocs(); }
int64_t fake_cross_waits() { return g_alloc->cross_stream_waits(); }
int64_t fake_device_syncs() { return g_syncs; }
int64_t fake_used() { return g_used; }
size_t fake_round(size_t n) { return tpb::round_request(n); }
void fake_capture_holding(int on) { g_alloc->set_capture_holding(on != 0); }
void fake_capture_freeze() { g_alloc->freeze_capture_blocks(); }
void fake_capture_drop() { g_alloc->drop_capture_blocks(); }
int64_t fake_capture_allocations() { return g_alloc->capture_allocations(); }
int64_t fake_capture_blocks() { return g_alloc->capture_blocks(); }
}
