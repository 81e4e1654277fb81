// Stream-ordered caching allocator, independent of CUDA so its bookkeeping
// can be exercised on a host without a GPU (the device calls come from the
// `Api` policy: allocator.cpp plugs in cudart, the CPU test a fake).
//
// Policy, following tensorplay-mlu's CachingAllocator
// (tensorplay_mlu/csrc/MLUAllocator.cpp:37-128):
//   * request sizes are rounded up to 512 B below 1 MiB and to 2 MiB above;
//   * a cached block is reused for a request when size <= cached <= 1.25 x size;
//   * on out-of-memory every cached block of the device is released and the
//     allocation is retried once;
//   * allocated / reserved bytes and their peaks are tracked per device.
//
// Where the reference can reuse any block at once because all work of a
// device runs on one queue, here blocks are stream-ordered: a freed block
// remembers the stream it was used on and an event recorded there at free
// time.  A request on the same stream reuses it immediately (stream order
// protects it); a request on another stream prefers a block whose event has
// completed, and otherwise takes the block and makes the new stream wait on
// that event on the device -- no host synchronisation either way.
//
// Recording (stream capture into a CUDA graph), after MLUAllocator.cpp:130-190:
// while `holding` is on, every block handed out or given back is marked
// `recorded`.  Recorded blocks are reused only by requests made during the
// same recording (the recorded work keeps its order), with no events -- an
// event recorded on a capturing stream is a graph node, not a completion the
// host can query.  When the recording ends its free blocks are frozen into
// the held list, and blocks the recorded work still uses go there when they
// are given back; the held list is released by drop_capture_blocks (after a
// device synchronisation) when the recording is dropped.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace tpb {

struct AllocStats {
    int64_t allocated = 0;
    int64_t reserved = 0;
    int64_t peak_allocated = 0;
    int64_t peak_reserved = 0;
};

constexpr size_t kSmallLimit = size_t(1) << 20;
constexpr size_t kSmallRound = 512;
constexpr size_t kLargeRound = size_t(2) << 20;

inline size_t round_request(size_t nbytes) {
    if (nbytes == 0) nbytes = 1;
    if (nbytes <= kSmallLimit) return (nbytes + kSmallRound - 1) / kSmallRound * kSmallRound;
    return (nbytes + kLargeRound - 1) / kLargeRound * kLargeRound;
}

// Api must provide (all static):
//   void* raw_alloc(size_t bytes, int dev);            // nullptr when out of memory
//   void  raw_free(void* p, int dev);
//   void* event_create(int dev);
//   void  event_destroy(void* ev, int dev);
//   void  event_record(void* ev, void* stream, int dev);
//   bool  event_done(void* ev, int dev);
//   void  stream_wait(void* stream, void* ev, int dev);
//   void  device_sync(int dev);
template <typename Api, int MaxDevices = 64>
class CachingAllocatorCore {
public:
    struct Block {
        void* ptr;
        size_t size;
        int dev;
        void* stream;   // stream the block was last used on
        void* event;    // recorded on `stream` when the block was freed
        bool in_use;
        bool recorded;  // touched by recorded (captured) work
    };

    void* allocate(size_t nbytes, int dev, void* stream) {
        const size_t size = round_request(nbytes);
        std::lock_guard<std::mutex> lock(mutex_);
        Pool& pool = pools_.at(dev);
        Block* block = holding_ ? take_cached_recording(pool, size) : take_cached(pool, size, stream);
        if (block == nullptr) {
            void* p = Api::raw_alloc(size, dev);
            if (p == nullptr && !holding_) {
                release_cached(dev);
                p = Api::raw_alloc(size, dev);
            }
            if (p == nullptr) return nullptr;
            block = new Block{p, size, dev, stream, nullptr, false, false};
            pool.stats.reserved += static_cast<int64_t>(size);
            pool.stats.peak_reserved = std::max(pool.stats.peak_reserved, pool.stats.reserved);
            ++raw_allocs_;
        }
        if (holding_) {
            block->recorded = true;
            ++capture_allocations_;
        }
        block->in_use = true;
        block->stream = stream;
        live_[block->ptr] = block;
        pool.stats.allocated += static_cast<int64_t>(block->size);
        pool.stats.peak_allocated = std::max(pool.stats.peak_allocated, pool.stats.allocated);
        return block->ptr;
    }

    // Returns false when `ptr` was not handed out by this allocator.
    bool release(void* ptr, void* stream) {
        if (ptr == nullptr) return true;
        std::lock_guard<std::mutex> lock(mutex_);
        auto it = live_.find(ptr);
        if (it == live_.end()) return false;
        Block* block = it->second;
        live_.erase(it);
        Pool& pool = pools_.at(block->dev);
        pool.stats.allocated -= static_cast<int64_t>(block->size);
        block->in_use = false;
        if (holding_) block->recorded = true;  // recorded work may still read it
        if (block->recorded) {
            if (holding_) pool.recorded_free.emplace(block->size, block);
            else held_.push_back(block);  // the recording replays over it
            return true;
        }
        if (stream != nullptr || block->stream == nullptr) block->stream = stream;
        if (block->event == nullptr) block->event = Api::event_create(block->dev);
        Api::event_record(block->event, block->stream, block->dev);
        pool.free_blocks.emplace(block->size, block);
        return true;
    }

    // Recording begins / ends (the caller starts / stops the capture).
    void set_capture_holding(bool on) {
        std::lock_guard<std::mutex> lock(mutex_);
        if (on) capture_allocations_ = 0;
        holding_ = on;
    }

    // The recording has ended: its free blocks leave the pool until it is
    // dropped.
    void freeze_capture_blocks() {
        std::lock_guard<std::mutex> lock(mutex_);
        for (Pool& pool : pools_) {
            for (auto& entry : pool.recorded_free) held_.push_back(entry.second);
            pool.recorded_free.clear();
        }
    }

    // The recording has been dropped: release what it held.
    void drop_capture_blocks() {
        std::lock_guard<std::mutex> lock(mutex_);
        if (held_.empty()) return;
        for (int dev = 0; dev < MaxDevices; ++dev) {
            for (Block* b : held_) {
                if (b->dev == dev) {
                    Api::device_sync(dev);
                    break;
                }
            }
        }
        for (Block* block : held_) {
            if (block->event != nullptr) Api::event_destroy(block->event, block->dev);
            Api::raw_free(block->ptr, block->dev);
            pools_.at(block->dev).stats.reserved -= static_cast<int64_t>(block->size);
            delete block;
        }
        held_.clear();
    }

    int64_t capture_allocations() {
        std::lock_guard<std::mutex> lock(mutex_);
        return capture_allocations_;
    }

    int64_t capture_blocks() {
        std::lock_guard<std::mutex> lock(mutex_);
        return static_cast<int64_t>(held_.size());
    }

    AllocStats stats(int dev) {
        std::lock_guard<std::mutex> lock(mutex_);
        return pools_.at(dev).stats;
    }

    void reset_peak(int dev) {
        std::lock_guard<std::mutex> lock(mutex_);
        AllocStats& s = pools_.at(dev).stats;
        s.peak_allocated = s.allocated;
        s.peak_reserved = s.reserved;
    }

    void empty_cache() {
        std::lock_guard<std::mutex> lock(mutex_);
        for (int dev = 0; dev < MaxDevices; ++dev) release_cached(dev);
    }

    int64_t raw_allocs() const { return raw_allocs_; }
    int64_t cross_stream_waits() const { return cross_stream_waits_; }

private:
    struct Pool {
        std::multimap<size_t, Block*> free_blocks;
        std::multimap<size_t, Block*> recorded_free;  // given back during a recording
        AllocStats stats;
    };

    // Caller holds mutex_.  During a recording: a block the recording gave
    // back, else a cached block whose last use has finished (no device-side
    // wait: a capture may not wait on work outside it).
    Block* take_cached_recording(Pool& pool, size_t size) {
        const size_t limit = size + size / 4;
        auto first = pool.recorded_free.lower_bound(size);
        auto last = pool.recorded_free.upper_bound(limit);
        if (first != last) {
            Block* block = first->second;
            pool.recorded_free.erase(first);
            return block;
        }
        first = pool.free_blocks.lower_bound(size);
        last = pool.free_blocks.upper_bound(limit);
        for (auto it = first; it != last; ++it) {
            if (Api::event_done(it->second->event, it->second->dev)) {
                Block* block = it->second;
                pool.free_blocks.erase(it);
                return block;
            }
        }
        return nullptr;
    }

    // Caller holds mutex_.
    Block* take_cached(Pool& pool, size_t size, void* stream) {
        const size_t limit = size + size / 4;
        auto first = pool.free_blocks.lower_bound(size);
        auto last = pool.free_blocks.upper_bound(limit);
        if (first == last) return nullptr;
        auto pick = last;
        // Same stream first: stream order already protects the block.
        for (auto it = first; it != last; ++it) {
            if (it->second->stream == stream) {
                pick = it;
                break;
            }
        }
        bool wait = false;
        if (pick == last) {
            // Another stream's block whose last use has finished...
            for (auto it = first; it != last; ++it) {
                if (Api::event_done(it->second->event, it->second->dev)) {
                    pick = it;
                    break;
                }
            }
        }
        if (pick == last) {
            // ...or else the closest fit, ordered behind its last use.
            pick = first;
            wait = true;
        }
        Block* block = pick->second;
        pool.free_blocks.erase(pick);
        if (wait) {
            Api::stream_wait(stream, block->event, block->dev);
            ++cross_stream_waits_;
        }
        return block;
    }

    // Caller holds mutex_.  Waits for the device so no queued kernel still
    // touches a block that goes back to the driver.
    void release_cached(int dev) {
        Pool& pool = pools_.at(dev);
        if (pool.free_blocks.empty()) return;
        Api::device_sync(dev);
        for (auto& entry : pool.free_blocks) {
            Block* block = entry.second;
            if (block->event != nullptr) Api::event_destroy(block->event, dev);
            Api::raw_free(block->ptr, dev);
            pool.stats.reserved -= static_cast<int64_t>(block->size);
            delete block;
        }
        pool.free_blocks.clear();
    }

    std::mutex mutex_;
    std::vector<Pool> pools_ = std::vector<Pool>(MaxDevices);
    std::unordered_map<void*, Block*> live_;
    std::vector<Block*> held_;
    bool holding_ = false;
    int64_t capture_allocations_ = 0;
    int64_t raw_allocs_ = 0;
    int64_t cross_stream_waits_ = 0;
};

}  // namespace tpb
