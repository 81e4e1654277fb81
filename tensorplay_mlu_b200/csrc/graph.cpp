// Recording a fixed sequence of device work and replaying it in one launch
// (tensorplay-mlu: GraphCapture.cpp:69-130 on CNRT task topologies; here CUDA
// stream capture into a graph, instantiated once, launched per replay).
//
// The stream recorded is the calling thread's current library stream of the
// device (tp_b200_set_stream), which must be a created stream: the legacy
// default stream cannot be captured.  Capture runs in relaxed mode, so the
// caching allocator may still reach cudaMalloc while recording; it marks the
// blocks it hands out then, freezes them when the recording ends and gives
// them back to the driver when the recording is dropped (allocator_core.h).
// One recording is held at a time, as in the reference.

#include <cuda_runtime.h>

#include <mutex>

#include "common.h"

using namespace tpb;

extern "C" int64_t tp_b200_launch_count();

namespace {

std::mutex g_lock;
cudaGraph_t g_graph = nullptr;
cudaGraphExec_t g_exec = nullptr;
int g_dev = -1;
cudaStream_t g_capturing = nullptr;
size_t g_kernel_nodes = 0;  // kernels one replay runs (for the launch counter)
int64_t g_launches_at_begin = 0;

}  // namespace

extern "C" {

int tp_b200_capture_ready() { return g_exec != nullptr ? 1 : 0; }

void tp_b200_capture_stats(int64_t* out) {
    out[0] = capture_allocations();
    out[1] = capture_blocks();
}

int tp_b200_capture_begin(int dev) {
    return guarded([&] {
        std::lock_guard<std::mutex> lock(g_lock);
        TPB_CHECK(g_exec == nullptr && g_graph == nullptr && g_capturing == nullptr,
                  "a recorded sequence is held already; drop it before recording another");
        DeviceGuard guard(dev);
        cudaStream_t s = thread_current_stream(dev);
        TPB_CHECK(s != nullptr && s != cudaStreamLegacy && s != cudaStreamPerThread,
                  "recording needs a created stream as the current stream of device %d "
                  "(the default stream cannot be captured)", dev);
        TPB_CUDA(cudaStreamSynchronize(s));
        TPB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
        capture_holding(true);
        g_capturing = s;
        g_dev = dev;
        g_launches_at_begin = tp_b200_launch_count();
    });
}

int tp_b200_capture_end(int dev) {
    return guarded([&] {
        std::lock_guard<std::mutex> lock(g_lock);
        TPB_CHECK(g_capturing != nullptr && g_dev == dev, "no recording is running on device %d", dev);
        DeviceGuard guard(dev);
        cudaGraph_t graph = nullptr;
        const cudaError_t status = cudaStreamEndCapture(g_capturing, &graph);
        capture_holding(false);
        g_capturing = nullptr;
        freeze_capture_blocks();
        TPB_CUDA(status);
        TPB_CHECK(graph != nullptr,
                  "the recording was invalidated; a recorded sequence holds device work only "
                  "(no host reads, synchronisation or work on other streams)");
        cudaGraphExec_t exec = nullptr;
        const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
        if (inst != cudaSuccess) {
            cudaGraphDestroy(graph);
            TPB_CUDA(inst);
        }
        g_graph = graph;
        g_exec = exec;
        // Launches counted while recording did not run; each replay runs them.
        g_kernel_nodes = static_cast<size_t>(tp_b200_launch_count() - g_launches_at_begin);
        uncount_launches(static_cast<int64_t>(g_kernel_nodes));
    });
}

int tp_b200_capture_invoke(int dev) {
    return guarded([&] {
        std::lock_guard<std::mutex> lock(g_lock);
        TPB_CHECK(g_exec != nullptr, "nothing has been recorded yet");
        TPB_CHECK(dev == g_dev, "the recording was made on device %d, not %d", g_dev, dev);
        DeviceGuard guard(dev);
        TPB_CUDA(cudaGraphLaunch(g_exec, thread_current_stream(dev)));
        count_launches(static_cast<int64_t>(g_kernel_nodes));
    });
}

int tp_b200_capture_reset() {
    return guarded([&] {
        std::lock_guard<std::mutex> lock(g_lock);
        if (g_capturing != nullptr) {  // abandon a recording that failed part-way
            DeviceGuard guard(g_dev);
            cudaGraph_t partial = nullptr;
            cudaStreamEndCapture(g_capturing, &partial);
            cudaGetLastError();
            if (partial != nullptr) cudaGraphDestroy(partial);
            capture_holding(false);
            freeze_capture_blocks();
            g_capturing = nullptr;
        }
        if (g_exec != nullptr) {
            DeviceGuard guard(g_dev);
            cudaGraphExecDestroy(g_exec);
            g_exec = nullptr;
        }
        if (g_graph != nullptr) {
            cudaGraphDestroy(g_graph);
            g_graph = nullptr;
        }
        drop_capture_blocks();
        g_dev = -1;
        g_kernel_nodes = 0;
    });
}

}  // extern "C"
