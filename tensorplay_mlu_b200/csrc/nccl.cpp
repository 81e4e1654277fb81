// Collectives over NCCL (NVLink 5 / NVSwitch within a node), exported with
// the argument order, codes and status convention of tensorplay-mlu's CNCL
// ABI (tensorplay_mlu/csrc/Cncl.cpp:71-387).  Each collective is enqueued on
// the calling thread's current stream of the device (tp_b200_set_stream), so
// a process group can put gradient exchange on its own stream and order it
// against compute with events.

#include <nccl.h>

#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.h"

namespace tpb {
namespace {

thread_local std::string g_nccl_error;

bool nccl_type(int code, ncclDataType_t* out) {
    switch (code) {
        case TPB_U8: *out = ncclUint8; return true;
        case TPB_I8: *out = ncclInt8; return true;
        case TPB_I32: *out = ncclInt32; return true;
        case TPB_I64: *out = ncclInt64; return true;
        case TPB_F16: *out = ncclFloat16; return true;
        case TPB_F32: *out = ncclFloat32; return true;
        case TPB_BF16: *out = ncclBfloat16; return true;
        case TPB_F64: *out = ncclFloat64; return true;
        case TPB_BOOL: *out = ncclUint8; return true;
        default: return false;  // int16 has no NCCL type
    }
}

bool nccl_op(int code, ncclRedOp_t* out) {
    switch (code) {
        case 0: *out = ncclSum; return true;
        case 1: *out = ncclProd; return true;
        case 2: *out = ncclMax; return true;
        case 3: *out = ncclMin; return true;
        default: return false;
    }
}

void check(ncclResult_t status, const char* what) {
    // A non-blocking communicator reports in-progress for enqueued work.
    if (status == ncclSuccess || status == ncclInProgress) return;
    throw Error(format("NCCL error: %s (%s)", ncclGetErrorString(status), what));
}

ncclComm_t as_comm(void* handle) {
    TPB_CHECK(handle != nullptr, "NCCL: null communicator handle");
    return static_cast<ncclComm_t>(handle);
}

ncclDataType_t type_of(int code) {
    ncclDataType_t t;
    TPB_CHECK(nccl_type(code, &t), "NCCL: unsupported data type code %d", code);
    return t;
}

ncclRedOp_t op_of(int code) {
    ncclRedOp_t o;
    TPB_CHECK(nccl_op(code, &o), "NCCL: unsupported reduction code %d", code);
    return o;
}

template <typename F>
int nccl_guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        g_nccl_error = e.what();
        set_last_error(e.what());
        return -1;
    } catch (...) {
        g_nccl_error = "unknown NCCL failure";
        return -1;
    }
}

cudaStream_t comm_stream(int dev) { return thread_current_stream(dev); }

// Communicators are created non-blocking (so creation can be bounded by a
// timeout), and a non-blocking communicator may answer a call with
// ncclInProgress; NCCL then requires polling its asynchronous state until it
// settles before the next call on it.  Inside a group the settling happens
// once, for every communicator the group touched, at group end.
thread_local int g_group_depth = 0;
thread_local std::vector<ncclComm_t> g_group_comms;
constexpr int kSettleMs = 120000;

void settle(ncclComm_t comm, const char* what) {
    ncclResult_t state = ncclInProgress;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(kSettleMs);
    while (true) {
        check(ncclCommGetAsyncError(comm, &state), "commGetAsyncError");
        if (state != ncclInProgress) break;
        if (std::chrono::steady_clock::now() > deadline) {
            throw Error(format("NCCL: %s did not settle within %d ms", what, kSettleMs));
        }
        std::this_thread::yield();
    }
    if (state != ncclSuccess) throw Error(format("NCCL error: %s (%s)", ncclGetErrorString(state), what));
}

// Issue one NCCL call on `comm`: check its status and settle it (or record
// the communicator for the enclosing group).
void run(ncclComm_t comm, ncclResult_t status, const char* what) {
    check(status, what);
    if (g_group_depth > 0) {
        g_group_comms.push_back(comm);
        return;
    }
    if (status == ncclInProgress) settle(comm, what);
}

}  // namespace
}  // namespace tpb

using namespace tpb;

extern "C" {

const char* tp_b200_nccl_last_error(void) { return g_nccl_error.c_str(); }

int tp_b200_nccl_unique_id_bytes(void) { return static_cast<int>(sizeof(ncclUniqueId)); }

int tp_b200_nccl_get_unique_id(void* out) {
    return nccl_guarded([&] {
        TPB_CHECK(out != nullptr, "NCCL: null unique-id buffer");
        check(ncclGetUniqueId(static_cast<ncclUniqueId*>(out)), "getUniqueId");
    });
}

int tp_b200_nccl_comm_init(int rank, int nranks, int dev, const void* id, void** comm_out) {
    return nccl_guarded([&] {
        TPB_CHECK(comm_out != nullptr, "NCCL: null output communicator");
        TPB_CHECK(rank >= 0 && rank < nranks, "NCCL: rank %d out of [0, %d)", rank, nranks);
        TPB_CHECK(id != nullptr, "NCCL: null unique id");
        DeviceGuard guard(dev);
        ncclComm_t comm = nullptr;
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof(uid));
        check(ncclCommInitRank(&comm, nranks, uid, rank), "commInitRank");
        *comm_out = comm;
    });
}

int tp_b200_nccl_comm_init_timeout(int rank, int nranks, int dev, const void* id, int timeout_ms,
                                   void** comm_out) {
    return tp_b200_nccl_comm_init_ctas(rank, nranks, dev, id, timeout_ms, 0, 0, comm_out);
}

int tp_b200_nccl_comm_init_ctas(int rank, int nranks, int dev, const void* id, int timeout_ms, int min_ctas,
                                int max_ctas, void** comm_out) {
    return nccl_guarded([&] {
        TPB_CHECK(min_ctas >= 0 && max_ctas >= 0 && (max_ctas == 0 || min_ctas <= max_ctas),
                  "NCCL: invalid CTA bounds [%d, %d]", min_ctas, max_ctas);
        TPB_CHECK(comm_out != nullptr, "NCCL: null output communicator");
        TPB_CHECK(rank >= 0 && rank < nranks, "NCCL: rank %d out of [0, %d)", rank, nranks);
        TPB_CHECK(id != nullptr, "NCCL: null unique id");
        DeviceGuard guard(dev);
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof(uid));
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        config.blocking = 0;
        if (min_ctas > 0) config.minCTAs = min_ctas;
        if (max_ctas > 0) config.maxCTAs = max_ctas;
        ncclComm_t comm = nullptr;
        ncclResult_t status = ncclCommInitRankConfig(&comm, nranks, uid, rank, &config);
        const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
        while (status == ncclInProgress) {
            if (std::chrono::steady_clock::now() > deadline) {
                ncclCommAbort(comm);
                throw Error(format("NCCL: communicator of rank %d/%d not ready after %d ms "
                                   "(a peer did not join)", rank, nranks, timeout_ms));
            }
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
            if (ncclCommGetAsyncError(comm, &status) != ncclSuccess) break;
        }
        if (status != ncclSuccess) {
            if (comm != nullptr) ncclCommAbort(comm);
            check(status, "commInitRankConfig");
        }
        *comm_out = comm;
    });
}

int tp_b200_nccl_comm_destroy(void* handle) {
    return nccl_guarded([&] {
        ncclComm_t comm = as_comm(handle);
        check(ncclCommFinalize(comm), "commFinalize");
        ncclResult_t status = ncclInProgress;
        while (status == ncclInProgress) {
            if (ncclCommGetAsyncError(comm, &status) != ncclSuccess) break;
            if (status == ncclInProgress) std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
        check(ncclCommDestroy(comm), "commDestroy");
    });
}

int tp_b200_nccl_comm_abort(void* handle) {
    return nccl_guarded([&] { check(ncclCommAbort(as_comm(handle)), "commAbort"); });
}

int tp_b200_nccl_comm_rank(void* handle, int* rank_out) {
    return nccl_guarded([&] { check(ncclCommUserRank(as_comm(handle), rank_out), "commUserRank"); });
}

int tp_b200_nccl_comm_count(void* handle, int* count_out) {
    return nccl_guarded([&] { check(ncclCommCount(as_comm(handle), count_out), "commCount"); });
}

int tp_b200_nccl_comm_check(void* handle) {
    return nccl_guarded([&] {
        ncclResult_t status = ncclSuccess;
        check(ncclCommGetAsyncError(as_comm(handle), &status), "commGetAsyncError");
        check(status, "asynchronous communicator error");
    });
}

int tp_b200_nccl_all_reduce(const void* send, void* recv, size_t count, int dtype, int op, int dev,
                            void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        const ncclRedOp_t o = op_of(op);
        DeviceGuard guard(dev);
        run(c, ncclAllReduce(send, recv, count, t, o, c, comm_stream(dev)), "allReduce");
    });
}

int tp_b200_nccl_broadcast(const void* send, void* recv, size_t count, int dtype, int root, int dev,
                           void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        DeviceGuard guard(dev);
        run(c, ncclBroadcast(send, recv, count, t, root, c, comm_stream(dev)), "broadcast");
    });
}

int tp_b200_nccl_reduce(const void* send, void* recv, size_t count, int dtype, int op, int root, int dev,
                        void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        const ncclRedOp_t o = op_of(op);
        DeviceGuard guard(dev);
        run(c, ncclReduce(send, recv, count, t, o, root, c, comm_stream(dev)), "reduce");
    });
}

int tp_b200_nccl_all_gather(const void* send, void* recv, size_t count, int dtype, int dev, void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        DeviceGuard guard(dev);
        run(c, ncclAllGather(send, recv, count, t, c, comm_stream(dev)), "allGather");
    });
}

int tp_b200_nccl_reduce_scatter(const void* send, void* recv, size_t count, int dtype, int op, int dev,
                                void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        const ncclRedOp_t o = op_of(op);
        DeviceGuard guard(dev);
        run(c, ncclReduceScatter(send, recv, count, t, o, c, comm_stream(dev)), "reduceScatter");
    });
}

// Even split of `count` elements per rank, as pairwise send/recv in one group.
int tp_b200_nccl_all_to_all(const void* send, void* recv, size_t count, int dtype, int dev, void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        DeviceGuard guard(dev);
        int n = 0;
        check(ncclCommCount(c, &n), "commCount");
        const size_t es = dtype_size(dtype);
        cudaStream_t s = comm_stream(dev);
        check(ncclGroupStart(), "groupStart");
        for (int peer = 0; peer < n; ++peer) {
            check(ncclSend(static_cast<const char*>(send) + peer * count * es, count, t, peer, c, s), "send");
            check(ncclRecv(static_cast<char*>(recv) + peer * count * es, count, t, peer, c, s), "recv");
        }
        run(c, ncclGroupEnd(), "allToAll");
    });
}

int tp_b200_nccl_send(const void* buf, size_t count, int dtype, int peer, int dev, void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        DeviceGuard guard(dev);
        run(c, ncclSend(buf, count, t, peer, c, comm_stream(dev)), "send");
    });
}

int tp_b200_nccl_recv(void* buf, size_t count, int dtype, int peer, int dev, void* comm) {
    return nccl_guarded([&] {
        ncclComm_t c = as_comm(comm);
        const ncclDataType_t t = type_of(dtype);
        DeviceGuard guard(dev);
        run(c, ncclRecv(buf, count, t, peer, c, comm_stream(dev)), "recv");
    });
}

int tp_b200_nccl_group_start(void) {
    return nccl_guarded([&] {
        check(ncclGroupStart(), "groupStart");
        ++g_group_depth;
    });
}

int tp_b200_nccl_group_end(void) {
    return nccl_guarded([&] {
        if (g_group_depth > 0) --g_group_depth;
        const ncclResult_t status = ncclGroupEnd();
        check(status, "groupEnd");
        if (g_group_depth == 0) {
            std::vector<ncclComm_t> comms;
            comms.swap(g_group_comms);
            for (ncclComm_t c : comms) settle(c, "groupEnd");
        }
    });
}

int tp_b200_nccl_synchronize(int dev) {
    return nccl_guarded([&] {
        DeviceGuard guard(dev);
        TPB_CUDA(cudaStreamSynchronize(comm_stream(dev)));
    });
}

int tp_b200_nccl_queue_idle(int dev) {
    int result = -1;
    const int status = nccl_guarded([&] {
        DeviceGuard guard(dev);
        const cudaError_t s = cudaStreamQuery(comm_stream(dev));
        if (s == cudaSuccess) {
            result = 1;
        } else if (s == cudaErrorNotReady) {
            cudaGetLastError();
            result = 0;
        } else {
            TPB_CUDA(s);
        }
    });
    return status < 0 ? status : result;
}

}  // extern "C"
