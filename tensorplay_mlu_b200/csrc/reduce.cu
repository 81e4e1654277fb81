// Reductions (sum, mean, amax, amin) and softmax / log_softmax with their
// backward kernels (tensorplay-mlu: ReduceKernels.cpp, on cnnlReduce_v2 and
// cnnlSoftmaxForward/Backward there).
//
// Reductions: the input's dimensions are split into kept and reduced ones and
// each group is coalesced.  Three kernels cover the layouts:
//   * rows: the reduced elements of one output are contiguous ([.., R]);
//     many rows take one warp each (grid-stride over rows); fewer rows take
//     one block per (row, split), 16-byte vector loads, warp-shuffle then
//     shared-memory block reduction;
//   * columns: the output index is the contiguous side ([O, R, K] over R);
//     threads own 16-byte column vectors and walk R; when the output is
//     small a block holds 8 row lanes (combined in shared memory) and the
//     rows are split over blocks;
//   * anything else is first gathered into a [kept, reduced] dense scratch
//     copy and takes the row kernel.
// Splits write per-block partials to stream-ordered scratch and a second
// pass combines them in a fixed order, so results are deterministic.
//
// Softmax: rows of up to 8192 (fp32) / 16384 (16-bit) elements stay in
// registers between the max, the sum and the write -- one read and one write
// of HBM.  With many such rows a persistent block streams them through a ring
// of shared-memory stages filled by bulk asynchronous copies (TMA), so the
// next rows' reads overlap the current row's reductions.  Longer rows use an
// online max/sum pass plus a write pass, and softmax over a non-innermost
// dimension walks columns.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <map>
#include <utility>
#include <mutex>
#include <type_traits>

#include "common.h"
#include "device.cuh"
#include "ptx.cuh"

// Completion tickets of single-row split reductions, one per (device,
// stream): the blocks of a launch count themselves in, the last one combines
// the partial results and resets its ticket to zero for the stream's next
// reduction (launches on one stream never overlap).
constexpr int kTicketSlots = 256;
static __device__ unsigned g_reduce_tickets[kTicketSlots];

namespace tpb {

void copy_impl(const tpb_tensor& dst, const tpb_tensor& src, cudaStream_t stream, int dev);

namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------ reduce algebra --

template <typename T> struct Acc { using type = int64_t; };
template <> struct Acc<float> { using type = float; };
template <> struct Acc<__half> { using type = float; };
template <> struct Acc<__nv_bfloat16> { using type = float; };
template <> struct Acc<double> { using type = double; };

template <typename A, int OP>
__device__ __forceinline__ A identity() {
    if constexpr (OP == TPB_AMAX) {
        if constexpr (std::is_integral<A>::value) return LLONG_MIN;
        else return -INFINITY;
    } else if constexpr (OP == TPB_AMIN) {
        if constexpr (std::is_integral<A>::value) return LLONG_MAX;
        else return INFINITY;
    } else {
        return A(0);
    }
}

template <typename A, int OP>
__device__ __forceinline__ A combine(A a, A b) {
    if constexpr (OP == TPB_AMAX) return max_nan(a, b);
    else if constexpr (OP == TPB_AMIN) return min_nan(a, b);
    else return a + b;
}

// One input element into an accumulator: combine(acc, widen(x)).  Sums of
// 16-bit floats use sm_100's mixed-precision add (add.rn.f32.bf16 / .f16:
// the widening is exact and the add rounds once, so the result is that of
// widen-then-add) -- one instruction instead of two.
template <typename A, int OP, typename T>
__device__ __forceinline__ A fold(A acc, T x) {
    if constexpr (OP == TPB_SUM || OP == TPB_MEAN) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            asm("add.rn.f32.bf16 %0, %1, %0;" : "+f"(acc) : "h"(__bfloat16_as_ushort(x)));
            return acc;
        } else if constexpr (std::is_same<T, __half>::value) {
            asm("add.rn.f32.f16 %0, %1, %0;" : "+f"(acc) : "h"(__half_as_ushort(x)));
            return acc;
        }
    }
    return combine<A, OP>(acc, load_as<A>(x));
}

// A 16-byte vector into an accumulator, elements in order.  max / min of
// 16-bit floats fold the vector pairwise in the input type first (exact and
// NaN-propagating, two lanes per instruction) and widen only the last pair.
template <typename A, int OP, typename T, int V>
__device__ __forceinline__ A fold_vec(A acc, const Vec<T, V>& v) {
    constexpr bool narrow = std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value;
    if constexpr ((OP == TPB_AMAX || OP == TPB_AMIN) && narrow && V == 8) {
        using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
        const T2* p = reinterpret_cast<const T2*>(v.v);
        T2 m;
        if constexpr (OP == TPB_AMAX) m = __hmax2_nan(__hmax2_nan(p[0], p[1]), __hmax2_nan(p[2], p[3]));
        else m = __hmin2_nan(__hmin2_nan(p[0], p[1]), __hmin2_nan(p[2], p[3]));
        return combine<A, OP>(combine<A, OP>(acc, load_as<A>(m.x)), load_as<A>(m.y));
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) acc = fold<A, OP>(acc, v.v[j]);
        return acc;
    }
}

// Four vectors into four accumulators.  Sums interleave the accumulators
// element by element (four independent add chains in flight); max / min
// fold each vector pairwise first.
template <typename A, int OP, typename T, int V>
__device__ __forceinline__ void fold4(A& a0, A& a1, A& a2, A& a3, const Vec<T, V>& a, const Vec<T, V>& b,
                                      const Vec<T, V>& c, const Vec<T, V>& d) {
    if constexpr (OP == TPB_SUM || OP == TPB_MEAN) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            a0 = fold<A, OP>(a0, a.v[j]);
            a1 = fold<A, OP>(a1, b.v[j]);
            a2 = fold<A, OP>(a2, c.v[j]);
            a3 = fold<A, OP>(a3, d.v[j]);
        }
    } else {
        a0 = fold_vec<A, OP>(a0, a);
        a1 = fold_vec<A, OP>(a1, b);
        a2 = fold_vec<A, OP>(a2, c);
        a3 = fold_vec<A, OP>(a3, d);
    }
}

template <typename A, int OP>
__device__ __forceinline__ A warp_combine(A v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = combine<A, OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide combine; the result is valid in thread 0.
template <typename A, int OP>
__device__ __forceinline__ A block_combine(A v) {
    __shared__ A warp_vals[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_combine<A, OP>(v);
    __syncthreads();
    if (lane == 0) warp_vals[warp] = v;
    __syncthreads();
    const int nwarps = (blockDim.x + 31) >> 5;
    if (warp == 0) {
        v = lane < nwarps ? warp_vals[lane] : identity<A, OP>();
        v = warp_combine<A, OP>(v);
    }
    return v;
}

// Store an accumulator into any output type (float accumulators into
// integer outputs truncate; int64 accumulators into floating outputs round).
template <typename To, typename A>
__device__ __forceinline__ To cvt_store(A v) {
    if constexpr (std::is_same<To, __half>::value || std::is_same<To, __nv_bfloat16>::value) {
        return store_as<To, float>(static_cast<float>(v));
    } else if constexpr (std::is_same<To, bool>::value) {
        return v != A(0);
    } else {
        return static_cast<To>(v);
    }
}

template <typename To, typename A, int OP>
__device__ __forceinline__ To finalize(A v, double count) {
    if constexpr (OP == TPB_MEAN) {
        if constexpr (std::is_integral<A>::value) return cvt_store<To>(static_cast<double>(v) / count);
        else return cvt_store<To>(v / static_cast<A>(count));
    } else {
        return cvt_store<To>(v);
    }
}

// -------------------------------------------------------- row reduce --

// rows x R, row r starting at x + row_off(r), elements contiguous.  Block b
// handles row b / splits as split b % splits: the row's 16-byte vectors are
// dealt out in an interleaved (grid-stride) order -- split s takes vectors
// s * kThreads + t, + splits * kThreads, ... -- so at any moment the blocks
// of a row sweep neighbouring memory, and every split gets the same share to
// within one vector per thread.  Split 0 also takes the scalar head (before
// the first 16-byte boundary) and tail.
template <typename T, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_rows(const T* __restrict__ x, To* __restrict__ out,
                                                        typename Acc<T>::type* __restrict__ partial,
                                                        OffsetCalc<1> rows_calc, int64_t R, int splits,
                                                        double count, unsigned* __restrict__ ticket) {
    pdl_entry();
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    using VT = Vec<T, V>;
    const int64_t row = blockIdx.x / splits;
    const int split = blockIdx.x % splits;
    int64_t off;
    rows_calc.get(static_cast<uint32_t>(row), &off);
    const T* base = x + off;
    A acc0 = identity<A, OP>(), acc1 = identity<A, OP>(), acc2 = identity<A, OP>(),
      acc3 = identity<A, OP>();
    const int64_t mis = static_cast<int64_t>(reinterpret_cast<uintptr_t>(base) & 15u);
    int64_t head = mis == 0 ? 0 : (16 - mis) / static_cast<int64_t>(sizeof(T));
    if (head > R) head = R;
    if (split == 0 && threadIdx.x < head) acc0 = combine<A, OP>(acc0, load_as<A>(base[threadIdx.x]));
    const int64_t nvec = (R - head) / V;
    const VT* vp = reinterpret_cast<const VT*>(base + head);
    // Eight 16-byte loads in flight per thread while at least eight
    // vectors remain (a full-tensor reduction runs as one wave of blocks,
    // each with tens of vectors per thread: four in flight left it
    // latency-bound), then four.
    const int64_t S = int64_t(splits) * kThreads;
    int64_t v = int64_t(split) * kThreads + threadIdx.x;
    for (; v + 7 * S < nvec; v += 8 * S) {
        const VT a = vp[v];
        const VT b = vp[v + S];
        const VT c = vp[v + 2 * S];
        const VT d = vp[v + 3 * S];
        const VT e = vp[v + 4 * S];
        const VT f = vp[v + 5 * S];
        const VT g = vp[v + 6 * S];
        const VT h = vp[v + 7 * S];
        fold4<A, OP>(acc0, acc1, acc2, acc3, a, b, c, d);
        fold4<A, OP>(acc0, acc1, acc2, acc3, e, f, g, h);
    }
    if (v + 3 * S < nvec) {
        const VT a = vp[v];
        const VT b = vp[v + S];
        const VT c = vp[v + 2 * S];
        const VT d = vp[v + 3 * S];
        fold4<A, OP>(acc0, acc1, acc2, acc3, a, b, c, d);
        v += 4 * S;
    }
    // The last (at most three) vectors of this thread, loaded together
    // rather than one round trip each.
    if (v < nvec) {
        const bool h1 = v + S < nvec, h2 = v + 2 * S < nvec;
        const VT a = vp[v];
        VT b, c;
        if (h1) b = vp[v + S];
        if (h2) c = vp[v + 2 * S];
        acc0 = fold_vec<A, OP>(acc0, a);
        if (h1) acc1 = fold_vec<A, OP>(acc1, b);
        if (h2) acc2 = fold_vec<A, OP>(acc2, c);
    }
    if (split == 0) {
        for (int64_t k = head + nvec * V + threadIdx.x; k < R; k += kThreads) {
            acc1 = combine<A, OP>(acc1, load_as<A>(base[k]));
        }
    }
    A acc = block_combine<A, OP>(combine<A, OP>(combine<A, OP>(acc0, acc1), combine<A, OP>(acc2, acc3)));
    if (threadIdx.x == 0) {
        if (splits == 1) out[row] = finalize<To, A, OP>(acc, count);
        else partial[row * splits + split] = acc;
    }
    if (ticket == nullptr) return;
    // One row split over the grid: the last block to finish combines the
    // partials, in the same order as reduce_row_partials (so the result does
    // not depend on which block is last).
    __shared__ bool last;
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(ticket, 1u) == static_cast<unsigned>(splits - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    A a = identity<A, OP>();
    for (int s = threadIdx.x; s < splits; s += kThreads) a = combine<A, OP>(a, __ldcg(partial + s));
    a = block_combine<A, OP>(a);
    if (threadIdx.x == 0) {
        out[0] = finalize<To, A, OP>(a, count);
        *ticket = 0u;
    }
}

// Many rows, none split: one warp per row, rows taken in a grid-stride loop,
// so an SM streams rows back to back with no block-wide barrier between them
// (a block per short row spends most of its life in launch, barriers and
// teardown).  Four 16-byte loads in flight per lane.
constexpr int kWarpsPerBlock = kThreads / 32;

template <typename T, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_rows_warp(const T* __restrict__ x, To* __restrict__ out,
                                                             OffsetCalc<1> rows_calc, int64_t rows,
                                                             int64_t R, double count) {
    pdl_entry();
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    using VT = Vec<T, V>;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = int64_t(gridDim.x) * kWarpsPerBlock;
    for (int64_t row = int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5); row < rows; row += nwarps) {
        int64_t off;
        rows_calc.get(static_cast<uint32_t>(row), &off);
        const T* base = x + off;
        A acc0 = identity<A, OP>(), acc1 = identity<A, OP>(), acc2 = identity<A, OP>(),
          acc3 = identity<A, OP>();
        // Elements before the first 16-byte boundary (fewer than V).
        const int64_t mis = static_cast<int64_t>(reinterpret_cast<uintptr_t>(base) & 15u);
        int64_t head = mis == 0 ? 0 : (16 - mis) / static_cast<int64_t>(sizeof(T));
        if (head > R) head = R;
        if (lane < head) acc0 = combine<A, OP>(acc0, load_as<A>(base[lane]));
        const int64_t nvec = (R - head) / V;
        const VT* vp = reinterpret_cast<const VT*>(base + head);
        int64_t v = lane;
        for (; v + 96 < nvec; v += 128) {
            const VT a = vp[v];
            const VT b = vp[v + 32];
            const VT c = vp[v + 64];
            const VT d = vp[v + 96];
            fold4<A, OP>(acc0, acc1, acc2, acc3, a, b, c, d);
        }
        // The last (at most three) vectors, loaded together.
        if (v < nvec) {
            const bool h1 = v + 32 < nvec, h2 = v + 64 < nvec;
            const VT a = vp[v];
            VT b, c;
            if (h1) b = vp[v + 32];
            if (h2) c = vp[v + 64];
            acc1 = fold_vec<A, OP>(acc1, a);
            if (h1) acc2 = fold_vec<A, OP>(acc2, b);
            if (h2) acc3 = fold_vec<A, OP>(acc3, c);
        }
        for (int64_t k = head + nvec * V + lane; k < R; k += 32) {
            acc2 = combine<A, OP>(acc2, load_as<A>(base[k]));
        }
        const A acc = warp_combine<A, OP>(combine<A, OP>(combine<A, OP>(acc0, acc1), combine<A, OP>(acc2, acc3)));
        if (lane == 0) out[row] = finalize<To, A, OP>(acc, count);
    }
}

// Rows streamed through shared memory: work items are (row, chunk of
// kChunkBytes), a persistent block takes items blockIdx.x, +gridDim.x, ...
// with kReduceStages of them in flight as bulk asynchronous copies (TMA), so
// reads continue while the block combines.  A row of one chunk is written
// to `out`; longer rows leave one partial per chunk for the second pass.
// Rows start on 16-byte boundaries; a chunk's last (< 16) bytes are read
// from global memory directly.  Waits are bounded as in the softmax ring.
constexpr uint32_t kChunkBytes = 16384;
constexpr int kReduceStages = 4;
constexpr int kErrReduceRing = 0x7c12;

template <typename T>
__device__ __forceinline__ void issue_chunk(const T* x, int64_t item, int64_t n_chunks, int64_t R,
                                            int64_t row_stride, int64_t chunk, uint32_t dst, uint32_t bar) {
    const int64_t row = item / n_chunks, c = item % n_chunks;
    const int64_t e0 = c * chunk;
    const int64_t n = R - e0 < chunk ? R - e0 : chunk;
    const uint32_t bytes = static_cast<uint32_t>(n * int64_t(sizeof(T))) & ~15u;
    if (bytes != 0) {
        mbar_expect_tx(bar, bytes);
        bulk_load(dst, x + row * row_stride + e0, bytes, bar);
    } else {
        mbar_arrive(bar);  // nothing to copy: complete the phase
    }
}

template <typename T, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_rows_ring(const T* __restrict__ x, To* __restrict__ out,
                                                             typename Acc<T>::type* __restrict__ partial,
                                                             int64_t rows, int64_t R, int64_t row_stride,
                                                             int64_t chunk, int64_t n_chunks, double count,
                                                             int* err) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    using VT = Vec<T, V>;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t full[kReduceStages];
    __shared__ volatile int gave_up;
    const int64_t items = rows * n_chunks;
    const int64_t first = blockIdx.x, stride = gridDim.x;
    if (threadIdx.x == 0) {
        gave_up = 0;
        for (int s = 0; s < kReduceStages; ++s) mbar_init(smem_addr(&full[s]), 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kReduceStages; ++s) {
            const int64_t item = first + int64_t(s) * stride;
            if (item >= items) break;
            issue_chunk(x, item, n_chunks, R, row_stride, chunk, smem_addr(ring + size_t(s) * kChunkBytes),
                        smem_addr(&full[s]));
        }
    }
    int it = 0, s = 0;
    uint32_t parity = 0;
    for (int64_t item = first; item < items; item += stride, ++it) {
        if (!mbar_wait_bounded(smem_addr(&full[s]), parity)) {
            gave_up = 1;
            atomicExch(err, kErrReduceRing);
        }
        const int64_t row = item / n_chunks, c = item % n_chunks;
        const int64_t e0 = c * chunk;
        const int64_t n = R - e0 < chunk ? R - e0 : chunk;
        const int64_t nvec = (n * int64_t(sizeof(T)) / 16);
        const VT* sv = reinterpret_cast<const VT*>(ring + size_t(s) * kChunkBytes);
        A acc0 = identity<A, OP>(), acc1 = identity<A, OP>(), acc2 = identity<A, OP>(),
          acc3 = identity<A, OP>();
        int64_t v = threadIdx.x;
        for (; v + 3 * kThreads < nvec; v += 4 * kThreads) {
            const VT a = sv[v];
            const VT b = sv[v + kThreads];
            const VT cc = sv[v + 2 * kThreads];
            const VT d = sv[v + 3 * kThreads];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                acc0 = combine<A, OP>(acc0, load_as<A>(a.v[j]));
                acc1 = combine<A, OP>(acc1, load_as<A>(b.v[j]));
                acc2 = combine<A, OP>(acc2, load_as<A>(cc.v[j]));
                acc3 = combine<A, OP>(acc3, load_as<A>(d.v[j]));
            }
        }
        for (; v < nvec; v += kThreads) {
            const VT a = sv[v];
#pragma unroll
            for (int j = 0; j < V; ++j) acc0 = combine<A, OP>(acc0, load_as<A>(a.v[j]));
        }
        const T* g = x + row * row_stride + e0;
        for (int64_t k = nvec * V + threadIdx.x; k < n; k += kThreads) {
            acc1 = combine<A, OP>(acc1, load_as<A>(g[k]));
        }
        const A acc = block_combine<A, OP>(combine<A, OP>(combine<A, OP>(acc0, acc1), combine<A, OP>(acc2, acc3)));
        // Every thread has read stage s (block_combine's barriers): refill it.
        if (threadIdx.x == 0) {
            const int64_t next = item + int64_t(kReduceStages) * stride;
            if (next < items && !gave_up) {
                issue_chunk(x, next, n_chunks, R, row_stride, chunk, smem_addr(ring + size_t(s) * kChunkBytes),
                            smem_addr(&full[s]));
            }
            if (n_chunks == 1) out[row] = finalize<To, A, OP>(acc, count);
            else partial[item] = acc;
        }
        if (gave_up) break;
        if (++s == kReduceStages) {
            s = 0;
            parity ^= 1u;
        }
    }
    if (threadIdx.x == 0 && gave_up) {
        for (int k = 0; k < kReduceStages; ++k) {
            const int j = it + k;
            if (first + int64_t(j) * stride >= items) break;
            mbar_wait_bounded(smem_addr(&full[j % kReduceStages]), static_cast<uint32_t>(j / kReduceStages) & 1u);
        }
    }
}

// One block per row: combine `splits` partials in index order.
template <typename A, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_row_partials(const A* __restrict__ partial,
                                                                To* __restrict__ out, int splits,
                                                                double count) {
    pdl_entry();
    const int64_t row = blockIdx.x;
    A acc = identity<A, OP>();
    for (int s = threadIdx.x; s < splits; s += kThreads) {
        acc = combine<A, OP>(acc, partial[row * splits + s]);
    }
    acc = block_combine<A, OP>(acc);
    if (threadIdx.x == 0) out[row] = finalize<To, A, OP>(acc, count);
}

// ----------------------------------------------------- column reduce --

// x viewed as [O, R, K]: offset o*os + r*rs + k (k contiguous).  A block is
// CX = kThreads / RL column vectors (V elements each) by RL row lanes; grid
// (ceil(K / (V * CX)), O, splits).  Row lane l = split * RL + ry of the
// grid's splits * RL lanes walks rows l, l + lanes, ... (neighbouring lanes
// read neighbouring rows), four rows in flight in two accumulator chains.
// With RL > 1 the block's lanes are combined in shared memory in lane
// order, so each block leaves one partial per column.
template <typename T, typename To, int OP, int V, int RL>
__global__ void __launch_bounds__(kThreads) reduce_cols(const T* __restrict__ x, To* __restrict__ out,
                                                        typename Acc<T>::type* __restrict__ partial,
                                                        int64_t O, int64_t R, int64_t K, int64_t os,
                                                        int64_t rs, double count) {
    pdl_entry();
    using A = typename Acc<T>::type;
    using VT = Vec<T, V>;
    constexpr int CX = kThreads / RL;
    const int cx = RL == 1 ? static_cast<int>(threadIdx.x) : static_cast<int>(threadIdx.x % CX);
    const int ry = RL == 1 ? 0 : static_cast<int>(threadIdx.x / CX);
    const int64_t kv = int64_t(blockIdx.x) * CX + cx;
    const bool active = kv * V < K;
    if (RL == 1 && !active) return;
    const int64_t o = blockIdx.y;
    const int split = blockIdx.z;
    const int splits = gridDim.z;
    const int64_t lanes = int64_t(splits) * RL;
    A acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = identity<A, OP>();
    if (active) {
        // Four rows in flight; the V column accumulators are independent
        // chains already, so one set of accumulators (fewer registers, more
        // resident blocks).
        const T* p = x + o * os + kv * V;
        const int64_t step = lanes * rs;
        int64_t r = int64_t(split) * RL + ry;
        for (; r + 3 * lanes < R; r += 4 * lanes) {
            const T* q = p + r * rs;
            const VT a = *reinterpret_cast<const VT*>(q);
            const VT b = *reinterpret_cast<const VT*>(q + step);
            const VT c = *reinterpret_cast<const VT*>(q + 2 * step);
            const VT d = *reinterpret_cast<const VT*>(q + 3 * step);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = fold<A, OP>(acc[j], a.v[j]);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = fold<A, OP>(acc[j], b.v[j]);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = fold<A, OP>(acc[j], c.v[j]);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = fold<A, OP>(acc[j], d.v[j]);
        }
        for (; r < R; r += lanes) {
            const VT a = *reinterpret_cast<const VT*>(p + r * rs);
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = fold<A, OP>(acc[j], a.v[j]);
        }
    }
    if constexpr (RL > 1) {
        __shared__ A lane_acc[RL - 1][V][CX];
        if (ry > 0) {
#pragma unroll
            for (int j = 0; j < V; ++j) lane_acc[ry - 1][j][cx] = acc[j];
        }
        __syncthreads();
        if (ry != 0 || !active) return;
#pragma unroll
        for (int l = 0; l < RL - 1; ++l)
#pragma unroll
            for (int j = 0; j < V; ++j) acc[j] = combine<A, OP>(acc[j], lane_acc[l][j][cx]);
    }
    if (splits == 1) {
#pragma unroll
        for (int j = 0; j < V; ++j) out[o * K + kv * V + j] = finalize<To, A, OP>(acc[j], count);
    } else {
        A* dst = partial + (int64_t(split) * O + o) * K + kv * V;
#pragma unroll
        for (int j = 0; j < V; ++j) dst[j] = acc[j];
    }
}

template <typename A, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_col_partials(const A* __restrict__ partial,
                                                                To* __restrict__ out, int64_t n,
                                                                int splits, double count) {
    pdl_entry();
    // Block = 32 columns x 8 split lanes: lane y combines splits y, y+8, ...
    // (two independent chains), then lane 0 combines the 8 lane results in
    // order -- a fixed order, so results are deterministic.
    __shared__ A lanes[8][33];
    const int x = threadIdx.x & 31, y = threadIdx.x >> 5;
    const int64_t i = int64_t(blockIdx.x) * 32 + x;
    A a0 = identity<A, OP>(), a1 = identity<A, OP>();
    if (i < n) {
        int s = y;
        for (; s + 8 < splits; s += 16) {
            a0 = combine<A, OP>(a0, partial[int64_t(s) * n + i]);
            a1 = combine<A, OP>(a1, partial[int64_t(s + 8) * n + i]);
        }
        if (s < splits) a0 = combine<A, OP>(a0, partial[int64_t(s) * n + i]);
    }
    lanes[y][x] = combine<A, OP>(a0, a1);
    __syncthreads();
    if (y == 0 && i < n) {
        A acc = lanes[0][x];
#pragma unroll
        for (int k = 1; k < 8; ++k) acc = combine<A, OP>(acc, lanes[k][x]);
        out[i] = finalize<To, A, OP>(acc, count);
    }
}

// ------------------------------------------------------------- softmax --

// exp / log of the softmax family.  16-bit outputs (rounded to 8 or 11
// mantissa bits) use the hardware ex2/lg2 approximations; fp32 / fp64 the
// accurate functions.
template <typename T, typename C>
__device__ __forceinline__ C sm_exp(C x) {
    if constexpr (std::is_same<C, double>::value) return exp(x);
    else if constexpr (sizeof(T) == 2) return __expf(x);
    else return expf(x);
}
template <typename T, typename C>
__device__ __forceinline__ C sm_log(C x) {
    if constexpr (std::is_same<C, double>::value) return log(x);
    else if constexpr (sizeof(T) == 2) return __logf(x);
    else return logf(x);
}

template <typename C>
__device__ __forceinline__ C block_max(C v) { return block_combine<C, TPB_AMAX>(v); }
template <typename C>
__device__ __forceinline__ C block_sum(C v) { return block_combine<C, TPB_SUM>(v); }

// Broadcast thread 0's value to the block.
template <typename C>
__device__ __forceinline__ C block_bcast(C v) {
    __shared__ C slot;
    __syncthreads();
    if (threadIdx.x == 0) slot = v;
    __syncthreads();
    return slot;
}

// exp(v - m).  For 16-bit outputs: one FFMA and one ex2.approx on
// v * log2(e) - m * log2(e) (ml2 = m * log2(e), computed once per row).
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T, typename C>
__device__ __forceinline__ C sm_exp_shift(C v, C m, C ml2) {
    if constexpr (sizeof(T) == 2) return ex2_approx(fmaf(v, kLog2e, -ml2));
    else return sm_exp<T>(v - m);
}

// Softmax of one row of D elements held by the block: VPT vectors of V
// elements per thread stay in registers between the max, the sum and the
// write.  `after_read()` runs once every thread has read its elements (the
// first block reduction's barriers have passed).
template <typename T, int V, int VPT, int THREADS, bool LOG, typename AfterRead>
__device__ __forceinline__ void softmax_row(const T* __restrict__ xr, T* __restrict__ yr, int64_t D,
                                            AfterRead after_read) {
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    C v[VPT][V];
    C m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            unpack_vec(*reinterpret_cast<const VT*>(xr + idx), v[k]);
#pragma unroll
            for (int j = 0; j < V; ++j) m = max_nan(m, v[k][j]);
        } else {
#pragma unroll
            for (int j = 0; j < V; ++j) v[k][j] = -INFINITY;
        }
    }
    m = block_bcast(block_max(m));
    after_read();
    const C ml2 = m * C(kLog2e);
    C s = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const C e = sm_exp_shift<T>(v[k][j], m, ml2);
            s += e;
            if constexpr (!LOG) v[k][j] = e;
        }
    }
    s = block_bcast(block_sum(s));
    if constexpr (LOG) {
        // (v - m) - log(s): two roundings of small numbers, not one of m + log(s).
        const C lse = sm_log<T>(s);
#pragma unroll
        for (int k = 0; k < VPT; ++k)
#pragma unroll
            for (int j = 0; j < V; ++j) v[k][j] = (v[k][j] - m) - lse;
    } else {
        const C inv = C(1) / s;
#pragma unroll
        for (int k = 0; k < VPT; ++k)
#pragma unroll
            for (int j = 0; j < V; ++j) v[k][j] *= inv;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            VT o;
            pack_vec(v[k], o);
            *reinterpret_cast<VT*>(yr + idx) = o;
        }
    }
}

// One block per row (V = 1 when the row is not vector-aligned).
template <typename T, int V, int VPT, int THREADS, bool LOG>
__global__ void __launch_bounds__(THREADS) softmax_rows_reg(const T* __restrict__ x, T* __restrict__ y,
                                                            int64_t D) {
    pdl_entry();
    const int64_t row = blockIdx.x;
    softmax_row<T, V, VPT, THREADS, LOG>(x + row * D, y + row * D, D, [] {});
}

// Many rows that fit in registers: a persistent block walks rows
// blockIdx.x, +gridDim.x, ... with `stages` of them in flight as bulk copies
// into shared memory (one mbarrier per stage), so HBM reads continue while
// the block's max / sum / write of the current row run.  Thread 0 refills a
// stage as soon as the first block reduction shows every thread has read it.
// A wait that gives up (kWaitNs) records kErrSoftmaxRing in the device error
// word; the block then finishes the row it is on, drains the copies it issued
// and returns.
constexpr int kMaxRingStages = 8;
constexpr int kErrSoftmaxRing = 0x7c11;

template <typename T, int V, int VPT, int THREADS, bool LOG>
__global__ void __launch_bounds__(THREADS) softmax_rows_ring(const T* __restrict__ x, T* __restrict__ y,
                                                             int64_t rows, int64_t D, int stages, int* err) {
    pdl_entry();
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t full[kMaxRingStages];
    __shared__ volatile int gave_up;
    const uint32_t row_bytes = static_cast<uint32_t>(D * sizeof(T));
    const uint32_t stage_bytes = (row_bytes + 127u) & ~127u;
    const int64_t first = blockIdx.x, stride = gridDim.x;
    if (threadIdx.x == 0) {
        gave_up = 0;
        for (int s = 0; s < stages; ++s) mbar_init(smem_addr(&full[s]), 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            const int64_t r = first + int64_t(s) * stride;
            if (r >= rows) break;
            mbar_expect_tx(smem_addr(&full[s]), row_bytes);
            bulk_load(smem_addr(ring + size_t(s) * stage_bytes), x + r * D, row_bytes, smem_addr(&full[s]));
        }
    }
    int it = 0;
    int s = 0;
    uint32_t parity = 0;
    for (int64_t r = first; r < rows; r += stride, ++it) {
        if (!mbar_wait_bounded(smem_addr(&full[s]), parity)) {
            gave_up = 1;
            atomicExch(err, kErrSoftmaxRing);
        }
        const T* xs = reinterpret_cast<const T*>(ring + size_t(s) * stage_bytes);
        const int64_t next = r + int64_t(stages) * stride;
        const int stage = s;
        softmax_row<T, V, VPT, THREADS, LOG>(xs, y + r * D, D, [&] {
            // Every thread has read stage `stage`: refill it.
            if (threadIdx.x == 0 && next < rows && !gave_up) {
                mbar_expect_tx(smem_addr(&full[stage]), row_bytes);
                bulk_load(smem_addr(ring + size_t(stage) * stage_bytes), x + next * D, row_bytes,
                          smem_addr(&full[stage]));
            }
        });
        // gave_up was set before the block reductions' barriers: uniform.
        if (gave_up) break;
        if (++s == stages) {
            s = 0;
            parity ^= 1u;
        }
    }
    // After giving up, wait (bounded) for the copies still in flight so none
    // lands in shared memory after the block has left.  Those are the
    // iterations it .. it + stages - 1 (the refill of iteration it was
    // skipped).
    if (threadIdx.x == 0 && gave_up) {
        for (int k = 0; k < stages; ++k) {
            const int j = it + k;
            if (first + int64_t(j) * stride >= rows) break;
            mbar_wait_bounded(smem_addr(&full[j % stages]), static_cast<uint32_t>(j / stages) & 1u);
        }
    }
}

// Rows too long for registers: online max/sum (one read), then the write.
template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_rows_online(const T* __restrict__ x, T* __restrict__ y,
                                                                int64_t D, bool log) {
    using C = typename Compute<T>::type;
    const int64_t row = blockIdx.x;
    const T* xr = x + row * D;
    T* yr = y + row * D;
    C m = -INFINITY, s = 0;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const C v = load_as<C>(xr[i]);
        if (v > m) {
            s = s * sm_exp<T>(m - v) + C(1);
            m = v;
        } else if (v != v) {
            m = v;
        } else {
            s += sm_exp<T>(v - m);
        }
    }
    const C gm = block_bcast(block_max(m));
    s = (m == -INFINITY) ? C(0) : s * sm_exp<T>(m - gm);
    s = block_bcast(block_sum(s));
    const C inv = C(1) / s, lse = sm_log<T>(s);
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const C v = load_as<C>(xr[i]);
        yr[i] = store_as<T>(log ? v - gm - lse : sm_exp<T>(v - gm) * inv);
    }
}

// Softmax over a non-innermost dimension: x is [outer, D, inner]; one thread
// per (outer, inner) column.
template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_cols(const T* __restrict__ x, T* __restrict__ y,
                                                         int64_t outer, int64_t D, int64_t inner, bool log) {
    using C = typename Compute<T>::type;
    const int64_t n = outer * inner;
    for (int64_t t = int64_t(blockIdx.x) * kThreads + threadIdx.x; t < n;
         t += int64_t(gridDim.x) * kThreads) {
        const int64_t o = t / inner, i = t - o * inner;
        const T* xc = x + o * D * inner + i;
        T* yc = y + o * D * inner + i;
        C m = -INFINITY, s = 0;
        for (int64_t d = 0; d < D; ++d) {
            const C v = load_as<C>(xc[d * inner]);
            if (v > m) {
                s = s * sm_exp<T>(m - v) + C(1);
                m = v;
            } else if (v != v) {
                m = v;
            } else {
                s += sm_exp<T>(v - m);
            }
        }
        const C inv = C(1) / s, lse = sm_log<T>(s);
        for (int64_t d = 0; d < D; ++d) {
            const C v = load_as<C>(xc[d * inner]);
            yc[d * inner] = store_as<T>(log ? v - m - lse : sm_exp<T>(v - m) * inv);
        }
    }
}

// Backward, rows in registers: softmax dx = y * (dy - sum(dy * y));
// log_softmax dx = dy - exp(y) * sum(dy).
template <typename T, int V, int VPT, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_bwd_rows_reg(const T* __restrict__ dy, const T* __restrict__ y,
                                                                T* __restrict__ dx, int64_t D, bool log) {
    pdl_entry();
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    const int64_t row = blockIdx.x;
    C g[VPT][V], o[VPT][V];
    C acc = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            const VT a = *reinterpret_cast<const VT*>(dy + row * D + idx);
            const VT b = *reinterpret_cast<const VT*>(y + row * D + idx);
#pragma unroll
            for (int j = 0; j < V; ++j) {
                g[k][j] = load_as<C>(a.v[j]);
                o[k][j] = load_as<C>(b.v[j]);
                acc += log ? g[k][j] : g[k][j] * o[k][j];
            }
        }
    }
    acc = block_bcast(block_sum(acc));
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            VT r;
#pragma unroll
            for (int j = 0; j < V; ++j) {
                r.v[j] = store_as<T>(log ? g[k][j] - sm_exp<T>(o[k][j]) * acc : o[k][j] * (g[k][j] - acc));
            }
            *reinterpret_cast<VT*>(dx + row * D + idx) = r;
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_bwd_rows_loop(const T* __restrict__ dy, const T* __restrict__ y,
                                                                  T* __restrict__ dx, int64_t D, bool log) {
    using C = typename Compute<T>::type;
    const int64_t row = blockIdx.x;
    C acc = 0;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const C g = load_as<C>(dy[row * D + i]);
        acc += log ? g : g * load_as<C>(y[row * D + i]);
    }
    acc = block_bcast(block_sum(acc));
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const C g = load_as<C>(dy[row * D + i]);
        const C o = load_as<C>(y[row * D + i]);
        dx[row * D + i] = store_as<T>(log ? g - sm_exp<T>(o) * acc : o * (g - acc));
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_bwd_cols(const T* __restrict__ dy, const T* __restrict__ y,
                                                             T* __restrict__ dx, int64_t outer, int64_t D,
                                                             int64_t inner, bool log) {
    using C = typename Compute<T>::type;
    const int64_t n = outer * inner;
    for (int64_t t = int64_t(blockIdx.x) * kThreads + threadIdx.x; t < n;
         t += int64_t(gridDim.x) * kThreads) {
        const int64_t o = t / inner, i = t - o * inner;
        const int64_t base = o * D * inner + i;
        C acc = 0;
        for (int64_t d = 0; d < D; ++d) {
            const C g = load_as<C>(dy[base + d * inner]);
            acc += log ? g : g * load_as<C>(y[base + d * inner]);
        }
        for (int64_t d = 0; d < D; ++d) {
            const C g = load_as<C>(dy[base + d * inner]);
            const C w = load_as<C>(y[base + d * inner]);
            dx[base + d * inner] = store_as<T>(log ? g - sm_exp<T>(w) * acc : w * (g - acc));
        }
    }
}

// ------------------------------------------------------------ host side --

struct DimGroup {
    int n = 0;
    int64_t sizes[TPB_MAX_DIMS];
    int64_t strides[TPB_MAX_DIMS];
    int64_t numel() const {
        int64_t p = 1;
        for (int i = 0; i < n; ++i) p *= sizes[i];
        return p;
    }
    // Merge neighbours laid out back to back (outermost first).
    void coalesce() {
        int m = 0;
        for (int i = 0; i < n; ++i) {
            if (sizes[i] == 1) continue;
            if (m > 0 && strides[m - 1] == strides[i] * sizes[i]) {
                sizes[m - 1] *= sizes[i];
                strides[m - 1] = strides[i];
                continue;
            }
            sizes[m] = sizes[i];
            strides[m] = strides[i];
            ++m;
        }
        n = m;
    }
};

Layout group_layout(const DimGroup& g) {
    Layout L;
    L.ndim = g.n;
    L.numel = g.numel();
    for (int i = 0; i < g.n; ++i) {
        L.sizes[i] = g.sizes[i];
        L.strides[0][i] = g.strides[i];
        L.strides[1][i] = L.strides[2][i] = 0;
    }
    return L;
}

tpb_tensor dense_like(void* data, int dtype, int ndim, const int64_t* sizes) {
    tpb_tensor t{};
    t.data = data;
    t.dtype = dtype;
    t.ndim = ndim;
    int64_t s = 1;
    for (int i = ndim - 1; i >= 0; --i) {
        t.sizes[i] = sizes[i];
        t.strides[i] = s;
        s *= sizes[i];
    }
    return t;
}

// Column kernel: split R over blocks until the device is filled once with
// resident blocks (at least 16 rows per split, at most 1024 splits).
// Column-reduce plan.  Enough 256-vector column blocks to fill the device:
// one row lane per block, no split.  Otherwise blocks of 32 column vectors
// (one warp per row segment, whole 128-byte lines) by 8 row lanes, and the
// rows split over `splits` blocks until the device is full; the partials
// are then about (resident blocks x 32 vectors), whatever K is, instead of
// growing with K.
struct ColPlan {
    int rl;
    int64_t kblocks;
    int splits;
};
constexpr int kColLanes = 8;

template <typename T, typename To, int OP>
ColPlan plan_cols(int64_t O, int64_t R, int64_t K, bool vec, int dev, int sms) {
    constexpr int V = VecWidth<T>::value;
    static int blocks_per_sm[64] = {};
    if (blocks_per_sm[dev] == 0) {
        int n = 0;
        TPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_cols<T, To, OP, V, kColLanes>, kThreads, 0));
        blocks_per_sm[dev] = std::max(n, 1);
    }
    const int64_t cap = int64_t(sms) * blocks_per_sm[dev];
    const int64_t vecs = vec ? K / V : K;
    ColPlan p{1, (vecs + kThreads - 1) / kThreads, 1};
    if (p.kblocks * O >= cap) return p;
    constexpr int CX = kThreads / kColLanes;
    p.rl = kColLanes;
    p.kblocks = (vecs + CX - 1) / CX;
    const int64_t base = p.kblocks * O;
    if (base >= cap) return p;
    // Whole waves only: splits * base <= cap.
    const int64_t splits = std::min<int64_t>(cap / base, std::max<int64_t>(R / (16 * kColLanes), 1));
    p.splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(splits, 1024)));
    return p;
}

template <typename T, typename To, int OP>
void launch_cols(const ColPlan& plan, bool vec, const T* x, To* o, typename Acc<T>::type* partial, int64_t O,
                 int64_t R, int64_t K, int64_t os, int64_t rs, double count, cudaStream_t stream) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    dim3 grid(static_cast<unsigned>(plan.kblocks), static_cast<unsigned>(O), static_cast<unsigned>(plan.splits));
    if (plan.rl == 1) {
        if (vec) {
            launch_pdl(reduce_cols<T, To, OP, V, 1>, grid, kThreads, 0, stream, x, o, partial, O, R, K, os, rs, count);
        } else {
            launch_pdl(reduce_cols<T, To, OP, 1, 1>, grid, kThreads, 0, stream, x, o, partial, O, R, K, os, rs, count);
        }
    } else {
        if (vec) {
            launch_pdl(reduce_cols<T, To, OP, V, kColLanes>, grid, kThreads, 0, stream, x, o, partial, O, R, K, os, rs,
                       count);
        } else {
            launch_pdl(reduce_cols<T, To, OP, 1, kColLanes>, grid, kThreads, 0, stream, x, o, partial, O, R, K, os, rs,
                       count);
        }
    }
    check_launch("reduce_cols");
    if (plan.splits > 1) {
        const int64_t n = O * K;
        const unsigned g2 = static_cast<unsigned>((n + 31) / 32);
        launch_pdl(reduce_col_partials<A, To, OP>, g2, kThreads, 0, stream, partial, o, n, plan.splits, count);
        check_launch("reduce_col_partials");
    }
}

// Resident blocks of the block-per-row kernel on the whole device.
template <typename T, typename To, int OP>
int64_t rows_capacity(int dev, int sms) {
    static int blocks_per_sm[64] = {};
    if (blocks_per_sm[dev] == 0) {
        int n = 0;
        TPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, reduce_rows<T, To, OP>, kThreads, 0));
        blocks_per_sm[dev] = std::max(n, 1);
    }
    return int64_t(sms) * blocks_per_sm[dev];
}

// Whether the shared-memory ring is the default row kernel (measured
// against the block kernel on the op sweep's shapes).
constexpr bool ring_by_default() { return false; }

// The completion ticket of `stream` on `dev`, or null (two-pass combine)
// when none may be used: streams that are being captured into a graph (a
// replay could run beside the stream's own launches), the per-thread default
// stream (one handle, many streams) and more streams than slots.
std::mutex g_ticket_lock;

// Device address of the ticket array on `dev` (the caller has made `dev`
// current), looked up once per device.
unsigned* ticket_base(int dev) {
    static unsigned* base[64] = {};
    std::lock_guard<std::mutex> g(g_ticket_lock);
    if (base[dev] == nullptr) {
        void* p = nullptr;
        TPB_CUDA(cudaGetSymbolAddress(&p, g_reduce_tickets));
        base[dev] = static_cast<unsigned*>(p);
    }
    return base[dev];
}

unsigned* reduce_ticket(int dev, cudaStream_t stream) {
    if (stream == cudaStreamPerThread || dev < 0 || dev >= 64) return nullptr;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    TPB_CUDA(cudaStreamIsCapturing(stream, &cap));
    if (cap != cudaStreamCaptureStatusNone) return nullptr;
    unsigned* base = ticket_base(dev);
    static std::map<std::pair<int, cudaStream_t>, int> slots;
    static int used[64] = {};
    std::lock_guard<std::mutex> g(g_ticket_lock);
    auto it = slots.find({dev, stream});
    if (it == slots.end()) {
        if (used[dev] >= kTicketSlots) return nullptr;
        it = slots.emplace(std::make_pair(dev, stream), used[dev]++).first;
    }
    return base + it->second;
}

// Row-kernel plan.  Three kernels:
//   ring  - rows on 16-byte boundaries with a uniform row stride, at least
//           one 4 KB chunk long: streamed through shared memory by bulk
//           copies (per-chunk partials when a row spans several chunks);
//   warp  - many short rows (at most 4 KB): one warp per row;
//   block - otherwise: a block per row; fewer rows than resident blocks are
//           split into chunks (with a second pass over the partials).
// TPB200_REDUCE_ROWS=ring|warp|block forces a kernel where its layout
// conditions hold (for A/B measurements).
enum RowKernel { kRowsBlock = 0, kRowsWarp = 1, kRowsRing = 2 };

struct RowPlan {
    RowKernel kind;
    int splits;
    int64_t chunk;
    int64_t row_stride;
};

template <typename T>
RowPlan plan_rows(const T* x, const DimGroup& kept_rows, int64_t rows, int64_t R, int sms, int64_t cap) {
    constexpr int V = VecWidth<T>::value;
    static const char* force = std::getenv("TPB200_REDUCE_ROWS");
    const bool f_ring = force != nullptr && std::strcmp(force, "ring") == 0;
    const bool f_warp = force != nullptr && std::strcmp(force, "warp") == 0;
    const bool f_block = force != nullptr && std::strcmp(force, "block") == 0;
    RowPlan p{kRowsBlock, 1, R, 0};
    const int64_t row_bytes = R * int64_t(sizeof(T));
    const int64_t stride = rows == 1 || kept_rows.n == 0 ? 0 : kept_rows.n == 1 ? kept_rows.strides[0] : -1;
    const bool ring_ok = aligned16(x) && stride >= 0 && (stride * int64_t(sizeof(T))) % 16 == 0 &&
                         row_bytes >= 4096;
    if (ring_ok && (f_ring || (!f_warp && !f_block && ring_by_default()))) {
        p.kind = kRowsRing;
        p.chunk = kChunkBytes / sizeof(T);
        p.splits = static_cast<int>((R + p.chunk - 1) / p.chunk);
        p.row_stride = stride;
        return p;
    }
    if (f_warp || (!f_block && row_bytes <= 4096 && rows >= int64_t(sms) * 32)) {
        p.kind = kRowsWarp;
        return p;
    }
    // Fewer rows than resident blocks (`cap`): split each row over enough
    // blocks to fill the device once (the interleaved sweep keeps the splits
    // equal), each split keeping at least four vectors per thread.
    if (rows < cap) {
        p.splits = static_cast<int>(std::min<int64_t>((cap + rows - 1) / rows,
                                                      std::max<int64_t>(R / (kThreads * V * 4), 1)));
    }
    return p;
}

template <typename T, typename To, int OP>
void launch_rows(const RowPlan& p, const T* x, To* o, typename Acc<T>::type* partial,
                 const OffsetCalc<1>& calc, int64_t rows, int64_t R, double count, int dev, int sms,
                 cudaStream_t stream) {
    using A = typename Acc<T>::type;
    if (p.kind == kRowsWarp) {
        const unsigned grid = static_cast<unsigned>(
            std::min<int64_t>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock, int64_t(sms) * 8));
        launch_pdl(reduce_rows_warp<T, To, OP>, grid, kThreads, 0, stream, x, o, calc, rows, R, count);
        check_launch("reduce_rows_warp");
        return;
    }
    if (p.kind == kRowsRing) {
        auto kern = reduce_rows_ring<T, To, OP>;
        constexpr size_t smem = size_t(kReduceStages) * kChunkBytes;
        static int blocks_per_sm[64] = {};
        if (blocks_per_sm[dev] == 0) {
            TPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
            int n = 0;
            TPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem));
            blocks_per_sm[dev] = std::max(n, 1);
        }
        const int64_t items = rows * p.splits;
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, int64_t(sms) * blocks_per_sm[dev]));
        kern<<<grid, kThreads, smem, stream>>>(x, o, partial, rows, R, p.row_stride, p.chunk, p.splits, count,
                                               device_error_word(dev));
        check_launch("reduce_rows_ring");
    } else {
        unsigned* ticket = rows == 1 && p.splits > 1 ? reduce_ticket(dev, stream) : nullptr;
        launch_pdl(reduce_rows<T, To, OP>, static_cast<unsigned>(rows * p.splits), kThreads, 0, stream, x, o, partial,
                   calc, R, p.splits, count, ticket);
        check_launch("reduce_rows");
        if (ticket != nullptr) return;
    }
    if (p.splits > 1) {
        launch_pdl(reduce_row_partials<A, To, OP>, static_cast<unsigned>(rows), kThreads, 0, stream, partial, o,
                   p.splits, count);
        check_launch("reduce_row_partials");
    }
}

template <typename T, typename To, int OP>
void reduce_launch(const tpb_tensor& out, const tpb_tensor& xin, uint32_t mask, int dev,
                   cudaStream_t stream) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    const int sms = num_sms(dev);
    DimGroup kept, red;
    for (int i = 0; i < xin.ndim; ++i) {
        DimGroup& g = (mask >> i) & 1 ? red : kept;
        g.sizes[g.n] = xin.sizes[i];
        g.strides[g.n] = xin.strides[i];
        ++g.n;
    }
    const int64_t rows = kept.numel();
    const int64_t R = red.numel();
    if (R == 1) {
        copy_impl(out, xin, stream, dev);
        return;
    }
    kept.coalesce();
    red.coalesce();
    To* o = static_cast<To*>(out.data);
    const double count = static_cast<double>(R);
    const T* x = static_cast<const T*>(xin.data);

    // Column layout: [O, R, K] with K the unit-stride kept side.
    const bool cols = red.n == 1 && kept.n >= 1 && kept.n <= 2 && kept.strides[kept.n - 1] == 1 &&
                      red.strides[0] != 1;
    if (cols) {
        const int64_t K = kept.sizes[kept.n - 1];
        const int64_t O = kept.n == 2 ? kept.sizes[0] : 1;
        const int64_t os = kept.n == 2 ? kept.strides[0] : 0;
        const int64_t rs = red.strides[0];
        const bool vec = K % V == 0 && rs % V == 0 && os % V == 0 && aligned16(x);
        if (O < 65536) {
            const ColPlan plan = plan_cols<T, To, OP>(O, R, K, vec, dev, sms);
            Scratch partial(plan.splits > 1 ? sizeof(A) * plan.splits * O * K : 0, dev, stream);
            launch_cols<T, To, OP>(plan, vec, x, o, static_cast<A*>(partial.get()), O, R, K, os, rs, count, stream);
            return;
        }
    }

    // Row layout needs the reduced elements contiguous.
    const bool rows_ok = red.n == 0 || (red.n == 1 && red.strides[0] == 1);
    Scratch gathered(rows_ok ? 0 : sizeof(T) * rows * R, dev, stream);
    DimGroup kept_rows = kept;
    if (!rows_ok) {
        // Dense [kept..., reduced...] copy, then rows of R contiguous elements.
        tpb_tensor src{};
        src.data = const_cast<T*>(x);
        src.dtype = xin.dtype;
        int nd = 0;
        int64_t sizes[TPB_MAX_DIMS];
        for (int pass = 0; pass < 2; ++pass) {
            for (int i = 0; i < xin.ndim; ++i) {
                const bool r = (mask >> i) & 1;
                if (r != (pass == 1)) continue;
                src.sizes[nd] = xin.sizes[i];
                src.strides[nd] = xin.strides[i];
                sizes[nd] = xin.sizes[i];
                ++nd;
            }
        }
        src.ndim = nd;
        const tpb_tensor dst = dense_like(gathered.get(), xin.dtype, nd, sizes);
        copy_impl(dst, src, stream, dev);
        x = static_cast<const T*>(gathered.get());
        kept_rows.n = 1;
        kept_rows.sizes[0] = rows;
        kept_rows.strides[0] = R;
    }
    TPB_CHECK(rows < (int64_t(1) << 31), "reduce: %lld output elements exceed the row kernel's limit",
              (long long)rows);
    const int which[1] = {0};
    const auto calc = OffsetCalc<1>::make(group_layout(kept_rows), which);
    const RowPlan plan = plan_rows<T>(x, kept_rows, rows, R, sms, rows_capacity<T, To, OP>(dev, sms));
    Scratch partial(plan.splits > 1 ? sizeof(A) * rows * plan.splits : 0, dev, stream);
    launch_rows<T, To, OP>(plan, x, o, static_cast<A*>(partial.get()), calc, rows, R, count, dev, sms, stream);
}

template <typename A> struct AccCode;
template <> struct AccCode<float> { static constexpr int value = TPB_F32; };
template <> struct AccCode<double> { static constexpr int value = TPB_F64; };
template <> struct AccCode<int64_t> { static constexpr int value = TPB_I64; };

// Results are written in the input's dtype or in the accumulator's; any other
// requested dtype is reduced into an accumulator-typed buffer and converted.
template <typename T, int OP>
void reduce_out_dispatch(const tpb_tensor& out, const tpb_tensor& x, uint32_t mask, int dev,
                         cudaStream_t stream) {
    using A = typename Acc<T>::type;
    if (out.dtype == x.dtype) {
        reduce_launch<T, T, OP>(out, x, mask, dev, stream);
    } else if (out.dtype == AccCode<A>::value) {
        reduce_launch<T, A, OP>(out, x, mask, dev, stream);
    } else {
        Scratch buf(sizeof(A) * numel_of(out), dev, stream);
        const tpb_tensor tmp = dense_like(buf.get(), AccCode<A>::value, out.ndim, out.sizes);
        reduce_launch<T, A, OP>(tmp, x, mask, dev, stream);
        copy_impl(out, tmp, stream, dev);
    }
}

template <typename T>
void reduce_op_dispatch(int op, const tpb_tensor& out, const tpb_tensor& x, uint32_t mask, int dev,
                        cudaStream_t stream) {
    switch (op) {
        case TPB_SUM: reduce_out_dispatch<T, TPB_SUM>(out, x, mask, dev, stream); break;
        case TPB_MEAN: reduce_out_dispatch<T, TPB_MEAN>(out, x, mask, dev, stream); break;
        case TPB_AMAX: reduce_launch<T, T, TPB_AMAX>(out, x, mask, dev, stream); break;
        case TPB_AMIN: reduce_launch<T, T, TPB_AMIN>(out, x, mask, dev, stream); break;
        default: TPB_CHECK(false, "reduce: unknown op %d", op);
    }
}

// Which row kernel: the shared-memory ring for many rows of 16-bit
// elements (whose per-row work is short next to the HBM latency), the
// one-block-per-row kernel otherwise.  TPB200_SOFTMAX=ring|reg overrides the
// choice (for A/B measurements).
bool use_softmax_ring(size_t elem_size, int64_t rows, int dev) {
    static const char* force = std::getenv("TPB200_SOFTMAX");
    if (rows < int64_t(num_sms(dev)) * 2) return false;
    if (force != nullptr && std::strcmp(force, "ring") == 0) return true;
    if (force != nullptr && std::strcmp(force, "reg") == 0) return false;
    return elem_size == 2;
}

// About 48 KB of rows per block in the ring (at least two stages): with the
// blocks an SM holds that keeps 100+ KB of reads in flight per SM.
constexpr uint32_t kRingBytes = 48 * 1024;
constexpr int kRingMaxSmem = 64 * 1024;  // two stages of a 32 KB row

template <typename T, int V, int VPT, int THREADS, bool LOG>
void launch_ring(T* y, const T* x, int64_t rows, int64_t D, int dev, cudaStream_t stream) {
    auto kern = softmax_rows_ring<T, V, VPT, THREADS, LOG>;
    const uint32_t stage_bytes = (static_cast<uint32_t>(D * sizeof(T)) + 127u) & ~127u;
    const int stages = std::max(2, std::min<int>(kMaxRingStages, static_cast<int>(kRingBytes / stage_bytes)));
    const size_t smem = size_t(stages) * stage_bytes;
    TPB_CHECK(smem <= size_t(kRingMaxSmem), "softmax: ring of %zu bytes", smem);
    static int blocks_per_sm[64][kMaxRingStages + 1] = {};
    int& nb = blocks_per_sm[dev][stages];
    if (nb == 0) {
        TPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRingMaxSmem));
        int n = 0;
        TPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, THREADS, smem));
        nb = std::max(n, 1);
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, int64_t(num_sms(dev)) * nb));
    launch_pdl(kern, grid, THREADS, smem, stream, x, y, rows, D, stages, device_error_word(dev));
    check_launch("softmax_rows_ring");
}

// Row kernels by row length: VPT vectors per thread of a 256- or 512-thread
// block; rows longer than 2048 vectors take the online two-pass kernel.
template <typename T, bool LOG>
void softmax_rows_launch(T* y, const T* x, int64_t rows, int64_t D, int dev, cudaStream_t stream) {
    constexpr int V = VecWidth<T>::value;
    const unsigned grid = static_cast<unsigned>(rows);
    const bool vec = D % V == 0 && aligned16(x) && aligned16(y);
    const int64_t nv = D / V;
    if (vec && nv <= 2048 && use_softmax_ring(sizeof(T), rows, dev)) {
        // 4096-wide 16-bit rows: 128-thread blocks, 32 elements per thread.
        // Same-box A/B ([32768, 4096] bf16, six ring stages): 128 threads
        // 0.87-0.89 of the HBM copy peak, 256 threads 0.81-0.83, 512
        // threads 0.64 -- the per-row block reductions' barriers, not
        // occupancy, set the rate; shallower rings (3-4 stages) lost
        // whatever the block size.  A persistent warp-per-row kernel (row
        // in registers, shuffle-only reductions, no block barrier) measured
        // 0.77 against 0.93 for this kernel on one box and was not kept.
        if (nv <= 256) launch_ring<T, V, 1, 256, LOG>(y, x, rows, D, dev, stream);
        else if (nv <= 512) launch_ring<T, V, 4, 128, LOG>(y, x, rows, D, dev, stream);
        else if (nv <= 1024) launch_ring<T, V, 4, 256, LOG>(y, x, rows, D, dev, stream);
        else launch_ring<T, V, 4, 512, LOG>(y, x, rows, D, dev, stream);
        return;
    }
    if (vec && nv <= 2048) {
        if (nv <= 256) launch_pdl(softmax_rows_reg<T, V, 1, 256, LOG>, grid, 256, 0, stream, x, y, D);
        else if (nv <= 512) launch_pdl(softmax_rows_reg<T, V, 2, 256, LOG>, grid, 256, 0, stream, x, y, D);
        else if (nv <= 1024) launch_pdl(softmax_rows_reg<T, V, 4, 256, LOG>, grid, 256, 0, stream, x, y, D);
        else launch_pdl(softmax_rows_reg<T, V, 4, 512, LOG>, grid, 512, 0, stream, x, y, D);
    } else if (!vec && D <= 1024) {
        launch_pdl(softmax_rows_reg<T, 1, 4, 256, LOG>, grid, 256, 0, stream, x, y, D);
    } else {
        softmax_rows_online<T><<<grid, kThreads, 0, stream>>>(x, y, D, LOG);
    }
    check_launch("softmax_rows");
}

template <typename T>
void softmax_launch(bool log, T* y, const T* x, int64_t outer, int64_t D, int64_t inner, int dev,
                    cudaStream_t stream) {
    if (inner != 1) {
        const int64_t n = outer * inner;
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks_for(n, kThreads), num_sms(dev) * 16));
        softmax_cols<T><<<grid, kThreads, 0, stream>>>(x, y, outer, D, inner, log);
        check_launch("softmax_cols");
        return;
    }
    TPB_CHECK(outer < (int64_t(1) << 31), "softmax: too many rows");
    if (log) softmax_rows_launch<T, true>(y, x, outer, D, dev, stream);
    else softmax_rows_launch<T, false>(y, x, outer, D, dev, stream);
}

template <typename T>
void softmax_bwd_launch(bool log, T* dx, const T* dy, const T* y, int64_t outer, int64_t D,
                        int64_t inner, int dev, cudaStream_t stream) {
    if (inner != 1) {
        const int64_t n = outer * inner;
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks_for(n, kThreads), num_sms(dev) * 16));
        softmax_bwd_cols<T><<<grid, kThreads, 0, stream>>>(dy, y, dx, outer, D, inner, log);
        check_launch("softmax_bwd_cols");
        return;
    }
    constexpr int V = VecWidth<T>::value;
    const unsigned rows = static_cast<unsigned>(outer);
    const bool vec = D % V == 0 && aligned16(dx) && aligned16(dy) && aligned16(y);
    if (vec) {
        const int64_t nv = D / V;
        if (nv <= 256) launch_pdl(softmax_bwd_rows_reg<T, V, 1, 256>, rows, 256, 0, stream, dy, y, dx, D, log);
        else if (nv <= 512) launch_pdl(softmax_bwd_rows_reg<T, V, 2, 256>, rows, 256, 0, stream, dy, y, dx, D, log);
        else if (nv <= 1024) launch_pdl(softmax_bwd_rows_reg<T, V, 4, 256>, rows, 256, 0, stream, dy, y, dx, D, log);
        else if (nv <= 2048) launch_pdl(softmax_bwd_rows_reg<T, V, 4, 512>, rows, 512, 0, stream, dy, y, dx, D, log);
        else softmax_bwd_rows_loop<T><<<rows, kThreads, 0, stream>>>(dy, y, dx, D, log);
    } else if (D <= 1024) {
        launch_pdl(softmax_bwd_rows_reg<T, 1, 4, 256>, rows, 256, 0, stream, dy, y, dx, D, log);
    } else {
        softmax_bwd_rows_loop<T><<<rows, kThreads, 0, stream>>>(dy, y, dx, D, log);
    }
    check_launch("softmax_bwd_rows");
}

// A dense copy of `t` (or `t` itself when already dense).
struct DenseView {
    tpb_tensor t;
    Scratch buf;
    DenseView(const tpb_tensor& src, int dev, cudaStream_t stream)
        : t(src), buf(is_contiguous(src) ? 0 : numel_of(src) * dtype_size(src.dtype), dev, stream) {
        if (!is_contiguous(src)) {
            t = dense_like(buf.get(), src.dtype, src.ndim, src.sizes);
            copy_impl(t, src, stream, dev);
        }
    }
};

void softmax_shape(const tpb_tensor& t, int dim, int64_t* outer, int64_t* D, int64_t* inner) {
    const int nd = t.ndim == 0 ? 1 : t.ndim;
    if (dim < 0) dim += nd;
    TPB_CHECK(dim >= 0 && dim < nd, "softmax: dimension out of range");
    *outer = 1;
    *inner = 1;
    *D = t.ndim == 0 ? 1 : t.sizes[dim];
    for (int i = 0; i < dim; ++i) *outer *= t.sizes[i];
    for (int i = dim + 1; i < t.ndim; ++i) *inner *= t.sizes[i];
}

void check_same_shape(const tpb_tensor& a, const tpb_tensor& b, const char* what) {
    TPB_CHECK(a.ndim == b.ndim, "%s: rank mismatch", what);
    for (int i = 0; i < a.ndim; ++i) TPB_CHECK(a.sizes[i] == b.sizes[i], "%s: shape mismatch", what);
}

}  // namespace
}  // namespace tpb

// ---------------------------------------------------------------------------
// Allocation-free reductions (tp_b200_reduce_noalloc).
//
// Some callers cannot allocate device memory at the moment they reduce: a
// serving process whose GPU memory is reserved up front by its own pool, so a
// library allocation behind its back can fail or break its accounting; or a
// latency-critical path that must not risk cudaMalloc (which can synchronise
// the device) when the caching allocator misses.  For them the reduction's
// per-block partial results live in this fixed array instead of the caching
// allocator.  It is 8 MiB per GPU, reserved by every GPU that loads the
// library until the process exits, and it is shared by every call: a call
// overwrites what the previous one left (every partial slot a launch reads is
// written by that launch first, so nothing needs clearing), and two calls
// whose work overlaps on the GPU race on it.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_reduce_noalloc_scratch[kNoAllocScratchBytes];

namespace tpb {
namespace {

std::mutex g_noalloc_lock;
void* g_noalloc_ptr[64] = {};

// Every kernel the allocation-free path can launch for input type T, result
// type To and operation OP, loaded now: under lazy module loading (the CUDA
// 12 default) a kernel's code is otherwise loaded, and device memory taken
// for it, at its first launch.  The occupancy queries the plans make are
// answered and cached here too.
template <typename T, typename To, int OP>
void preload_kernels(int dev, int sms) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    cudaFuncAttributes fa;
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_rows<T, To, OP>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_rows_warp<T, To, OP>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_rows_ring<T, To, OP>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_row_partials<A, To, OP>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_cols<T, To, OP, V, 1>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_cols<T, To, OP, 1, 1>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_cols<T, To, OP, V, kColLanes>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_cols<T, To, OP, 1, kColLanes>));
    TPB_CUDA(cudaFuncGetAttributes(&fa, reduce_col_partials<A, To, OP>));
    (void)rows_capacity<T, To, OP>(dev, sms);
    (void)plan_cols<T, To, OP>(1, 1, 1, false, dev, sms);
}

template <typename T>
void preload_type(int dev, int sms) {
    using A = typename Acc<T>::type;
    preload_kernels<T, T, TPB_SUM>(dev, sms);
    preload_kernels<T, T, TPB_MEAN>(dev, sms);
    preload_kernels<T, T, TPB_AMAX>(dev, sms);
    preload_kernels<T, T, TPB_AMIN>(dev, sms);
    if constexpr (!std::is_same<T, A>::value) {
        preload_kernels<T, A, TPB_SUM>(dev, sms);
        preload_kernels<T, A, TPB_MEAN>(dev, sms);
    }
}

// Device address of the array on `dev` (the caller has made `dev` current).
// In host code the array's name is only a host-side handle, so the address is
// looked up once per device and cached.  That first lookup is the entry
// point's set-up on the device: it loads this file's module (committing the
// array and the completion tickets) and every kernel the entry point can
// launch, so that no later call on the device takes device memory.
void* noalloc_scratch(int dev) {
    TPB_CHECK(dev >= 0 && dev < 64, "invalid device index %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_lock);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        TPB_CUDA(cudaGetSymbolAddress(&p, g_reduce_noalloc_scratch));
        TPB_CHECK(p != nullptr, "reduce_noalloc: no device address for the static scratch");
        (void)ticket_base(dev);
        const int sms = num_sms(dev);
        preload_type<uint8_t>(dev, sms);
        preload_type<int8_t>(dev, sms);
        preload_type<int16_t>(dev, sms);
        preload_type<int32_t>(dev, sms);
        preload_type<int64_t>(dev, sms);
        preload_type<__half>(dev, sms);
        preload_type<float>(dev, sms);
        preload_type<__nv_bfloat16>(dev, sms);
        preload_type<double>(dev, sms);
        preload_type<bool>(dev, sms);
        g_noalloc_ptr[dev] = p;
    }
    return g_noalloc_ptr[dev];
}

void check_noalloc_fit(size_t nbytes) {
    TPB_CHECK(nbytes <= kNoAllocScratchBytes,
              "reduce_noalloc: this reduction needs %zu bytes of partial results, more than the "
              "%zu-byte static scratch of the allocation-free entry point; use tp_b200_reduce",
              nbytes, kNoAllocScratchBytes);
}

// Same kernels and the same split policy as reduce_launch, with the partial
// results in the static array; layouts that would need a gathered copy of the
// input are refused.
template <typename T, typename To, int OP>
void reduce_launch_noalloc(const tpb_tensor& out, const tpb_tensor& xin, uint32_t mask, int dev,
                           cudaStream_t stream, void* scratch) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    const int sms = num_sms(dev);
    DimGroup kept, red;
    for (int i = 0; i < xin.ndim; ++i) {
        DimGroup& g = (mask >> i) & 1 ? red : kept;
        g.sizes[g.n] = xin.sizes[i];
        g.strides[g.n] = xin.strides[i];
        ++g.n;
    }
    const int64_t rows = kept.numel();
    const int64_t R = red.numel();
    // R == 1 (nothing to reduce) runs through the row kernels below like any
    // other reduction (one element per row; exact for every op and result
    // type), not through a copy, whose kernels live in another module that
    // the set-up does not load.
    kept.coalesce();
    red.coalesce();
    To* o = static_cast<To*>(out.data);
    const double count = static_cast<double>(R);
    const T* x = static_cast<const T*>(xin.data);
    A* partial = static_cast<A*>(scratch);

    const bool cols = red.n == 1 && kept.n >= 1 && kept.n <= 2 && kept.strides[kept.n - 1] == 1 &&
                      red.strides[0] != 1;
    if (cols) {
        const int64_t K = kept.sizes[kept.n - 1];
        const int64_t O = kept.n == 2 ? kept.sizes[0] : 1;
        const int64_t os = kept.n == 2 ? kept.strides[0] : 0;
        const int64_t rs = red.strides[0];
        const bool vec = K % V == 0 && rs % V == 0 && os % V == 0 && aligned16(x);
        TPB_CHECK(O < 65536, "reduce_noalloc: %lld outer rows exceed the column kernel's grid",
                  (long long)O);
        const ColPlan plan = plan_cols<T, To, OP>(O, R, K, vec, dev, sms);
        if (plan.splits > 1) check_noalloc_fit(sizeof(A) * plan.splits * O * K);
        launch_cols<T, To, OP>(plan, vec, x, o, partial, O, R, K, os, rs, count, stream);
        return;
    }
    const bool rows_ok = red.n == 0 || (red.n == 1 && red.strides[0] == 1);
    TPB_CHECK(rows_ok,
              "reduce_noalloc: the reduced dimensions are not laid out contiguously; this layout "
              "needs a gathered copy of the input (%lld bytes), which the allocation-free entry "
              "point does not make -- pass a contiguous input or use tp_b200_reduce",
              (long long)(numel_of(xin) * (int64_t)sizeof(T)));
    TPB_CHECK(rows < (int64_t(1) << 31), "reduce_noalloc: too many output elements");
    const int which[1] = {0};
    const auto calc = OffsetCalc<1>::make(group_layout(kept), which);
    const RowPlan plan = plan_rows<T>(x, kept, rows, R, sms, rows_capacity<T, To, OP>(dev, sms));
    if (plan.splits > 1) check_noalloc_fit(sizeof(A) * rows * plan.splits);
    launch_rows<T, To, OP>(plan, x, o, partial, calc, rows, R, count, dev, sms, stream);
}

template <typename T, int OP>
void reduce_noalloc_out(const tpb_tensor& out, const tpb_tensor& x, uint32_t mask, int dev,
                        cudaStream_t stream, void* scratch) {
    using A = typename Acc<T>::type;
    if (out.dtype == x.dtype) {
        reduce_launch_noalloc<T, T, OP>(out, x, mask, dev, stream, scratch);
    } else if (out.dtype == AccCode<A>::value) {
        reduce_launch_noalloc<T, A, OP>(out, x, mask, dev, stream, scratch);
    } else {
        TPB_CHECK(false, "reduce_noalloc: a %s result of a %s input needs a conversion buffer; use "
                  "tp_b200_reduce", dtype_name(out.dtype), dtype_name(x.dtype));
    }
}

template <typename T>
void reduce_noalloc_op(int op, const tpb_tensor& out, const tpb_tensor& x, uint32_t mask, int dev,
                       cudaStream_t stream, void* scratch) {
    switch (op) {
        case TPB_SUM: reduce_noalloc_out<T, TPB_SUM>(out, x, mask, dev, stream, scratch); break;
        case TPB_MEAN: reduce_noalloc_out<T, TPB_MEAN>(out, x, mask, dev, stream, scratch); break;
        case TPB_AMAX: reduce_launch_noalloc<T, T, TPB_AMAX>(out, x, mask, dev, stream, scratch); break;
        case TPB_AMIN: reduce_launch_noalloc<T, T, TPB_AMIN>(out, x, mask, dev, stream, scratch); break;
        default: TPB_CHECK(false, "reduce_noalloc: unknown op %d", op);
    }
}

}  // namespace
}  // namespace tpb

using namespace tpb;

extern "C" {

int tp_b200_reduce_noalloc(int op, const tpb_tensor* out, const tpb_tensor* x, uint32_t dim_mask,
                           void* stream) {
    return guarded([&] {
        check_tensor(out, "reduce_noalloc out");
        check_tensor(x, "reduce_noalloc input");
        TPB_CHECK(out->ndim == x->ndim, "reduce_noalloc: the output keeps every dimension (keepdim layout)");
        TPB_CHECK(x->ndim == 0 || (dim_mask >> x->ndim) == 0, "reduce_noalloc: dimension mask out of range");
        for (int i = 0; i < x->ndim; ++i) {
            const int64_t want = (dim_mask >> i) & 1 ? 1 : x->sizes[i];
            TPB_CHECK(out->sizes[i] == want, "reduce_noalloc: output size %lld at dimension %d, expected %lld",
                      (long long)out->sizes[i], i, (long long)want);
        }
        TPB_CHECK(is_contiguous(*out), "reduce_noalloc: the output must be contiguous");
        if (op == TPB_AMAX || op == TPB_AMIN) {
            TPB_CHECK(out->dtype == x->dtype, "amax/amin: output dtype must match the input");
        }
        if (numel_of(*out) == 0) return;
        TPB_CHECK(numel_of(*x) > 0, "reduce_noalloc: empty reductions are not supported here; use tp_b200_reduce");
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        void* scratch = noalloc_scratch(dev);
        TPB_DISPATCH_ALL(x->dtype, "reduce_noalloc",
                         { reduce_noalloc_op<scalar_t>(op, *out, *x, dim_mask, dev, s, scratch); });
    });
}

}  // extern "C"

extern "C" {

int tp_b200_reduce(int op, const tpb_tensor* out, const tpb_tensor* x, uint32_t dim_mask,
                   void* stream) {
    return guarded([&] {
        check_tensor(out, "reduce out");
        check_tensor(x, "reduce input");
        TPB_CHECK(out->ndim == x->ndim, "reduce: the output keeps every dimension (keepdim layout)");
        TPB_CHECK(x->ndim == 0 || (dim_mask >> x->ndim) == 0, "reduce: dimension mask out of range");
        for (int i = 0; i < x->ndim; ++i) {
            const int64_t want = (dim_mask >> i) & 1 ? 1 : x->sizes[i];
            TPB_CHECK(out->sizes[i] == want, "reduce: output size %lld at dimension %d, expected %lld",
                      (long long)out->sizes[i], i, (long long)want);
        }
        TPB_CHECK(is_contiguous(*out), "reduce: the output must be contiguous");
        if (op == TPB_AMAX || op == TPB_AMIN) {
            TPB_CHECK(out->dtype == x->dtype, "amax/amin: output dtype must match the input");
        }
        const int64_t n_out = numel_of(*out);
        if (n_out == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        if (numel_of(*x) == 0) {
            TPB_CHECK(op == TPB_SUM || op == TPB_MEAN,
                      "amax/amin: expected a non-empty reduction (the operation has no identity)");
            tpb_tensor o = *out;
            const double v = op == TPB_MEAN ? NAN : 0.0;
            TPB_CHECK(tp_b200_fill(&o, v, 0, s) == 0, "%s", tp_b200_last_error());
            return;
        }
        TPB_DISPATCH_ALL(x->dtype, "reduce", { reduce_op_dispatch<scalar_t>(op, *out, *x, dim_mask, dev, s); });
    });
}

int tp_b200_softmax(int log, const tpb_tensor* out, const tpb_tensor* x, int dim, void* stream) {
    return guarded([&] {
        check_tensor(out, "softmax out");
        check_tensor(x, "softmax input");
        TPB_CHECK(out->dtype == x->dtype, "softmax: output dtype must match the input");
        check_same_shape(*out, *x, "softmax");
        TPB_CHECK(is_contiguous(*out), "softmax: the output must be contiguous");
        if (numel_of(*x) == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int64_t outer, D, inner;
        softmax_shape(*x, dim, &outer, &D, &inner);
        DenseView xd(*x, dev, s);
        TPB_DISPATCH_FLOAT(x->dtype, "softmax", {
            softmax_launch<scalar_t>(log != 0, static_cast<scalar_t*>(out->data),
                                     static_cast<const scalar_t*>(xd.t.data), outer, D, inner, dev, s);
        });
    });
}

int tp_b200_softmax_backward(int log, const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* y,
                             int dim, void* stream) {
    return guarded([&] {
        check_tensor(dx, "softmax_backward dx");
        check_tensor(dy, "softmax_backward dy");
        check_tensor(y, "softmax_backward output");
        TPB_CHECK(dx->dtype == dy->dtype && y->dtype == dy->dtype,
                  "softmax_backward: operands must share one dtype");
        check_same_shape(*dx, *dy, "softmax_backward");
        check_same_shape(*dx, *y, "softmax_backward");
        TPB_CHECK(is_contiguous(*dx), "softmax_backward: dx must be contiguous");
        if (numel_of(*dx) == 0) return;
        const int dev = device_of(dx->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int64_t outer, D, inner;
        softmax_shape(*dy, dim, &outer, &D, &inner);
        DenseView dyd(*dy, dev, s);
        DenseView yd(*y, dev, s);
        TPB_DISPATCH_FLOAT(dx->dtype, "softmax_backward", {
            softmax_bwd_launch<scalar_t>(log != 0, static_cast<scalar_t*>(dx->data),
                                         static_cast<const scalar_t*>(dyd.t.data),
                                         static_cast<const scalar_t*>(yd.t.data), outer, D, inner, dev, s);
        });
    });
}

}  // extern "C"
