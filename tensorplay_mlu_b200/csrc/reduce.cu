// Reductions (sum, mean, amax, amin) and softmax / log_softmax with their
// backward kernels (tensorplay-mlu: ReduceKernels.cpp, on cnnlReduce_v2 and
// cnnlSoftmaxForward/Backward there).
//
// Reductions: the input's dimensions are split into kept and reduced ones and
// each group is coalesced.  Three kernels cover the layouts:
//   * rows: the reduced elements of one output are contiguous ([.., R]);
//     one block per (row, split), 16-byte vector loads, warp-shuffle then
//     shared-memory block reduction;
//   * columns: the output index is the contiguous side ([O, R, K] over R);
//     threads own 16-byte column vectors and walk R, split over blocks when
//     the output is small;
//   * anything else is first gathered into a [kept, reduced] dense scratch
//     copy and takes the row kernel.
// Splits write per-block partials to stream-ordered scratch and a second
// pass combines them in a fixed order, so results are deterministic.
//
// Softmax: rows of up to 8192 (fp32) / 16384 (16-bit) elements stay in
// registers between the max, the sum and the write -- one read and one write
// of HBM; longer rows use an online max/sum pass plus a write pass, and
// softmax over a non-innermost dimension walks columns.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>
#include <climits>
#include <mutex>
#include <type_traits>

#include "common.h"
#include "device.cuh"

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
// handles row b / splits, chunk b % splits.
template <typename T, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_rows(const T* __restrict__ x, To* __restrict__ out,
                                                        typename Acc<T>::type* __restrict__ partial,
                                                        OffsetCalc<1> rows_calc, int64_t R, int splits,
                                                        int64_t chunk, double count) {
    using A = typename Acc<T>::type;
    constexpr int V = VecWidth<T>::value;
    using VT = Vec<T, V>;
    const int64_t row = blockIdx.x / splits;
    const int split = blockIdx.x % splits;
    int64_t off;
    rows_calc.get(static_cast<uint32_t>(row), &off);
    const T* base = x + off;
    const int64_t begin = int64_t(split) * chunk;
    const int64_t end = begin + chunk < R ? begin + chunk : R;
    A acc0 = identity<A, OP>(), acc1 = identity<A, OP>();
    int64_t i = begin;
    // Scalar head until the pointer is 16-byte aligned, then vectors.
    while (i < end && !aligned16(base + i) && (i - begin) < V) {
        if (threadIdx.x == 0) acc0 = combine<A, OP>(acc0, load_as<A>(base[i]));
        ++i;
    }
    if (aligned16(base + i)) {
        const int64_t nvec = (end - i) / V;
        const VT* vp = reinterpret_cast<const VT*>(base + i);
        int64_t v = threadIdx.x;
        for (; v + kThreads < nvec; v += 2 * kThreads) {
            const VT a = vp[v];
            const VT b = vp[v + kThreads];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                acc0 = combine<A, OP>(acc0, load_as<A>(a.v[j]));
                acc1 = combine<A, OP>(acc1, load_as<A>(b.v[j]));
            }
        }
        for (; v < nvec; v += kThreads) {
            const VT a = vp[v];
#pragma unroll
            for (int j = 0; j < V; ++j) acc0 = combine<A, OP>(acc0, load_as<A>(a.v[j]));
        }
        i += nvec * V;
    }
    for (int64_t k = i + threadIdx.x; k < end; k += kThreads) {
        acc1 = combine<A, OP>(acc1, load_as<A>(base[k]));
    }
    A acc = block_combine<A, OP>(combine<A, OP>(acc0, acc1));
    if (threadIdx.x == 0) {
        if (splits == 1) out[row] = finalize<To, A, OP>(acc, count);
        else partial[row * splits + split] = acc;
    }
}

// One block per row: combine `splits` partials in index order.
template <typename A, typename To, int OP>
__global__ void __launch_bounds__(kThreads) reduce_row_partials(const A* __restrict__ partial,
                                                                To* __restrict__ out, int splits,
                                                                double count) {
    const int64_t row = blockIdx.x;
    A acc = identity<A, OP>();
    for (int s = threadIdx.x; s < splits; s += kThreads) {
        acc = combine<A, OP>(acc, partial[row * splits + s]);
    }
    acc = block_combine<A, OP>(acc);
    if (threadIdx.x == 0) out[row] = finalize<To, A, OP>(acc, count);
}

// ----------------------------------------------------- column reduce --

// x viewed as [O, R, K]: offset o*os + r*rs + k (k contiguous).  Grid:
// (ceil(K / (V*threads)), O, splits).
template <typename T, typename To, int OP, int V>
__global__ void __launch_bounds__(kThreads) reduce_cols(const T* __restrict__ x, To* __restrict__ out,
                                                        typename Acc<T>::type* __restrict__ partial,
                                                        int64_t O, int64_t R, int64_t K, int64_t os,
                                                        int64_t rs, int64_t rchunk, double count) {
    using A = typename Acc<T>::type;
    using VT = Vec<T, V>;
    const int64_t kv = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (kv * V >= K) return;
    const int64_t o = blockIdx.y;
    const int split = blockIdx.z;
    const int splits = gridDim.z;
    const int64_t r0 = int64_t(split) * rchunk;
    const int64_t r1 = r0 + rchunk < R ? r0 + rchunk : R;
    A acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = identity<A, OP>();
    const T* p = x + o * os + kv * V;
    int64_t r = r0;
    for (; r + 1 < r1; r += 2) {
        const VT a = *reinterpret_cast<const VT*>(p + r * rs);
        const VT b = *reinterpret_cast<const VT*>(p + (r + 1) * rs);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            acc[j] = combine<A, OP>(acc[j], load_as<A>(a.v[j]));
            acc[j] = combine<A, OP>(acc[j], load_as<A>(b.v[j]));
        }
    }
    if (r < r1) {
        const VT a = *reinterpret_cast<const VT*>(p + r * rs);
#pragma unroll
        for (int j = 0; j < V; ++j) acc[j] = combine<A, OP>(acc[j], load_as<A>(a.v[j]));
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
    for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += int64_t(gridDim.x) * kThreads) {
        A acc = identity<A, OP>();
        for (int s = 0; s < splits; ++s) acc = combine<A, OP>(acc, partial[int64_t(s) * n + i]);
        out[i] = finalize<To, A, OP>(acc, count);
    }
}

// ------------------------------------------------------------- softmax --

template <typename C>
__device__ __forceinline__ C sm_exp(C x) {
    if constexpr (std::is_same<C, double>::value) return exp(x);
    else return expf(x);
}
template <typename C>
__device__ __forceinline__ C sm_log(C x) {
    if constexpr (std::is_same<C, double>::value) return log(x);
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

// One block per row of D elements kept in registers: VPT vectors of V
// elements per thread (V = 1 when the row is not vector-aligned).
template <typename T, int V, int VPT, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_rows_reg(const T* __restrict__ x, T* __restrict__ y,
                                                            int64_t D, bool log) {
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    const int64_t row = blockIdx.x;
    const T* xr = x + row * D;
    T* yr = y + row * D;
    C v[VPT][V];
    C m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            const VT a = *reinterpret_cast<const VT*>(xr + idx);
#pragma unroll
            for (int j = 0; j < V; ++j) {
                v[k][j] = load_as<C>(a.v[j]);
                m = max_nan(m, v[k][j]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < V; ++j) v[k][j] = -INFINITY;
        }
    }
    m = block_bcast(block_max(m));
    C s = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const C e = sm_exp(v[k][j] - m);
            s += e;
            if (!log) v[k][j] = e;
        }
    }
    s = block_bcast(block_sum(s));
    const C inv = C(1) / s;
    const C lse = sm_log(s);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * THREADS + threadIdx.x) * V;
        if (idx < D) {
            VT o;
#pragma unroll
            for (int j = 0; j < V; ++j) o.v[j] = store_as<T>(log ? v[k][j] - m - lse : v[k][j] * inv);
            *reinterpret_cast<VT*>(yr + idx) = o;
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
            s = s * sm_exp(m - v) + C(1);
            m = v;
        } else if (v != v) {
            m = v;
        } else {
            s += sm_exp(v - m);
        }
    }
    const C gm = block_bcast(block_max(m));
    s = (m == -INFINITY) ? C(0) : s * sm_exp(m - gm);
    s = block_bcast(block_sum(s));
    const C inv = C(1) / s, lse = sm_log(s);
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const C v = load_as<C>(xr[i]);
        yr[i] = store_as<T>(log ? v - gm - lse : sm_exp(v - gm) * inv);
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
                s = s * sm_exp(m - v) + C(1);
                m = v;
            } else if (v != v) {
                m = v;
            } else {
                s += sm_exp(v - m);
            }
        }
        const C inv = C(1) / s, lse = sm_log(s);
        for (int64_t d = 0; d < D; ++d) {
            const C v = load_as<C>(xc[d * inner]);
            yc[d * inner] = store_as<T>(log ? v - m - lse : sm_exp(v - m) * inv);
        }
    }
}

// Backward, rows in registers: softmax dx = y * (dy - sum(dy * y));
// log_softmax dx = dy - exp(y) * sum(dy).
template <typename T, int V, int VPT, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_bwd_rows_reg(const T* __restrict__ dy, const T* __restrict__ y,
                                                                T* __restrict__ dx, int64_t D, bool log) {
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
                r.v[j] = store_as<T>(log ? g[k][j] - sm_exp(o[k][j]) * acc : o[k][j] * (g[k][j] - acc));
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
        dx[row * D + i] = store_as<T>(log ? g - sm_exp(o) * acc : o * (g - acc));
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
            dx[base + d * inner] = store_as<T>(log ? g - sm_exp(w) * acc : w * (g - acc));
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
        const int vw = vec ? V : 1;
        const int64_t kblocks = (K / vw + kThreads - 1) / kThreads;
        if (O < 65536) {
            int splits = 1;
            const int64_t base_blocks = kblocks * O;
            const int64_t want = int64_t(sms) * 4;
            if (base_blocks < want) {
                splits = static_cast<int>(std::min<int64_t>((want + base_blocks - 1) / base_blocks,
                                                            std::max<int64_t>(R / 16, 1)));
                splits = std::min(splits, 1024);
            }
            const int64_t rchunk = (R + splits - 1) / splits;
            splits = static_cast<int>((R + rchunk - 1) / rchunk);
            if (splits < 1) splits = 1;
            Scratch partial(splits > 1 ? sizeof(A) * splits * O * K : 0, dev, stream);
            dim3 grid(static_cast<unsigned>(kblocks), static_cast<unsigned>(O), static_cast<unsigned>(splits));
            if (vec) {
                reduce_cols<T, To, OP, V><<<grid, kThreads, 0, stream>>>(
                    x, o, static_cast<A*>(partial.get()), O, R, K, os, rs, rchunk, count);
            } else {
                reduce_cols<T, To, OP, 1><<<grid, kThreads, 0, stream>>>(
                    x, o, static_cast<A*>(partial.get()), O, R, K, os, rs, rchunk, count);
            }
            check_launch("reduce_cols");
            if (splits > 1) {
                const int64_t n = O * K;
                const unsigned g2 = static_cast<unsigned>(std::min<int64_t>(blocks_for(n, kThreads), sms * 8));
                reduce_col_partials<A, To, OP><<<g2, kThreads, 0, stream>>>(
                    static_cast<const A*>(partial.get()), o, n, splits, count);
                check_launch("reduce_col_partials");
            }
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
    int splits = 1;
    const int64_t want = int64_t(sms) * 4;
    if (rows < want) {
        splits = static_cast<int>(std::min<int64_t>((want + rows - 1) / rows,
                                                    std::max<int64_t>(R / (kThreads * V * 4), 1)));
    }
    int64_t chunk = (R + splits - 1) / splits;
    chunk = (chunk + V - 1) / V * V;
    if (chunk < 1) chunk = 1;
    splits = static_cast<int>(std::max<int64_t>((R + chunk - 1) / chunk, 1));
    Scratch partial(splits > 1 ? sizeof(A) * rows * splits : 0, dev, stream);
    reduce_rows<T, To, OP><<<static_cast<unsigned>(rows * splits), kThreads, 0, stream>>>(
        x, o, static_cast<A*>(partial.get()), calc, R, splits, chunk, count);
    check_launch("reduce_rows");
    if (splits > 1) {
        reduce_row_partials<A, To, OP><<<static_cast<unsigned>(rows), kThreads, 0, stream>>>(
            static_cast<const A*>(partial.get()), o, splits, count);
        check_launch("reduce_row_partials");
    }
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
    constexpr int V = VecWidth<T>::value;
    const unsigned rows = static_cast<unsigned>(outer);
    TPB_CHECK(outer < (int64_t(1) << 31), "softmax: too many rows");
    const bool vec = D % V == 0 && aligned16(x) && aligned16(y);
    if (vec) {
        const int64_t nv = D / V;
        if (nv <= 256) softmax_rows_reg<T, V, 1, 256><<<rows, 256, 0, stream>>>(x, y, D, log);
        else if (nv <= 512) softmax_rows_reg<T, V, 2, 256><<<rows, 256, 0, stream>>>(x, y, D, log);
        else if (nv <= 1024) softmax_rows_reg<T, V, 4, 256><<<rows, 256, 0, stream>>>(x, y, D, log);
        else if (nv <= 2048) softmax_rows_reg<T, V, 4, 512><<<rows, 512, 0, stream>>>(x, y, D, log);
        else softmax_rows_online<T><<<rows, kThreads, 0, stream>>>(x, y, D, log);
    } else if (D <= 1024) {
        softmax_rows_reg<T, 1, 4, 256><<<rows, 256, 0, stream>>>(x, y, D, log);
    } else {
        softmax_rows_online<T><<<rows, kThreads, 0, stream>>>(x, y, D, log);
    }
    check_launch("softmax_rows");
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
        if (nv <= 256) softmax_bwd_rows_reg<T, V, 1, 256><<<rows, 256, 0, stream>>>(dy, y, dx, D, log);
        else if (nv <= 512) softmax_bwd_rows_reg<T, V, 2, 256><<<rows, 256, 0, stream>>>(dy, y, dx, D, log);
        else if (nv <= 1024) softmax_bwd_rows_reg<T, V, 4, 256><<<rows, 256, 0, stream>>>(dy, y, dx, D, log);
        else if (nv <= 2048) softmax_bwd_rows_reg<T, V, 4, 512><<<rows, 512, 0, stream>>>(dy, y, dx, D, log);
        else softmax_bwd_rows_loop<T><<<rows, kThreads, 0, stream>>>(dy, y, dx, D, log);
    } else if (D <= 1024) {
        softmax_bwd_rows_reg<T, 1, 4, 256><<<rows, 256, 0, stream>>>(dy, y, dx, D, log);
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

// Device address of the array on `dev` (the caller has made `dev` current).
// In host code the array's name is only a host-side handle, so the address is
// looked up once per device and cached.
void* noalloc_scratch(int dev) {
    TPB_CHECK(dev >= 0 && dev < 64, "invalid device index %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_lock);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        TPB_CUDA(cudaGetSymbolAddress(&p, g_reduce_noalloc_scratch));
        TPB_CHECK(p != nullptr, "reduce_noalloc: no device address for the static scratch");
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
    if (R == 1) {
        copy_impl(out, xin, stream, dev);
        return;
    }
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
        const int vw = vec ? V : 1;
        const int64_t kblocks = (K / vw + kThreads - 1) / kThreads;
        TPB_CHECK(O < 65536, "reduce_noalloc: %lld outer rows exceed the column kernel's grid",
                  (long long)O);
        int splits = 1;
        const int64_t base_blocks = kblocks * O;
        const int64_t want = int64_t(sms) * 4;
        if (base_blocks < want) {
            splits = static_cast<int>(std::min<int64_t>((want + base_blocks - 1) / base_blocks,
                                                        std::max<int64_t>(R / 16, 1)));
            splits = std::min(splits, 1024);
        }
        const int64_t rchunk = (R + splits - 1) / splits;
        splits = static_cast<int>((R + rchunk - 1) / rchunk);
        if (splits < 1) splits = 1;
        if (splits > 1) check_noalloc_fit(sizeof(A) * splits * O * K);
        dim3 grid(static_cast<unsigned>(kblocks), static_cast<unsigned>(O), static_cast<unsigned>(splits));
        if (vec) {
            reduce_cols<T, To, OP, V><<<grid, kThreads, 0, stream>>>(x, o, partial, O, R, K, os, rs,
                                                                      rchunk, count);
        } else {
            reduce_cols<T, To, OP, 1><<<grid, kThreads, 0, stream>>>(x, o, partial, O, R, K, os, rs,
                                                                      rchunk, count);
        }
        check_launch("reduce_cols");
        if (splits > 1) {
            const int64_t n = O * K;
            const unsigned g2 = static_cast<unsigned>(std::min<int64_t>(blocks_for(n, kThreads), sms * 8));
            reduce_col_partials<A, To, OP><<<g2, kThreads, 0, stream>>>(partial, o, n, splits, count);
            check_launch("reduce_col_partials");
        }
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
    int splits = 1;
    const int64_t want = int64_t(sms) * 4;
    if (rows < want) {
        splits = static_cast<int>(std::min<int64_t>((want + rows - 1) / rows,
                                                    std::max<int64_t>(R / (kThreads * V * 4), 1)));
    }
    int64_t chunk = (R + splits - 1) / splits;
    chunk = (chunk + V - 1) / V * V;
    if (chunk < 1) chunk = 1;
    splits = static_cast<int>(std::max<int64_t>((R + chunk - 1) / chunk, 1));
    if (splits > 1) check_noalloc_fit(sizeof(A) * rows * splits);
    reduce_rows<T, To, OP><<<static_cast<unsigned>(rows * splits), kThreads, 0, stream>>>(
        x, o, partial, calc, R, splits, chunk, count);
    check_launch("reduce_rows");
    if (splits > 1) {
        reduce_row_partials<A, To, OP><<<static_cast<unsigned>(rows), kThreads, 0, stream>>>(
            partial, o, splits, count);
        check_launch("reduce_row_partials");
    }
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
