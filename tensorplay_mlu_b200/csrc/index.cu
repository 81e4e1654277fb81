// Indexing, scattering, prefix scans and where (tensorplay-mlu:
// IndexKernels.cpp:45-352, cnnlGather / cnnlIndexSelect / cnnlScatter /
// cnnlCumsum_v2 / cnnlCumprod / cnnlSelectV2 there, which cover a few dtypes
// and send the rest to the host).  Every dtype runs here.
//
//   gather        out[c] = self[c with c[dim] <- index[c]]   (out shaped like index)
//   index_select  out[.., l, ..] = self[.., index[l], ..]   (16-byte row copies
//                 when the inner extent allows: the embedding lookup)
//   scatter       out[c with c[dim] <- index[c]] (op)= src[c] for c over index's
//                 shape; op: replace, add, multiply, amax, amin, mean
//   index_add     out[.., index[l], ..] += src[.., l, ..]  (index_select's backward)
//   scan          inclusive cumulative sum / product along dim
//   where         out = cond ? a : b, broadcast
//
// Reductions into the same element use atomics: native atomicAdd where the
// type has one, otherwise a compare-and-swap loop (on the enclosing 32-bit
// word for 8- and 16-bit types) capped at kCasTries attempts, after which the
// element is left unchanged and kErrCasTries goes to the device error word.
// Floating sums into one element therefore round in an order that depends
// on scheduling; integer results, amax / amin and replace-without-duplicates
// are exact.  An index outside [-size, size) writes nothing and sets
// kErrIndexRange (negative indices count from the end, as in the reference's
// schema).

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <type_traits>

#include "common.h"
#include "device.cuh"

namespace tpb {
namespace {

constexpr int kThreads = 256;
constexpr int kErrIndexRange = 0x7c31;
constexpr int kErrCasTries = 0x7c32;
constexpr int kCasTries = 1 << 22;

enum ScatterMode { kReplace = 0, kAdd = 1, kMultiply = 2, kAmax = 3, kAmin = 4, kMean = 5 };

// Offsets of N operands for a linear index over `size` (row-major).
template <int N>
struct Offsets {
    int ndim;
    FastDiv div[TPB_MAX_DIMS];
    uint32_t size[TPB_MAX_DIMS];
    int64_t stride[N][TPB_MAX_DIMS];

    __device__ __forceinline__ void get(uint32_t linear, int64_t* off, uint32_t* coord_dim, int dim) const {
#pragma unroll
        for (int k = 0; k < N; ++k) off[k] = 0;
        for (int i = ndim - 1; i >= 0; --i) {
            const uint32_t q = div[i].div(linear);
            const uint32_t r = linear - q * size[i];
            linear = q;
            if (i == dim) *coord_dim = r;
#pragma unroll
            for (int k = 0; k < N; ++k) off[k] += static_cast<int64_t>(r) * stride[k][i];
        }
    }
};

template <int N>
Offsets<N> make_offsets(int ndim, const int64_t* sizes, const int64_t* const* strides) {
    Offsets<N> o{};
    o.ndim = ndim;
    for (int i = 0; i < ndim; ++i) {
        o.size[i] = static_cast<uint32_t>(sizes[i]);
        o.div[i] = FastDiv(static_cast<uint32_t>(sizes[i]));
        for (int k = 0; k < N; ++k) o.stride[k][i] = strides[k][i];
    }
    return o;
}

template <typename T> struct IntLimits;
template <> struct IntLimits<int8_t> { static constexpr int64_t lo = -128, hi = 127; };
template <> struct IntLimits<uint8_t> { static constexpr int64_t lo = 0, hi = 255; };
template <> struct IntLimits<int16_t> { static constexpr int64_t lo = -32768, hi = 32767; };
template <> struct IntLimits<int32_t> { static constexpr int64_t lo = -2147483648LL, hi = 2147483647LL; };
template <> struct IntLimits<int64_t> {
    static constexpr int64_t lo = -9223372036854775807LL - 1, hi = 9223372036854775807LL;
};

// The value a reduction starts from where include_self is false.
template <typename T>
__device__ __forceinline__ T reduce_identity(int mode) {
    if constexpr (std::is_integral<T>::value && !std::is_same<T, bool>::value) {
        if (mode == kMultiply) return T(1);
        if (mode == kAmax) return static_cast<T>(IntLimits<T>::lo);
        if (mode == kAmin) return static_cast<T>(IntLimits<T>::hi);
        return T(0);
    } else {
        using C = typename Compute<T>::type;
        if (mode == kMultiply) return store_as<T>(C(1));
        if (mode == kAmax) return store_as<T>(C(-INFINITY));
        if (mode == kAmin) return store_as<T>(C(INFINITY));
        return store_as<T>(C(0));
    }
}

// Accumulator -> stored value of a scan (integers wrap like the host).
template <typename To, typename A>
__device__ __forceinline__ To cvt_scan(A v) {
    if constexpr (std::is_same<To, bool>::value) return v != A(0);
    else if constexpr (std::is_integral<To>::value) return static_cast<To>(static_cast<uint64_t>(v));
    else return store_as<To>(v);
}

// ------------------------------------------------------------- atomics --

template <typename T>
__device__ __forceinline__ T combine_values(int mode, T a, T b) {
    using C = typename Compute<T>::type;
    const C x = load_as<C>(a), y = load_as<C>(b);
    C r;
    switch (mode) {
        case kMultiply: r = x * y; break;
        case kAmax: r = max_nan(x, y); break;
        case kAmin: r = min_nan(x, y); break;
        default: r = x + y; break;  // kAdd, kMean
    }
    return store_as<T>(r);
}

template <typename T>
__device__ __forceinline__ uint64_t to_bits(T v) {
    uint64_t u = 0;
    memcpy(&u, &v, sizeof(T));
    return u;
}
template <typename T>
__device__ __forceinline__ T from_bits(uint64_t u) {
    T v;
    memcpy(&v, &u, sizeof(T));
    return v;
}

// *addr = combine(*addr, v) by compare-and-swap.
template <typename T>
__device__ bool atomic_combine_cas(T* addr, T v, int mode) {
    if constexpr (sizeof(T) == 8) {
        auto* a = reinterpret_cast<unsigned long long*>(addr);
        unsigned long long old = *a;
        for (int i = 0; i < kCasTries; ++i) {
            const unsigned long long nw = to_bits(combine_values<T>(mode, from_bits<T>(old), v));
            const unsigned long long seen = atomicCAS(a, old, nw);
            if (seen == old) return true;
            old = seen;
        }
        return false;
    } else if constexpr (sizeof(T) == 4) {
        auto* a = reinterpret_cast<unsigned int*>(addr);
        unsigned int old = *a;
        for (int i = 0; i < kCasTries; ++i) {
            const unsigned int nw =
                static_cast<unsigned int>(to_bits(combine_values<T>(mode, from_bits<T>(old), v)));
            const unsigned int seen = atomicCAS(a, old, nw);
            if (seen == old) return true;
            old = seen;
        }
        return false;
    } else {
        // 8- / 16-bit element inside an aligned 32-bit word.
        const uintptr_t p = reinterpret_cast<uintptr_t>(addr);
        auto* word = reinterpret_cast<unsigned int*>(p & ~uintptr_t(3));
        const unsigned shift = static_cast<unsigned>(p & 3) * 8;
        const unsigned mask = (sizeof(T) == 1 ? 0xffu : 0xffffu) << shift;
        unsigned int old = *word;
        for (int i = 0; i < kCasTries; ++i) {
            const T cur = from_bits<T>((old & mask) >> shift);
            const unsigned int part = static_cast<unsigned int>(to_bits(combine_values<T>(mode, cur, v))) << shift;
            const unsigned int nw = (old & ~mask) | (part & mask);
            const unsigned int seen = atomicCAS(word, old, nw);
            if (seen == old) return true;
            old = seen;
        }
        return false;
    }
}

template <typename T>
__device__ __forceinline__ void atomic_combine(T* addr, T v, int mode, int* err) {
    if (mode == kAdd || mode == kMean) {
        if constexpr (std::is_same<T, float>::value || std::is_same<T, double>::value ||
                      std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value ||
                      std::is_same<T, int32_t>::value) {
            atomicAdd(addr, v);
            return;
        } else if constexpr (std::is_same<T, int64_t>::value) {
            atomicAdd(reinterpret_cast<unsigned long long*>(addr), static_cast<unsigned long long>(v));
            return;
        }
    }
    if (!atomic_combine_cas(addr, v, mode)) atomicExch(err, kErrCasTries);
}

template <typename I>
__device__ __forceinline__ bool resolve_index(const I* index, int64_t off, int64_t size, int64_t* out, int* err) {
    int64_t i = static_cast<int64_t>(index[off]);
    if (i < 0) i += size;
    if (i < 0 || i >= size) {
        atomicExch(err, kErrIndexRange);
        return false;
    }
    *out = i;
    return true;
}

// --------------------------------------------------------------- gather --

// Operands over index's shape: 0 out, 1 index, 2 self (stride along dim 0).
template <typename T, typename I>
__global__ void __launch_bounds__(kThreads) gather_kernel(T* out, const I* index, const T* self, Offsets<3> o,
                                                          uint32_t n, int dim, int64_t self_dim_size,
                                                          int64_t self_dim_stride, int* err) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
        int64_t off[3];
        uint32_t c = 0;
        o.get(i, off, &c, dim);
        int64_t k;
        out[off[0]] = resolve_index(index, off[1], self_dim_size, &k, err) ? self[off[2] + k * self_dim_stride]
                                                                            : T(0);
    }
}

// ---------------------------------------------------------- index_select --

// Contiguous self [outer, S, inner] -> out [outer, L, inner]; V-element
// vectors along inner (V = 1 when inner or the pointers do not allow more).
template <typename T, typename I, int V>
__global__ void __launch_bounds__(kThreads) index_select_kernel(T* __restrict__ out, const T* __restrict__ self,
                                                                const I* __restrict__ index, int64_t index_stride,
                                                                int64_t outer, int64_t S, int64_t L,
                                                                int64_t inner, int* err) {
    using VT = Vec<T, V>;
    const int64_t iv = inner / V;
    const int64_t n = outer * L * iv;
    for (int64_t e = int64_t(blockIdx.x) * kThreads + threadIdx.x; e < n; e += int64_t(gridDim.x) * kThreads) {
        const int64_t v = e % iv;
        const int64_t ol = e / iv;
        const int64_t l = ol % L, o = ol / L;
        int64_t k;
        VT val;
        if (resolve_index(index, l * index_stride, S, &k, err)) {
            val = reinterpret_cast<const VT*>(self + (o * S + k) * inner)[v];
        } else {
#pragma unroll
            for (int j = 0; j < V; ++j) val.v[j] = T(0);
        }
        reinterpret_cast<VT*>(out + ol * inner)[v] = val;
    }
}

// index_add: out [outer, S, inner] += src [outer, L, inner] at index[l].
template <typename T, typename I>
__global__ void __launch_bounds__(kThreads) index_add_kernel(T* out, const T* src, const I* index,
                                                             int64_t index_stride, int64_t outer, int64_t S,
                                                             int64_t L, int64_t inner, int* err) {
    const int64_t n = outer * L * inner;
    for (int64_t e = int64_t(blockIdx.x) * kThreads + threadIdx.x; e < n; e += int64_t(gridDim.x) * kThreads) {
        const int64_t j = e % inner;
        const int64_t ol = e / inner;
        const int64_t l = ol % L, o = ol / L;
        int64_t k;
        if (resolve_index(index, l * index_stride, S, &k, err)) {
            atomic_combine(out + (o * S + k) * inner + j, src[e], kAdd, err);
        }
    }
}

// -------------------------------------------------------------- scatter --

// Operands over index's shape: 0 index, 1 src, 2 out (stride along dim 0).
// `reset`: write the mode's identity where the scatter lands (include_self
// false) instead of combining.  `count` (mean): scatters per out element.
template <typename T, typename I>
__global__ void __launch_bounds__(kThreads) scatter_kernel(T* out, const I* index, const T* src, Offsets<3> o,
                                                           uint32_t n, int dim, int64_t out_dim_size,
                                                           int64_t out_dim_stride, int mode, bool reset,
                                                           int32_t* count, int* err) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
        int64_t off[3];
        uint32_t c = 0;
        o.get(i, off, &c, dim);
        int64_t k;
        if (!resolve_index(index, off[0], out_dim_size, &k, err)) continue;
        T* dst = out + off[2] + k * out_dim_stride;
        if (reset) {
            *dst = reduce_identity<T>(mode);
            continue;
        }
        if (mode == kReplace) {
            *dst = src[off[1]];
        } else {
            atomic_combine(dst, src[off[1]], mode, err);
            if (count != nullptr) atomicAdd(count + (dst - out), 1);
        }
    }
}

// mean: out = out / (count + include_self) where the scatter landed.
template <typename T>
__global__ void __launch_bounds__(kThreads) scatter_mean_finish(T* out, const int32_t* count, int64_t n,
                                                                bool include_self) {
    using C = typename Compute<T>::type;
    for (int64_t e = int64_t(blockIdx.x) * kThreads + threadIdx.x; e < n; e += int64_t(gridDim.x) * kThreads) {
        const int32_t c = count[e];
        if (c == 0) continue;
        const C d = C(c + (include_self ? 1 : 0));
        const C v = load_as<C>(out[e]);
        if constexpr (std::is_integral<C>::value) {
            C q = v / d;
            if ((v % d != 0) && ((v < 0) != (d < 0))) --q;  // floor division
            out[e] = store_as<T>(q);
        } else {
            out[e] = store_as<T>(v / d);
        }
    }
}

// ----------------------------------------------------------------- scan --

// Accumulators of the scans: integers in int64 (wrapping to the stored
// type), fp32 in fp64 and 16-bit floats in fp32, as the host's scans do.
template <typename T> struct ScanAcc { using type = typename Compute<T>::type; };
template <> struct ScanAcc<float> { using type = double; };
template <> struct ScanAcc<int8_t> { using type = int64_t; };
template <> struct ScanAcc<uint8_t> { using type = int64_t; };
template <> struct ScanAcc<int16_t> { using type = int64_t; };
template <> struct ScanAcc<int32_t> { using type = int64_t; };
template <> struct ScanAcc<bool> { using type = int64_t; };

// Rows of D contiguous elements ([rows, D], inner == 1): one block per row,
// the row scanned in tiles of kThreads elements with a carry.
template <typename T, typename To>
__global__ void __launch_bounds__(kThreads) scan_rows(const T* __restrict__ x, To* __restrict__ out, int64_t D,
                                                      bool product) {
    using A = typename ScanAcc<To>::type;
    __shared__ A warp_tot[kThreads / 32];
    __shared__ A carry_s;
    const T* xr = x + int64_t(blockIdx.x) * D;
    To* yr = out + int64_t(blockIdx.x) * D;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    A carry = product ? A(1) : A(0);
    for (int64_t base = 0; base < D; base += kThreads) {
        const int64_t i = base + threadIdx.x;
        A v = i < D ? load_as<A>(xr[i]) : (product ? A(1) : A(0));
        // Inclusive warp scan.
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const A u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v = product ? v * u : v + u;
        }
        if (lane == 31) warp_tot[warp] = v;
        __syncthreads();
        if (warp == 0) {
            A w = lane < kThreads / 32 ? warp_tot[lane] : (product ? A(1) : A(0));
#pragma unroll
            for (int o = 1; o < kThreads / 32; o <<= 1) {
                const A u = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w = product ? w * u : w + u;
            }
            if (lane < kThreads / 32) warp_tot[lane] = w;  // inclusive prefix of warp totals
        }
        __syncthreads();
        if (warp > 0) v = product ? v * warp_tot[warp - 1] : v + warp_tot[warp - 1];
        v = product ? v * carry : v + carry;
        if (i < D) yr[i] = cvt_scan<To>(v);
        if (threadIdx.x == kThreads - 1) carry_s = v;
        __syncthreads();
        carry = carry_s;
        __syncthreads();
    }
}

// Any [outer, D, inner] layout: a thread walks one (outer, inner) column.
template <typename T, typename To>
__global__ void __launch_bounds__(kThreads) scan_cols(const T* __restrict__ x, To* __restrict__ out, int64_t outer,
                                                      int64_t D, int64_t inner, bool product) {
    using A = typename ScanAcc<To>::type;
    const int64_t n = outer * inner;
    for (int64_t c = int64_t(blockIdx.x) * kThreads + threadIdx.x; c < n; c += int64_t(gridDim.x) * kThreads) {
        const int64_t o = c / inner, j = c % inner;
        const int64_t base = o * D * inner + j;
        A acc = product ? A(1) : A(0);
        for (int64_t d = 0; d < D; ++d) {
            const A v = load_as<A>(x[base + d * inner]);
            acc = product ? acc * v : acc + v;
            out[base + d * inner] = cvt_scan<To>(acc);
        }
    }
}

// ---------------------------------------------------------------- where --

// Operands over out's shape: 0 out, 1 cond, 2 a, 3 b.
template <typename T>
__global__ void __launch_bounds__(kThreads) where_kernel(T* out, const bool* cond, const T* a, const T* b,
                                                         Offsets<4> o, uint32_t n) {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) {
        int64_t off[4];
        uint32_t c = 0;
        o.get(i, off, &c, -1);
        out[off[0]] = cond[off[1]] ? a[off[2]] : b[off[3]];
    }
}

}  // namespace
}  // namespace tpb

// ------------------------------------------------------------ host side --

namespace tpb {
namespace {

unsigned grid_for(int64_t n, int dev) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks_for(n, kThreads),
                                                                        int64_t(num_sms(dev)) * 16)));
}

int norm_dim(int dim, int nd, const char* what) {
    if (dim < 0) dim += nd;
    TPB_CHECK(dim >= 0 && dim < (nd == 0 ? 1 : nd), "%s: dimension out of range", what);
    return dim;
}

template <typename Fn>
void with_index(int dtype, const char* what, Fn fn) {
    if (dtype == TPB_I64) fn(static_cast<int64_t*>(nullptr));
    else if (dtype == TPB_I32) fn(static_cast<int32_t*>(nullptr));
    else TPB_CHECK(false, "%s: index must be int64 or int32, got %s", what, dtype_name(dtype));
}

// The same dispatch as TPB_DISPATCH_ALL, usable with a generic lambda.
template <typename Fn>
void with_value(int dtype, const char* what, Fn fn) {
    switch (dtype) {
        case TPB_U8: fn(static_cast<uint8_t*>(nullptr)); break;
        case TPB_I8: fn(static_cast<int8_t*>(nullptr)); break;
        case TPB_I16: fn(static_cast<int16_t*>(nullptr)); break;
        case TPB_I32: fn(static_cast<int32_t*>(nullptr)); break;
        case TPB_I64: fn(static_cast<int64_t*>(nullptr)); break;
        case TPB_F16: fn(static_cast<__half*>(nullptr)); break;
        case TPB_F32: fn(static_cast<float*>(nullptr)); break;
        case TPB_BF16: fn(static_cast<__nv_bfloat16*>(nullptr)); break;
        case TPB_F64: fn(static_cast<double*>(nullptr)); break;
        case TPB_BOOL: fn(static_cast<bool*>(nullptr)); break;
        default: TPB_CHECK(false, "%s: unsupported dtype %d", what, dtype);
    }
}

template <typename P>
using pointee_t = std::remove_pointer_t<P>;

}  // namespace
}  // namespace tpb

using namespace tpb;

extern "C" {

int tp_b200_gather(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index, int dim, void* stream) {
    return guarded([&] {
        check_tensor(out, "gather result");
        check_tensor(self, "gather input");
        check_tensor(index, "gather index");
        const int nd = self->ndim;
        TPB_CHECK(index->ndim == nd && out->ndim == nd, "gather: index and result need the input's rank");
        TPB_CHECK(out->dtype == self->dtype, "gather: result dtype must match the input");
        const int d = norm_dim(dim, nd, "gather");
        for (int i = 0; i < nd; ++i) {
            TPB_CHECK(out->sizes[i] == index->sizes[i], "gather: result must have the index's shape");
            TPB_CHECK(i == d || index->sizes[i] <= self->sizes[i],
                      "gather: index size %lld exceeds the input's %lld at dimension %d",
                      (long long)index->sizes[i], (long long)self->sizes[i], i);
        }
        const int64_t n = numel_of(*index);
        if (n == 0) return;
        TPB_CHECK(n < (int64_t(1) << 32), "gather: too many elements");
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int64_t self_st[TPB_MAX_DIMS];
        for (int i = 0; i < nd; ++i) self_st[i] = i == d ? 0 : self->strides[i];
        const int64_t* strides[3] = {out->strides, index->strides, self_st};
        const Offsets<3> o = make_offsets<3>(nd, index->sizes, strides);
        const int64_t self_dim = nd == 0 ? 1 : self->sizes[d];
        const int64_t self_dim_stride = nd == 0 ? 0 : self->strides[d];
        int* err = device_error_word(dev);
        with_value(self->dtype, "gather", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            with_index(index->dtype, "gather", [&](auto it) {
                using I = pointee_t<decltype(it)>;
                gather_kernel<T, I><<<grid_for(n, dev), kThreads, 0, s>>>(
                    static_cast<T*>(out->data), static_cast<const I*>(index->data),
                    static_cast<const T*>(self->data), o, static_cast<uint32_t>(n), nd == 0 ? -1 : d, self_dim,
                    self_dim_stride, err);
                check_launch("gather");
            });
        });
    });
}

int tp_b200_index_select(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index, int dim,
                         void* stream) {
    return guarded([&] {
        check_tensor(out, "index_select result");
        check_tensor(self, "index_select input");
        check_tensor(index, "index_select index");
        TPB_CHECK(is_contiguous(*self) && is_contiguous(*out), "index_select: input and result must be contiguous");
        TPB_CHECK(index->ndim <= 1, "index_select: index must be 0-d or 1-d");
        TPB_CHECK(out->dtype == self->dtype, "index_select: result dtype must match the input");
        const int nd = self->ndim;
        const int d = norm_dim(dim, nd, "index_select");
        const int64_t L = numel_of(*index);
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < d; ++i) outer *= self->sizes[i];
        for (int i = d + 1; i < nd; ++i) inner *= self->sizes[i];
        const int64_t S = nd == 0 ? 1 : self->sizes[d];
        TPB_CHECK(numel_of(*out) == outer * L * inner, "index_select: result size does not match");
        if (outer * L * inner == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int* err = device_error_word(dev);
        const int64_t istride = index->ndim == 1 ? index->strides[0] : 0;
        with_value(self->dtype, "index_select", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            constexpr int V = 16 / sizeof(T) > 0 ? 16 / sizeof(T) : 1;
            const bool vec = inner % V == 0 && aligned16(self->data) && aligned16(out->data);
            with_index(index->dtype, "index_select", [&](auto it) {
                using I = pointee_t<decltype(it)>;
                const int64_t n = outer * L * (vec ? inner / V : inner);
                if (vec) {
                    index_select_kernel<T, I, V><<<grid_for(n, dev), kThreads, 0, s>>>(
                        static_cast<T*>(out->data), static_cast<const T*>(self->data),
                        static_cast<const I*>(index->data), istride, outer, S, L, inner, err);
                } else {
                    index_select_kernel<T, I, 1><<<grid_for(n, dev), kThreads, 0, s>>>(
                        static_cast<T*>(out->data), static_cast<const T*>(self->data),
                        static_cast<const I*>(index->data), istride, outer, S, L, inner, err);
                }
                check_launch("index_select");
            });
        });
    });
}

int tp_b200_index_add(const tpb_tensor* out, const tpb_tensor* src, const tpb_tensor* index, int dim,
                      void* stream) {
    return guarded([&] {
        check_tensor(out, "index_add result");
        check_tensor(src, "index_add source");
        check_tensor(index, "index_add index");
        TPB_CHECK(is_contiguous(*out) && is_contiguous(*src), "index_add: result and source must be contiguous");
        TPB_CHECK(index->ndim <= 1 && out->dtype == src->dtype && out->ndim == src->ndim,
                  "index_add: a 1-d index and a source of the result's dtype and rank");
        TPB_CHECK(out->dtype != TPB_BOOL, "index_add: bool has no addition");
        const int nd = out->ndim;
        const int d = norm_dim(dim, nd, "index_add");
        const int64_t L = numel_of(*index);
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < d; ++i) {
            TPB_CHECK(out->sizes[i] == src->sizes[i], "index_add: shapes differ outside the dimension");
            outer *= out->sizes[i];
        }
        for (int i = d + 1; i < nd; ++i) {
            TPB_CHECK(out->sizes[i] == src->sizes[i], "index_add: shapes differ outside the dimension");
            inner *= out->sizes[i];
        }
        TPB_CHECK(nd == 0 || src->sizes[d] == L, "index_add: source length along the dimension must be the index's");
        const int64_t S = nd == 0 ? 1 : out->sizes[d];
        if (outer * L * inner == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int* err = device_error_word(dev);
        const int64_t istride = index->ndim == 1 ? index->strides[0] : 0;
        with_value(out->dtype, "index_add", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            if constexpr (!std::is_same<T, bool>::value) {
                with_index(index->dtype, "index_add", [&](auto it) {
                    using I = pointee_t<decltype(it)>;
                    index_add_kernel<T, I><<<grid_for(outer * L * inner, dev), kThreads, 0, s>>>(
                        static_cast<T*>(out->data), static_cast<const T*>(src->data),
                        static_cast<const I*>(index->data), istride, outer, S, L, inner, err);
                    check_launch("index_add");
                });
            }
        });
    });
}

int tp_b200_scatter(const tpb_tensor* out, const tpb_tensor* index, const tpb_tensor* src, int dim, int mode,
                    int include_self, void* stream) {
    return guarded([&] {
        check_tensor(out, "scatter result");
        check_tensor(index, "scatter index");
        check_tensor(src, "scatter source");
        TPB_CHECK(mode >= kReplace && mode <= kMean, "scatter: unknown mode %d", mode);
        TPB_CHECK(out->dtype == src->dtype, "scatter: source dtype must match the result");
        TPB_CHECK(mode == kReplace || out->dtype != TPB_BOOL, "scatter: bool supports replacement only");
        const int nd = out->ndim;
        TPB_CHECK(index->ndim == nd && src->ndim == nd, "scatter: index and source need the result's rank");
        const int d = norm_dim(dim, nd, "scatter");
        for (int i = 0; i < nd; ++i) {
            TPB_CHECK(index->sizes[i] <= src->sizes[i], "scatter: index larger than the source at dimension %d", i);
            TPB_CHECK(i == d || index->sizes[i] <= out->sizes[i],
                      "scatter: index larger than the result at dimension %d", i);
        }
        TPB_CHECK(mode != kMean || is_contiguous(*out), "scatter: mean needs a contiguous result");
        const int64_t n = numel_of(*index);
        if (n == 0) return;
        TPB_CHECK(n < (int64_t(1) << 32), "scatter: too many elements");
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int64_t out_st[TPB_MAX_DIMS];
        for (int i = 0; i < nd; ++i) out_st[i] = i == d ? 0 : out->strides[i];
        const int64_t* strides[3] = {index->strides, src->strides, out_st};
        const Offsets<3> o = make_offsets<3>(nd, index->sizes, strides);
        const int64_t out_dim = nd == 0 ? 1 : out->sizes[d];
        const int64_t out_dim_stride = nd == 0 ? 0 : out->strides[d];
        int* err = device_error_word(dev);
        const int64_t out_n = numel_of(*out);
        std::unique_ptr<Scratch> count;
        if (mode == kMean) {
            count.reset(new Scratch(sizeof(int32_t) * size_t(out_n), dev, s));
            TPB_CUDA(cudaMemsetAsync(count->get(), 0, sizeof(int32_t) * size_t(out_n), s));
        }
        with_value(out->dtype, "scatter", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            with_index(index->dtype, "scatter", [&](auto it) {
                using I = pointee_t<decltype(it)>;
                auto run = [&](bool reset, int32_t* cnt) {
                    scatter_kernel<T, I><<<grid_for(n, dev), kThreads, 0, s>>>(
                        static_cast<T*>(out->data), static_cast<const I*>(index->data),
                        static_cast<const T*>(src->data), o, static_cast<uint32_t>(n), nd == 0 ? -1 : d, out_dim,
                        out_dim_stride, mode, reset, cnt, err);
                    check_launch("scatter");
                };
                if (mode != kReplace && !include_self) run(true, nullptr);
                run(false, count ? static_cast<int32_t*>(count->get()) : nullptr);
                if (mode == kMean) {
                    if constexpr (!std::is_same<T, bool>::value) {
                        scatter_mean_finish<T><<<grid_for(out_n, dev), kThreads, 0, s>>>(
                            static_cast<T*>(out->data), static_cast<const int32_t*>(count->get()), out_n,
                            include_self != 0);
                        check_launch("scatter_mean");
                    }
                }
            });
        });
    });
}

int tp_b200_scan(int product, const tpb_tensor* out, const tpb_tensor* x, int dim, void* stream) {
    return guarded([&] {
        check_tensor(out, "scan result");
        check_tensor(x, "scan input");
        TPB_CHECK(out->dtype == x->dtype, "scan: input and result dtypes differ; convert first");
        TPB_CHECK(is_contiguous(*out) && is_contiguous(*x), "scan: input and result must be contiguous");
        const int nd = x->ndim;
        TPB_CHECK(out->ndim == nd, "scan: shapes differ");
        for (int i = 0; i < nd; ++i) TPB_CHECK(out->sizes[i] == x->sizes[i], "scan: shapes differ");
        const int d = norm_dim(dim, nd, "scan");
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < d; ++i) outer *= x->sizes[i];
        for (int i = d + 1; i < nd; ++i) inner *= x->sizes[i];
        const int64_t D = nd == 0 ? 1 : x->sizes[d];
        if (outer * D * inner == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        with_value(x->dtype, "scan", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            if (inner == 1 && outer < (int64_t(1) << 31) && (D >= 64 || outer < int64_t(num_sms(dev)) * 32)) {
                scan_rows<T, T><<<static_cast<unsigned>(outer), kThreads, 0, s>>>(
                    static_cast<const T*>(x->data), static_cast<T*>(out->data), D, product != 0);
            } else {
                scan_cols<T, T><<<grid_for(outer * inner, dev), kThreads, 0, s>>>(
                    static_cast<const T*>(x->data), static_cast<T*>(out->data), outer, D, inner, product != 0);
            }
            check_launch("scan");
        });
    });
}

int tp_b200_where(const tpb_tensor* out, const tpb_tensor* cond, const tpb_tensor* a, const tpb_tensor* b,
                  void* stream) {
    return guarded([&] {
        check_tensor(out, "where result");
        check_tensor(cond, "where condition");
        check_tensor(a, "where input");
        check_tensor(b, "where other");
        TPB_CHECK(cond->dtype == TPB_BOOL, "where: the condition must be bool");
        TPB_CHECK(a->dtype == out->dtype && b->dtype == out->dtype, "where: operands must share the result dtype");
        const int64_t n = numel_of(*out);
        if (n == 0) return;
        TPB_CHECK(n < (int64_t(1) << 32), "where: too many elements");
        int64_t sc[TPB_MAX_DIMS], sa[TPB_MAX_DIMS], sb[TPB_MAX_DIMS];
        broadcast_strides(*cond, *out, sc);
        broadcast_strides(*a, *out, sa);
        broadcast_strides(*b, *out, sb);
        const int64_t* strides[4] = {out->strides, sc, sa, sb};
        const Offsets<4> o = make_offsets<4>(out->ndim, out->sizes, strides);
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        with_value(out->dtype, "where", [&](auto vt) {
            using T = pointee_t<decltype(vt)>;
            where_kernel<T><<<grid_for(n, dev), kThreads, 0, s>>>(
                static_cast<T*>(out->data), static_cast<const bool*>(cond->data), static_cast<const T*>(a->data),
                static_cast<const T*>(b->data), o, static_cast<uint32_t>(n));
            check_launch("where");
        });
    });
}

}  // extern "C"
