// Device-side building blocks shared by the memory-bound kernels: element
// types and their compute types, 16-byte vector access, fast index division
// and strided offset calculation.
#pragma once

#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace tpb {

// ---------------------------------------------------------------- types --

// The type an element is computed in: fp32 for the 16-bit floats and fp32,
// fp64 for float64, int64 for every integer type and bool (wrapped back to
// the storage type on store, which gives the storage type's two's-complement
// result for +, -, *).
template <typename T> struct Compute { using type = int64_t; };
template <> struct Compute<float> { using type = float; };
template <> struct Compute<__half> { using type = float; };
template <> struct Compute<__nv_bfloat16> { using type = float; };
template <> struct Compute<double> { using type = double; };

template <typename T> struct IsFloat { static constexpr bool value = false; };
template <> struct IsFloat<float> { static constexpr bool value = true; };
template <> struct IsFloat<__half> { static constexpr bool value = true; };
template <> struct IsFloat<__nv_bfloat16> { static constexpr bool value = true; };
template <> struct IsFloat<double> { static constexpr bool value = true; };

template <typename C, typename T> __device__ __forceinline__ C load_as(T v) { return static_cast<C>(v); }
template <> __device__ __forceinline__ float load_as<float, __half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float load_as<float, __nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ double load_as<double, __half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ double load_as<double, __nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ int64_t load_as<int64_t, bool>(bool v) { return v ? 1 : 0; }

template <typename T, typename C> __device__ __forceinline__ T store_as(C v) { return static_cast<T>(v); }
template <> __device__ __forceinline__ __half store_as<__half, float>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 store_as<__nv_bfloat16, float>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ bool store_as<bool, int64_t>(int64_t v) { return v != 0; }

// ----------------------------------------------------------- vectors --

template <typename T, int N>
struct alignas(sizeof(T) * N) Vec {
    T v[N];
};

template <typename T> struct VecWidth { static constexpr int value = 16 / sizeof(T); };

__host__ __device__ inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// --------------------------------------------------- index arithmetic --

// Unsigned 32-bit division by a run-time invariant divisor with one
// multiply-high, after Granlund & Montgomery, "Division by Invariant Integers
// using Multiplication" (PLDI 1994): for d > 1 pick s = ceil(log2 d) and
// m = floor(2^32 * (2^s - d) / d) + 1; then n / d = (umulhi(n, m) + n) >> s
// for every 32-bit n (the sum is formed in 64 bits).
struct FastDiv {
    uint32_t d = 1, m = 0, s = 0;
    FastDiv() = default;
    __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
        if (d <= 1) {
            m = 0;
            s = 0;
            return;
        }
        s = 0;
        while ((uint64_t(1) << s) < d) ++s;
        m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << s) - d)) / d + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        if (d == 1) return n;
        const uint32_t t = __umulhi(n, m);
        return static_cast<uint32_t>((uint64_t(t) + n) >> s);
    }
};

// Element offsets of NARGS operands for a linear index over a coalesced
// layout (dimension 0 outermost).  32-bit linear indices: launchers use it
// only for tensors below 2^32 elements and fall back to 64-bit arithmetic
// otherwise.
template <int NARGS>
struct OffsetCalc {
    int ndim;
    FastDiv div[TPB_MAX_DIMS];
    uint32_t size[TPB_MAX_DIMS];
    int64_t stride[NARGS][TPB_MAX_DIMS];

    __host__ static OffsetCalc make(const Layout& L, const int* which) {
        OffsetCalc oc;
        oc.ndim = L.ndim;
        for (int i = 0; i < L.ndim; ++i) {
            oc.size[i] = static_cast<uint32_t>(L.sizes[i]);
            oc.div[i] = FastDiv(static_cast<uint32_t>(L.sizes[i]));
            for (int k = 0; k < NARGS; ++k) oc.stride[k][i] = L.strides[which[k]][i];
        }
        return oc;
    }

    __device__ __forceinline__ void get(uint32_t linear, int64_t* off) const {
#pragma unroll
        for (int k = 0; k < NARGS; ++k) off[k] = 0;
        for (int i = ndim - 1; i >= 0; --i) {
            const uint32_t q = div[i].div(linear);
            const uint32_t r = linear - q * size[i];
            linear = q;
#pragma unroll
            for (int k = 0; k < NARGS; ++k) off[k] += static_cast<int64_t>(r) * stride[k][i];
        }
    }
};

// Same, with 64-bit linear indices (tensors of 2^32 elements or more).
template <int NARGS>
struct OffsetCalc64 {
    int ndim;
    int64_t size[TPB_MAX_DIMS];
    int64_t stride[NARGS][TPB_MAX_DIMS];

    __host__ static OffsetCalc64 make(const Layout& L, const int* which) {
        OffsetCalc64 oc;
        oc.ndim = L.ndim;
        for (int i = 0; i < L.ndim; ++i) {
            oc.size[i] = L.sizes[i];
            for (int k = 0; k < NARGS; ++k) oc.stride[k][i] = L.strides[which[k]][i];
        }
        return oc;
    }

    __device__ __forceinline__ void get(int64_t linear, int64_t* off) const {
#pragma unroll
        for (int k = 0; k < NARGS; ++k) off[k] = 0;
        for (int i = ndim - 1; i >= 0; --i) {
            const int64_t q = linear / size[i];
            const int64_t r = linear - q * size[i];
            linear = q;
#pragma unroll
            for (int k = 0; k < NARGS; ++k) off[k] += r * stride[k][i];
        }
    }
};

// --------------------------------------------------------- reductions --

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// NaN-propagating max/min (amax/amin and softmax semantics).
template <typename T> __device__ __forceinline__ bool is_nan(T v) { return false; }
template <> __device__ __forceinline__ bool is_nan<float>(float v) { return v != v; }
template <> __device__ __forceinline__ bool is_nan<double>(double v) { return v != v; }

template <typename T>
__device__ __forceinline__ T max_nan(T a, T b) {
    return (a > b || is_nan(a)) ? a : b;
}
template <typename T>
__device__ __forceinline__ T min_nan(T a, T b) {
    return (a < b || is_nan(a)) ? a : b;
}
// fp32: one max.NaN / min.NaN instruction (a NaN operand gives NaN; of two
// zeros, max gives +0 and min -0 whatever their order).
template <>
__device__ __forceinline__ float max_nan<float>(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
template <>
__device__ __forceinline__ float min_nan<float>(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Vector <-> compute-type conversion; 16-bit floats convert in pairs
// (one packed f32x2 -> bf16x2 / f16x2 instruction per two elements).
template <typename T, int V, typename C>
__device__ __forceinline__ void unpack_vec(const Vec<T, V>& v, C (&out)[V]) {
#pragma unroll
    for (int j = 0; j < V; ++j) out[j] = load_as<C>(v.v[j]);
}
template <int V>
__device__ __forceinline__ void unpack_vec(const Vec<__nv_bfloat16, V>& v, float (&out)[V]) {
    if constexpr (V % 2 == 0) {
#pragma unroll
        for (int j = 0; j < V; j += 2) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.v[j]));
            out[j] = f.x;
            out[j + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) out[j] = __bfloat162float(v.v[j]);
    }
}
template <int V>
__device__ __forceinline__ void unpack_vec(const Vec<__half, V>& v, float (&out)[V]) {
    if constexpr (V % 2 == 0) {
#pragma unroll
        for (int j = 0; j < V; j += 2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v.v[j]));
            out[j] = f.x;
            out[j + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) out[j] = __half2float(v.v[j]);
    }
}
template <typename T, int V, typename C>
__device__ __forceinline__ void pack_vec(const C (&in)[V], Vec<T, V>& v) {
#pragma unroll
    for (int j = 0; j < V; ++j) v.v[j] = store_as<T>(in[j]);
}
template <int V>
__device__ __forceinline__ void pack_vec(const float (&in)[V], Vec<__nv_bfloat16, V>& v) {
    if constexpr (V % 2 == 0) {
#pragma unroll
        for (int j = 0; j < V; j += 2) {
            *reinterpret_cast<__nv_bfloat162*>(&v.v[j]) = __floats2bfloat162_rn(in[j], in[j + 1]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) v.v[j] = __float2bfloat16_rn(in[j]);
    }
}
template <int V>
__device__ __forceinline__ void pack_vec(const float (&in)[V], Vec<__half, V>& v) {
    if constexpr (V % 2 == 0) {
#pragma unroll
        for (int j = 0; j < V; j += 2) {
            *reinterpret_cast<__half2*>(&v.v[j]) = __floats2half2_rn(in[j], in[j + 1]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) v.v[j] = __float2half_rn(in[j]);
    }
}


// Launch helper: number of 256-thread blocks for `work` items of `per_block`.
inline unsigned blocks_for(int64_t work, int64_t per_block) {
    const int64_t b = (work + per_block - 1) / per_block;
    return static_cast<unsigned>(b < 1 ? 1 : b);
}

// ------------------------------------------- programmatic dependent launch --
//
// Kernels launched with launch_pdl may start while the previous kernel on the
// stream is finishing: pdl_entry() lets the next kernel launch (its trigger
// fires once every CTA of this one has started) and then waits until the
// previous kernel has completed and its memory is visible, before any global
// access.  The launch and CTA ramp of a kernel overlap its predecessor's last
// wave; memory ordering is exactly stream order.  Without the launch
// attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_entry() {
    pdl_trigger();
    pdl_wait();
}

bool pdl_enabled();  // false when TPB200_NO_PDL is set (A/B measurements)

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    TPB_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

}  // namespace tpb

// dtype code -> C++ type dispatch.  `body` is instantiated once per type with
// `scalar_t` bound to it.
#define TPB_DISPATCH_ALL(dtype, what, ...)                                        \
    switch (dtype) {                                                              \
        case TPB_U8: { using scalar_t = uint8_t; __VA_ARGS__; break; }            \
        case TPB_I8: { using scalar_t = int8_t; __VA_ARGS__; break; }             \
        case TPB_I16: { using scalar_t = int16_t; __VA_ARGS__; break; }           \
        case TPB_I32: { using scalar_t = int32_t; __VA_ARGS__; break; }           \
        case TPB_I64: { using scalar_t = int64_t; __VA_ARGS__; break; }           \
        case TPB_F16: { using scalar_t = __half; __VA_ARGS__; break; }            \
        case TPB_F32: { using scalar_t = float; __VA_ARGS__; break; }             \
        case TPB_BF16: { using scalar_t = __nv_bfloat16; __VA_ARGS__; break; }    \
        case TPB_F64: { using scalar_t = double; __VA_ARGS__; break; }            \
        case TPB_BOOL: { using scalar_t = bool; __VA_ARGS__; break; }             \
        default: TPB_CHECK(false, "%s: unsupported dtype code %d", what, (int)(dtype)); \
    }

#define TPB_DISPATCH_FLOAT(dtype, what, ...)                                      \
    switch (dtype) {                                                              \
        case TPB_F16: { using scalar_t = __half; __VA_ARGS__; break; }            \
        case TPB_F32: { using scalar_t = float; __VA_ARGS__; break; }             \
        case TPB_BF16: { using scalar_t = __nv_bfloat16; __VA_ARGS__; break; }    \
        case TPB_F64: { using scalar_t = double; __VA_ARGS__; break; }            \
        default: TPB_CHECK(false, "%s: dtype %s is not a floating type", what, ::tpb::dtype_name(dtype)); \
    }
