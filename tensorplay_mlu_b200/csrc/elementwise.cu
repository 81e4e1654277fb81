// Copy, cast and fill (tensorplay-mlu: CopyKernels.cpp and strided_copy in
// Cnnl.cpp, cnnlCopy_v2 / cnnlCastDataType / cnnlFill_v3 there): dense copies
// go to cudaMemcpyAsync, 2-D transposes through a shared-memory tile, other
// strided copies and every dtype conversion through offset-calculator
// kernels.  The arithmetic operators live in ew_binary.cu and ew_unary.cu.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.h"
#include "device.cuh"

namespace tpb {

namespace {

constexpr int kThreads = 256;

// ----------------------------------------------------------- casting --

template <typename T> struct IsHalfLike { static constexpr bool value = false; };
template <> struct IsHalfLike<__half> { static constexpr bool value = true; };
template <> struct IsHalfLike<__nv_bfloat16> { static constexpr bool value = true; };

// Value conversion with the host framework's semantics: 16-bit floats go
// through fp32 in both directions (so float64 -> bfloat16 rounds twice, as
// a conversion through the float constructor does), float -> integer
// truncates, anything -> bool tests != 0.
template <typename D, typename S>
__device__ __forceinline__ D cvt(S v) {
    if constexpr (std::is_same<D, S>::value) {
        return v;
    } else if constexpr (IsHalfLike<S>::value) {
        return cvt<D, float>(load_as<float>(v));
    } else if constexpr (std::is_same<D, bool>::value) {
        return v != S(0);
    } else if constexpr (IsHalfLike<D>::value) {
        return store_as<D, float>(static_cast<float>(v));
    } else {
        return static_cast<D>(v);
    }
}

template <typename D>
__device__ __forceinline__ D load_convert(const char* p, int src) {
    switch (src) {
        case TPB_U8: return cvt<D>(*reinterpret_cast<const uint8_t*>(p));
        case TPB_I8: return cvt<D>(*reinterpret_cast<const int8_t*>(p));
        case TPB_I16: return cvt<D>(*reinterpret_cast<const int16_t*>(p));
        case TPB_I32: return cvt<D>(*reinterpret_cast<const int32_t*>(p));
        case TPB_I64: return cvt<D>(*reinterpret_cast<const int64_t*>(p));
        case TPB_F16: return cvt<D>(*reinterpret_cast<const __half*>(p));
        case TPB_F32: return cvt<D>(*reinterpret_cast<const float*>(p));
        case TPB_BF16: return cvt<D>(*reinterpret_cast<const __nv_bfloat16*>(p));
        case TPB_F64: return cvt<D>(*reinterpret_cast<const double*>(p));
        default: return cvt<D>(*reinterpret_cast<const bool*>(p));
    }
}

template <typename D, typename Calc, typename Index>
__global__ void __launch_bounds__(kThreads) cast_general(D* out, const char* src, int src_dtype,
                                                         int src_es, Index n, Calc calc, bool dense) {
    for (Index i = Index(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += Index(gridDim.x) * kThreads) {
        int64_t off[2];
        if (dense) {
            off[0] = off[1] = static_cast<int64_t>(i);
        } else {
            calc.get(i, off);
        }
        out[off[0]] = load_convert<D>(src + off[1] * src_es, src_dtype);
    }
}

// Same-dtype strided copy by element size.
template <typename U, typename Calc, typename Index>
__global__ void __launch_bounds__(kThreads) copy_general(U* out, const U* src, Index n, Calc calc) {
    for (Index i = Index(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += Index(gridDim.x) * kThreads) {
        int64_t off[2];
        calc.get(i, off);
        out[off[0]] = src[off[1]];
    }
}

// 2-D transpose-like copies ([R,C] with one side column-major) through a
// shared-memory tile so both global sides stay coalesced.
template <typename U>
__global__ void __launch_bounds__(256) copy_transpose(U* out, const U* src, int64_t rows, int64_t cols,
                                                      int64_t out_rs, int64_t out_cs, int64_t src_rs,
                                                      int64_t src_cs) {
    __shared__ U tile[32][33];
    const int64_t r0 = int64_t(blockIdx.y) * 32, c0 = int64_t(blockIdx.x) * 32;
    // Read along the source's unit-stride side (rows here: src_rs == 1).
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int64_t c = c0 + k, r = r0 + threadIdx.x;
        if (r < rows && c < cols) tile[k][threadIdx.x] = src[r * src_rs + c * src_cs];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int64_t r = r0 + k, c = c0 + threadIdx.x;
        if (r < rows && c < cols) out[r * out_rs + c * out_cs] = tile[threadIdx.x][k];
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_kernel(T* out, int64_t n, T value) {
    constexpr int V = VecWidth<T>::value;
    using VT = Vec<T, V>;
    VT vv;
#pragma unroll
    for (int j = 0; j < V; ++j) vv.v[j] = value;
    const int64_t nvec = n / V;
    for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < nvec;
         i += int64_t(gridDim.x) * kThreads) {
        reinterpret_cast<VT*>(out)[i] = vv;
    }
    if (blockIdx.x == 0 && threadIdx.x < n - nvec * V) out[nvec * V + threadIdx.x] = value;
}

template <typename T, typename Calc, typename Index>
__global__ void __launch_bounds__(kThreads) fill_general(T* out, Index n, Calc calc, T value) {
    for (Index i = Index(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += Index(gridDim.x) * kThreads) {
        int64_t off[1];
        calc.get(i, off);
        out[off[0]] = value;
    }
}

template <typename T>
__host__ T host_value(double v, int64_t iv) {
    if constexpr (std::is_same<T, __half>::value) return __float2half_rn(static_cast<float>(v));
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(static_cast<float>(v));
    else if constexpr (std::is_same<T, bool>::value) return iv != 0;
    else if constexpr (std::is_floating_point<T>::value) return static_cast<T>(v);
    else return static_cast<T>(iv);
}

int tensor_device(const tpb_tensor& t) { return device_of(t.data); }

void require_same_shape(const tpb_tensor& a, const tpb_tensor& b, const char* what) {
    TPB_CHECK(a.ndim == b.ndim, "%s: rank mismatch (%d vs %d)", what, a.ndim, b.ndim);
    for (int i = 0; i < a.ndim; ++i) {
        TPB_CHECK(a.sizes[i] == b.sizes[i], "%s: size mismatch at dimension %d (%lld vs %lld)", what,
                  i, (long long)a.sizes[i], (long long)b.sizes[i]);
    }
}

}  // namespace

// ------------------------------------------------------------ C entry --

void copy_impl(const tpb_tensor& dst, const tpb_tensor& src, cudaStream_t stream, int dev) {
    const tpb_tensor* ins[1] = {&src};
    const Layout L = make_layout(dst, ins, 1);
    const int64_t n = L.numel;
    if (n == 0) return;
    const int which[2] = {0, 1};
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>(blocks_for(n, kThreads), int64_t(num_sms(dev)) * 16));
    if (dst.dtype == src.dtype) {
        const size_t es = dtype_size(dst.dtype);
        if (L.ndim <= 1 && (L.ndim == 0 || (L.strides[0][0] == 1 && L.strides[1][0] == 1))) {
            TPB_CUDA(cudaMemcpyAsync(dst.data, src.data, n * es, cudaMemcpyDeviceToDevice, stream));
            return;
        }
        // A 2-D copy with the unit stride on opposite sides: tiled transpose.
        if (L.ndim == 2 && L.strides[0][1] == 1 && L.strides[1][0] == 1 && L.sizes[0] >= 32 &&
            L.sizes[1] >= 32) {
            dim3 tgrid(static_cast<unsigned>((L.sizes[1] + 31) / 32),
                       static_cast<unsigned>((L.sizes[0] + 31) / 32));
            dim3 tblock(32, 8);
#define TPB_TRANSPOSE(U)                                                                      \
    copy_transpose<U><<<tgrid, tblock, 0, stream>>>(                                          \
        static_cast<U*>(dst.data), static_cast<const U*>(src.data), L.sizes[0], L.sizes[1],    \
        L.strides[0][0], L.strides[0][1], L.strides[1][0], L.strides[1][1])
            if (tgrid.y < 65536) {
                switch (es) {
                    case 1: TPB_TRANSPOSE(uint8_t); break;
                    case 2: TPB_TRANSPOSE(uint16_t); break;
                    case 4: TPB_TRANSPOSE(uint32_t); break;
                    default: TPB_TRANSPOSE(uint64_t); break;
                }
#undef TPB_TRANSPOSE
                check_launch("copy_transpose");
                return;
            }
        }
#define TPB_COPY(U)                                                                              \
    if (n < (int64_t(1) << 32)) {                                                                \
        copy_general<U><<<grid, kThreads, 0, stream>>>(static_cast<U*>(dst.data),                \
                                                       static_cast<const U*>(src.data),          \
                                                       static_cast<uint32_t>(n),                 \
                                                       OffsetCalc<2>::make(L, which));           \
    } else {                                                                                     \
        copy_general<U><<<grid, kThreads, 0, stream>>>(static_cast<U*>(dst.data),                \
                                                       static_cast<const U*>(src.data), n,       \
                                                       OffsetCalc64<2>::make(L, which));         \
    }
        switch (es) {
            case 1: TPB_COPY(uint8_t); break;
            case 2: TPB_COPY(uint16_t); break;
            case 4: TPB_COPY(uint32_t); break;
            default: TPB_COPY(uint64_t); break;
        }
#undef TPB_COPY
        check_launch("copy_general");
        return;
    }
    const bool dense = L.ndim <= 1 && (L.ndim == 0 || (L.strides[0][0] == 1 && L.strides[1][0] == 1));
    const int src_es = static_cast<int>(dtype_size(src.dtype));
    TPB_DISPATCH_ALL(dst.dtype, "copy", {
        if (n < (int64_t(1) << 32)) {
            cast_general<scalar_t><<<grid, kThreads, 0, stream>>>(
                static_cast<scalar_t*>(dst.data), static_cast<const char*>(src.data), src.dtype,
                src_es, static_cast<uint32_t>(n), OffsetCalc<2>::make(L, which), dense);
        } else {
            cast_general<scalar_t><<<grid, kThreads, 0, stream>>>(
                static_cast<scalar_t*>(dst.data), static_cast<const char*>(src.data), src.dtype,
                src_es, n, OffsetCalc64<2>::make(L, which), dense);
        }
    });
    check_launch("cast");
}

}  // namespace tpb

using namespace tpb;

extern "C" {

int tp_b200_copy(const tpb_tensor* dst, const tpb_tensor* src, void* stream) {
    return guarded([&] {
        check_tensor(dst, "copy_ destination");
        check_tensor(src, "copy_ source");
        if (numel_of(*dst) == 0) return;
        const int dev = tensor_device(*dst);
        DeviceGuard guard(dev);
        copy_impl(*dst, *src, resolve_stream(stream, dev), dev);
    });
}

int tp_b200_fill(const tpb_tensor* dst, double value, int64_t ivalue, void* stream) {
    return guarded([&] {
        check_tensor(dst, "fill_");
        const int64_t n = numel_of(*dst);
        if (n == 0) return;
        const int dev = tensor_device(*dst);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const Layout L = make_layout(*dst, nullptr, 0);
        const int which[1] = {0};
        const unsigned grid = static_cast<unsigned>(
            std::min<int64_t>(blocks_for(n, kThreads * 4), int64_t(num_sms(dev)) * 16));
        TPB_DISPATCH_ALL(dst->dtype, "fill_", {
            const scalar_t v = host_value<scalar_t>(value, ivalue);
            const bool dense = L.ndim == 0 || (L.ndim == 1 && L.strides[0][0] == 1);
            if (dense && aligned16(dst->data)) {
                fill_kernel<scalar_t><<<grid, kThreads, 0, s>>>(static_cast<scalar_t*>(dst->data), n, v);
            } else if (n < (int64_t(1) << 32)) {
                fill_general<scalar_t><<<grid, kThreads, 0, s>>>(
                    static_cast<scalar_t*>(dst->data), static_cast<uint32_t>(n),
                    OffsetCalc<1>::make(L, which), v);
            } else {
                fill_general<scalar_t><<<grid, kThreads, 0, s>>>(static_cast<scalar_t*>(dst->data), n,
                                                                OffsetCalc64<1>::make(L, which), v);
            }
        });
        check_launch("fill");
    });
}

}  // extern "C"
