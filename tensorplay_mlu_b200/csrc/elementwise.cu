// Memory-bound elementwise kernels: copy/cast/fill, broadcasting binary
// arithmetic and its scalar forms, unary math and activations with their
// backward kernels (tensorplay-mlu: CopyKernels.cpp, BinaryKernels.cpp,
// UnaryKernels.cpp, all on CNNL there).
//
// Every operand is described by a coalesced layout (common.h make_layout).
// Three launch shapes cover it:
//   * contiguous: every operand dense in the same order -- 16-byte vector
//     loads/stores, two vectors in flight per thread;
//   * row broadcast: out and one input dense, the other input a dense row of
//     `inner` elements repeated over the outer dimensions (the [M,N] (+) [N]
//     bias pattern) or a single element -- vectorised as well;
//   * general: any strides, offsets from a fast-division offset calculator.
// Floating types compute in fp32 (fp64 for float64); integer types in int64,
// wrapped back to the storage type.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.h"
#include "device.cuh"

namespace tpb {

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;

// ------------------------------------------------------------ math ops --

__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return exp(x); }
__device__ __forceinline__ float m_log(float x) { return logf(x); }
__device__ __forceinline__ double m_log(double x) { return log(x); }
__device__ __forceinline__ float m_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double m_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float m_erf(float x) { return erff(x); }
__device__ __forceinline__ double m_erf(double x) { return erf(x); }
__device__ __forceinline__ float m_pow(float x, float p) { return powf(x, p); }
__device__ __forceinline__ double m_pow(double x, double p) { return pow(x, p); }
__device__ __forceinline__ float m_abs(float x) { return fabsf(x); }
__device__ __forceinline__ double m_abs(double x) { return fabs(x); }

template <typename C>
__device__ __forceinline__ C bin_apply(int op, C a, C b, C alpha) {
    switch (op) {
        case TPB_ADD: return a + alpha * b;
        case TPB_SUB: return a - alpha * b;
        case TPB_MUL: return a * b;
        case TPB_DIV:
            if constexpr (std::is_integral<C>::value) return b == 0 ? C(0) : a / b;
            else return a / b;
        default: return b - alpha * a;  // TPB_RSUB
    }
}

// pow with the exponents that have exact cheaper forms (a square is what a
// squared-error loss asks for; UnaryKernels.cpp:140-179 special-cases the
// same set).
template <typename C>
__device__ __forceinline__ C pow_apply(C x, C p) {
    if (p == C(2)) return x * x;
    if (p == C(1)) return x;
    if (p == C(0)) return C(1);
    if (p == C(3)) return x * x * x;
    if (p == C(0.5)) return m_sqrt(x);
    if (p == C(-0.5)) return C(1) / m_sqrt(x);
    if (p == C(-1)) return C(1) / x;
    if (p == C(-2)) return C(1) / (x * x);
    return m_pow(x, p);
}

template <typename C>
__device__ __forceinline__ C unary_apply(int op, C x, C p) {
    if constexpr (std::is_integral<C>::value) {
        switch (op) {
            case TPB_NEG: return -x;
            case TPB_ABS: return x < 0 ? -x : x;
            case TPB_RELU: return x > 0 ? x : C(0);
            case TPB_SQUARE: return x * x;
            default: {  // TPB_POW with a non-negative integral exponent
                C r = 1, b = x;
                for (int64_t e = p; e > 0; e >>= 1) {
                    if (e & 1) r *= b;
                    b *= b;
                }
                return r;
            }
        }
    } else {
        switch (op) {
            case TPB_EXP: return m_exp(x);
            case TPB_LOG: return m_log(x);
            case TPB_SQRT: return m_sqrt(x);
            case TPB_RSQRT: return C(1) / m_sqrt(x);
            case TPB_NEG: return -x;
            case TPB_ABS: return m_abs(x);
            case TPB_POW: return pow_apply(x, p);
            case TPB_RELU: return (x > C(0) || x != x) ? x : C(0);
            case TPB_SIGMOID: return C(1) / (C(1) + m_exp(-x));
            case TPB_TANH: return m_tanh(x);
            case TPB_SILU: return x / (C(1) + m_exp(-x));
            case TPB_GELU: return C(0.5) * x * (C(1) + m_erf(x * C(0.70710678118654752440)));
            case TPB_GELU_TANH: {
                const C k_beta = C(0.79788456080286535588);  // sqrt(2/pi)
                const C inner = k_beta * (x + C(0.044715) * x * x * x);
                return C(0.5) * x * (C(1) + m_tanh(inner));
            }
            default: return x * x;  // TPB_SQUARE
        }
    }
}

// Derivatives of the activations (standard calculus; the gelu forms follow
// the two definitions above).
template <typename C>
__device__ __forceinline__ C unary_backward_apply(int op, C dy, C z, C p) {
    switch (op) {
        case TPB_THRESHOLD_BACKWARD: return z <= p ? C(0) : dy;
        case TPB_SIGMOID_BACKWARD: return dy * (C(1) - z) * z;
        case TPB_TANH_BACKWARD: return dy * (C(1) - z * z);
        case TPB_GELU_BACKWARD: {
            if constexpr (std::is_integral<C>::value) return dy;
            else {
                const C cdf = C(0.5) * (C(1) + m_erf(z * C(0.70710678118654752440)));
                const C pdf = m_exp(C(-0.5) * z * z) * C(0.39894228040143267794);  // 1/sqrt(2pi)
                return dy * (cdf + z * pdf);
            }
        }
        case TPB_GELU_TANH_BACKWARD: {
            if constexpr (std::is_integral<C>::value) return dy;
            else {
                const C k_beta = C(0.79788456080286535588);
                const C k_kappa = C(0.044715);
                const C x2 = z * z;
                const C inner = k_beta * (z + k_kappa * x2 * z);
                const C t = m_tanh(inner);
                const C left = C(0.5) * z;
                const C right = C(1) + t;
                const C left_d = C(0.5) * right;
                const C right_d = left * (C(1) - t * t) * k_beta * (C(1) + C(3) * k_kappa * x2);
                return dy * (left_d + right_d);
            }
        }
        default: {  // TPB_SILU_BACKWARD
            if constexpr (std::is_integral<C>::value) return dy;
            else {
                const C s = C(1) / (C(1) + m_exp(-z));
                return dy * s * (C(1) + z * (C(1) - s));
            }
        }
    }
}

// Functors with the common shape C f(C a, C b).
template <typename C>
struct BinaryF {
    int op;
    C alpha;
    __device__ __forceinline__ C operator()(C a, C b) const { return bin_apply(op, a, b, alpha); }
};
template <typename C>
struct ScalarF {
    int op;
    C s, alpha;
    __device__ __forceinline__ C operator()(C a, C) const { return bin_apply(op, a, s, alpha); }
};
template <typename C>
struct UnaryF {
    int op;
    C p;
    __device__ __forceinline__ C operator()(C a, C) const { return unary_apply(op, a, p); }
};
template <typename C>
struct UnaryBackwardF {
    int op;
    C p;
    __device__ __forceinline__ C operator()(C dy, C z) const {
        return unary_backward_apply(op, dy, z, p);
    }
};

// ------------------------------------------------------------ kernels --

// All operands dense: V-element vectors (V = 16 bytes / element size, or 1
// when a pointer is not 16-byte aligned), kUnroll vectors per thread.
template <typename T, int V, int NIN, typename F>
__global__ void __launch_bounds__(kThreads) ew_contig(T* __restrict__ out, const T* __restrict__ a,
                                                      const T* __restrict__ b, int64_t n, F f) {
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    const int64_t nvec = n / V;
    const int64_t base = int64_t(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
    VT va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = base + int64_t(u) * kThreads;
        if (i < nvec) {
            va[u] = reinterpret_cast<const VT*>(a)[i];
            if (NIN > 1) vb[u] = reinterpret_cast<const VT*>(b)[i];
        }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = base + int64_t(u) * kThreads;
        if (i < nvec) {
            VT vo;
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const C x = load_as<C>(va[u].v[j]);
                const C y = NIN > 1 ? load_as<C>(vb[u].v[j]) : C(0);
                vo.v[j] = store_as<T>(f(x, y));
            }
            reinterpret_cast<VT*>(out)[i] = vo;
        }
    }
    // The last n % V elements.
    if (V > 1 && blockIdx.x == 0 && threadIdx.x < n - nvec * V) {
        const int64_t i = nvec * V + threadIdx.x;
        const C x = load_as<C>(a[i]);
        const C y = NIN > 1 ? load_as<C>(b[i]) : C(0);
        out[i] = store_as<T>(f(x, y));
    }
}

// out and `full` dense; `row` holds `inner` dense elements repeated over the
// outer dimensions (inner == 1: a single broadcast element).  `row_first`
// says whether the row is f's first argument.
template <typename T, int V, typename F>
__global__ void __launch_bounds__(kThreads) ew_rowbcast(T* __restrict__ out, const T* __restrict__ full,
                                                        const T* __restrict__ row, int64_t n,
                                                        FastDiv inner_vecs, uint32_t inner_v,
                                                        bool single, bool row_first, F f) {
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    const int64_t nvec = n / V;
    const int64_t base = int64_t(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
    const C single_value = single ? load_as<C>(row[0]) : C(0);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = base + int64_t(u) * kThreads;
        if (i < nvec) {
            const VT vf = reinterpret_cast<const VT*>(full)[i];
            VT vr;
            if (!single) {
                const uint32_t iv = static_cast<uint32_t>(i);
                const uint32_t r = iv - inner_vecs.div(iv) * inner_v;
                vr = reinterpret_cast<const VT*>(row)[r];
            }
            VT vo;
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const C x = load_as<C>(vf.v[j]);
                const C y = single ? single_value : load_as<C>(vr.v[j]);
                vo.v[j] = store_as<T>(row_first ? f(y, x) : f(x, y));
            }
            reinterpret_cast<VT*>(out)[i] = vo;
        }
    }
}

// Any strides.
template <typename T, int NIN, typename F, typename Calc, typename Index>
__global__ void __launch_bounds__(kThreads) ew_general(T* out, const T* a, const T* b, Index n,
                                                       Calc calc, F f) {
    using C = typename Compute<T>::type;
    for (Index i = Index(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += Index(gridDim.x) * kThreads) {
        int64_t off[NIN + 1];
        calc.get(i, off);
        const C x = load_as<C>(a[off[1]]);
        C y = C(0);
        if constexpr (NIN > 1) y = load_as<C>(b[off[2]]);
        out[off[0]] = store_as<T>(f(x, y));
    }
}

template <typename T, int NIN, typename F>
void launch_elementwise(const char* what, T* out, const T* a, const T* b, const Layout& L, F f,
                        int dev, cudaStream_t stream) {
    const int64_t n = L.numel;
    if (n == 0) return;
    constexpr int V = VecWidth<T>::value;
    // Dense: one coalesced dimension with unit strides everywhere.
    bool dense = L.ndim <= 1;
    for (int k = 0; k <= NIN && dense; ++k) {
        if (L.ndim == 1 && L.strides[k][0] != 1) dense = false;
    }
    if (dense) {
        const bool vec_ok = aligned16(out) && aligned16(a) && (NIN < 2 || aligned16(b));
        if (vec_ok) {
            const unsigned grid = blocks_for(n / V, kThreads * kUnroll);
            ew_contig<T, V, NIN><<<grid, kThreads, 0, stream>>>(out, a, b, n, f);
        } else {
            const unsigned grid = blocks_for(n, kThreads * kUnroll);
            ew_contig<T, 1, NIN><<<grid, kThreads, 0, stream>>>(out, a, b, n, f);
        }
        check_launch(what);
        return;
    }
    // Row broadcast: [outer, inner] with out/full strides (inner, 1) and the
    // row's (0, 1); or one dimension where the broadcast operand has stride 0.
    if (NIN == 2 && n < (int64_t(1) << 32) && aligned16(out)) {
        for (int which = 1; which <= 2; ++which) {
            const int other = 3 - which;  // `which` is the broadcast operand
            const T* full = which == 1 ? b : a;
            const T* row = which == 1 ? a : b;
            bool match = false, single = false;
            int64_t inner = 1;
            if (L.ndim == 1 && L.strides[0][0] == 1 && L.strides[other][0] == 1 &&
                L.strides[which][0] == 0) {
                match = single = true;
            } else if (L.ndim == 2 && L.strides[0][1] == 1 && L.strides[0][0] == L.sizes[1] &&
                       L.strides[other][1] == 1 && L.strides[other][0] == L.sizes[1] &&
                       L.strides[which][1] == 1 && L.strides[which][0] == 0) {
                match = true;
                inner = L.sizes[1];
            }
            if (!match) continue;
            // Vector form needs whole vectors per row (and in total).
            if (!aligned16(full) || n % V != 0 ||
                (!single && (!aligned16(row) || inner % V != 0))) {
                break;
            }
            const unsigned grid = blocks_for(n / V, kThreads * kUnroll);
            const uint32_t inner_v = static_cast<uint32_t>(single ? 1 : inner / V);
            ew_rowbcast<T, V><<<grid, kThreads, 0, stream>>>(out, full, row, n, FastDiv(inner_v),
                                                            inner_v, single, which == 1, f);
            check_launch(what);
            return;
        }
    }
    const int which[3] = {0, 1, 2};
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>(blocks_for(n, kThreads), int64_t(num_sms(dev)) * 16));
    if (n < (int64_t(1) << 32)) {
        auto calc = OffsetCalc<NIN + 1>::make(L, which);
        ew_general<T, NIN><<<grid, kThreads, 0, stream>>>(out, a, b, static_cast<uint32_t>(n), calc, f);
    } else {
        auto calc = OffsetCalc64<NIN + 1>::make(L, which);
        ew_general<T, NIN><<<grid, kThreads, 0, stream>>>(out, a, b, n, calc, f);
    }
    check_launch(what);
}

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

int tp_b200_binary(int op, const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b,
                   double alpha, void* stream) {
    return guarded([&] {
        check_tensor(out, "binary out");
        check_tensor(a, "binary a");
        check_tensor(b, "binary b");
        TPB_CHECK(op >= TPB_ADD && op <= TPB_RSUB, "binary: unknown op %d", op);
        TPB_CHECK(a->dtype == out->dtype && b->dtype == out->dtype,
                  "binary: operands must share the result dtype (%s, %s -> %s); promote first",
                  dtype_name(a->dtype), dtype_name(b->dtype), dtype_name(out->dtype));
        if (numel_of(*out) == 0) return;
        const int dev = tensor_device(*out);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[2] = {a, b};
        const Layout L = make_layout(*out, ins, 2);
        TPB_DISPATCH_ALL(out->dtype, "binary", {
            using C = typename Compute<scalar_t>::type;
            BinaryF<C> f{op, static_cast<C>(std::is_integral<C>::value ? static_cast<double>(static_cast<int64_t>(alpha)) : alpha)};
            launch_elementwise<scalar_t, 2>("binary", static_cast<scalar_t*>(out->data),
                                            static_cast<const scalar_t*>(a->data),
                                            static_cast<const scalar_t*>(b->data), L, f, dev, s);
        });
    });
}

int tp_b200_binary_scalar(int op, const tpb_tensor* out, const tpb_tensor* a, double sv,
                          int64_t si, double alpha, void* stream) {
    return guarded([&] {
        check_tensor(out, "binary_scalar out");
        check_tensor(a, "binary_scalar a");
        TPB_CHECK(op >= TPB_ADD && op <= TPB_RSUB, "binary_scalar: unknown op %d", op);
        TPB_CHECK(a->dtype == out->dtype, "binary_scalar: operand and result dtypes differ");
        if (numel_of(*out) == 0) return;
        const int dev = tensor_device(*out);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[1] = {a};
        const Layout L = make_layout(*out, ins, 1);
        TPB_DISPATCH_ALL(out->dtype, "binary_scalar", {
            using C = typename Compute<scalar_t>::type;
            C scalar, al;
            if constexpr (std::is_integral<C>::value) {
                scalar = static_cast<C>(si);
                al = static_cast<C>(static_cast<int64_t>(alpha));
            } else {
                scalar = static_cast<C>(sv);
                al = static_cast<C>(alpha);
            }
            ScalarF<C> f{op, scalar, al};
            launch_elementwise<scalar_t, 1>("binary_scalar", static_cast<scalar_t*>(out->data),
                                            static_cast<const scalar_t*>(a->data), nullptr, L, f,
                                            dev, s);
        });
    });
}

int tp_b200_unary(int op, const tpb_tensor* out, const tpb_tensor* x, double p, void* stream) {
    return guarded([&] {
        check_tensor(out, "unary out");
        check_tensor(x, "unary x");
        TPB_CHECK(op >= TPB_EXP && op <= TPB_SQUARE, "unary: unknown op %d", op);
        TPB_CHECK(x->dtype == out->dtype, "unary: input and result dtypes differ");
        require_same_shape(*out, *x, "unary");
        const bool int_ok = op == TPB_NEG || op == TPB_ABS || op == TPB_RELU || op == TPB_SQUARE ||
                            (op == TPB_POW && p >= 0 && p == static_cast<double>(static_cast<int64_t>(p)));
        TPB_CHECK(is_floating(out->dtype) || int_ok,
                  "unary: op %d on %s needs a floating dtype; promote first", op, dtype_name(out->dtype));
        if (numel_of(*out) == 0) return;
        const int dev = tensor_device(*out);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[1] = {x};
        const Layout L = make_layout(*out, ins, 1);
        TPB_DISPATCH_ALL(out->dtype, "unary", {
            using C = typename Compute<scalar_t>::type;
            UnaryF<C> f{op, static_cast<C>(p)};
            launch_elementwise<scalar_t, 1>("unary", static_cast<scalar_t*>(out->data),
                                            static_cast<const scalar_t*>(x->data), nullptr, L, f,
                                            dev, s);
        });
    });
}

int tp_b200_unary_backward(int op, const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* z,
                           double p, void* stream) {
    return guarded([&] {
        check_tensor(dx, "backward dx");
        check_tensor(dy, "backward dy");
        check_tensor(z, "backward input");
        TPB_CHECK(op >= TPB_THRESHOLD_BACKWARD && op <= TPB_SILU_BACKWARD,
                  "unary_backward: unknown op %d", op);
        TPB_CHECK(dy->dtype == dx->dtype && z->dtype == dx->dtype,
                  "unary_backward: operands must share one dtype");
        TPB_CHECK(is_floating(dx->dtype) || op == TPB_THRESHOLD_BACKWARD,
                  "unary_backward: op %d needs a floating dtype", op);
        require_same_shape(*dx, *dy, "unary_backward");
        require_same_shape(*dx, *z, "unary_backward");
        if (numel_of(*dx) == 0) return;
        const int dev = tensor_device(*dx);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[2] = {dy, z};
        const Layout L = make_layout(*dx, ins, 2);
        TPB_DISPATCH_ALL(dx->dtype, "unary_backward", {
            using C = typename Compute<scalar_t>::type;
            UnaryBackwardF<C> f{op, static_cast<C>(p)};
            launch_elementwise<scalar_t, 2>("unary_backward", static_cast<scalar_t*>(dx->data),
                                            static_cast<const scalar_t*>(dy->data),
                                            static_cast<const scalar_t*>(z->data), L, f, dev, s);
        });
    });
}

}  // extern "C"
