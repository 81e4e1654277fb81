// Elementwise machinery shared by the operator files (elementwise.cu,
// ew_binary.cu, ew_unary.cu): math, functors, vector packing, the three
// launch shapes and their launcher.  Everything is internal to each
// translation unit (anonymous namespace).
//
// Every operand is described by a coalesced layout (common.h make_layout).
// Three launch shapes cover it:
//   * contiguous: every operand dense in the same order -- 16-byte vector
//     loads/stores, two vectors in flight per thread;
//   * row broadcast: out and one input dense, the other input a dense row of
//     `inner` elements repeated over the outer dimensions (the [M,N] (+) [N]
//     bias pattern) or a single element -- vectorised as well;
//   * general: any strides, offsets from a fast-division offset calculator.
// The two dense shapes are instantiated per operator (the op is a template
// argument, so each kernel holds only its own arithmetic and stays small in
// the instruction cache); the general shape takes the op at run time.
// Floating types compute in fp32 (fp64 for float64); integer types in int64,
// wrapped back to the storage type.
#pragma once

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

// Storage types whose results are rounded to 8 (bf16) or 11 (f16) mantissa
// bits: for them the transcendental functions use the hardware
// approximations, whose relative errors (2^-11 for tanh.approx, ~2^-21 for
// ex2.approx / rcp.approx) are below that rounding, and erf uses the
// rational approximation of Abramowitz & Stegun, Handbook of Mathematical
// Functions (1964), formula 7.1.28 -- erf(x) = 1 - (1 + a1 x + ... + a6 x^6)^-16
// for x >= 0, absolute error <= 3e-7 -- one reciprocal and four squarings, so
// one special-function-unit operation per element (bf16 streams elements
// fast enough for that unit to become the limit).  fp32 and fp64 results
// keep the accurate library functions.
template <typename T> struct Narrow { static constexpr bool value = false; };
template <> struct Narrow<__half> { static constexpr bool value = true; };
template <> struct Narrow<__nv_bfloat16> { static constexpr bool value = true; };

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float erf_as7128(float x) {
    const float ax = fabsf(x);
    float d = fmaf(fmaf(fmaf(fmaf(fmaf(fmaf(0.0000430638f, ax, 0.0002765672f), ax, 0.0001520143f), ax,
                                  0.0092705272f), ax, 0.0422820123f), ax, 0.0705230784f), ax, 1.0f);
    float r = __fdividef(1.0f, d);  // (1 + ...)^-1, then ^16 by four squarings
    r *= r;
    r *= r;
    r *= r;
    r *= r;
    return copysignf(1.0f - r, x);
}

// The normal CDF Phi(x) = (1 + erf(x / sqrt 2)) / 2 in the same form, for
// gelu and its derivative: with h = erfc(|x| / sqrt 2) / 2,
// Phi(x) = 1 - h (x >= 0) or h (x < 0).  7.1.28's coefficients a_k are
// pre-scaled by 2^(-k/2) (the argument |x| / sqrt 2) and the whole
// polynomial by 2^(1/16) (so that the 16th power of its reciprocal is
// erfc / 2): one reciprocal, four squarings, no further scaling.
constexpr double kR2 = 0.70710678118654752440;      // 2^-1/2
constexpr double kS16 = 1.04427378242741384032;     // 2^(1/16)
constexpr float kPhiA0 = float(kS16);
constexpr float kPhiA1 = float(kS16 * 0.0705230784 * kR2);
constexpr float kPhiA2 = float(kS16 * 0.0422820123 * kR2 * kR2);
constexpr float kPhiA3 = float(kS16 * 0.0092705272 * kR2 * kR2 * kR2);
constexpr float kPhiA4 = float(kS16 * 0.0001520143 * kR2 * kR2 * kR2 * kR2);
constexpr float kPhiA5 = float(kS16 * 0.0002765672 * kR2 * kR2 * kR2 * kR2 * kR2);
constexpr float kPhiA6 = float(kS16 * 0.0000430638 * kR2 * kR2 * kR2 * kR2 * kR2 * kR2);

__device__ __forceinline__ float phi_narrow(float x) {
    const float ax = fabsf(x);
    const float d = fmaf(fmaf(fmaf(fmaf(fmaf(fmaf(kPhiA6, ax, kPhiA5), ax, kPhiA4), ax, kPhiA3), ax, kPhiA2), ax,
                              kPhiA1), ax, kPhiA0);
    float h;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(h) : "f"(d));  // d >= 1: no subnormals
    h *= h;
    h *= h;
    h *= h;
    h *= h;
    return x >= 0.0f ? 1.0f - h : h;  // NaN x: d, h are NaN
}

// Two fp32 lanes at once: sm_100's packed FFMA2 / FMUL2 / FADD2 take a
// register pair and round each lane exactly as the scalar instruction does,
// so the pair forms below give the scalar forms' results bit for bit with
// half the floating-point issue slots.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 phi_narrow2(float2 x) {
    const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
    float2 d = __ffma2_rn(f2(kPhiA6), ax, f2(kPhiA5));
    d = __ffma2_rn(d, ax, f2(kPhiA4));
    d = __ffma2_rn(d, ax, f2(kPhiA3));
    d = __ffma2_rn(d, ax, f2(kPhiA2));
    d = __ffma2_rn(d, ax, f2(kPhiA1));
    d = __ffma2_rn(d, ax, f2(kPhiA0));
    float2 h;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(h.x) : "f"(d.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(h.y) : "f"(d.y));
    h = __fmul2_rn(h, h);
    h = __fmul2_rn(h, h);
    h = __fmul2_rn(h, h);
    h = __fmul2_rn(h, h);
    const float2 c = __ffma2_rn(h, f2(-1.0f), f2(1.0f));  // 1 - h, one rounding
    return make_float2(x.x >= 0.0f ? c.x : h.x, x.y >= 0.0f ? c.y : h.y);
}

// Functors that also have a two-lane form declare `kPair = true` and a
// `float2 pair(float2, float2)` member; the dense kernel uses it for even
// vector widths of fp32 compute.
template <typename F, typename = void>
struct PairOf { static constexpr bool value = false; };
template <typename F>
struct PairOf<F, std::void_t<decltype(F::kPair)>> { static constexpr bool value = F::kPair; };

template <bool Fast, typename C>
__device__ __forceinline__ C f_exp(C x) {
    if constexpr (Fast && std::is_same<C, float>::value) return __expf(x);
    else return m_exp(x);
}
template <bool Fast, typename C>
__device__ __forceinline__ C f_log(C x) {
    if constexpr (Fast && std::is_same<C, float>::value) return __logf(x);
    else return m_log(x);
}
template <bool Fast, typename C>
__device__ __forceinline__ C f_tanh(C x) {
    if constexpr (Fast && std::is_same<C, float>::value) return tanh_approx(x);
    else return m_tanh(x);
}
template <bool Fast, typename C>
__device__ __forceinline__ C f_erf(C x) {
    if constexpr (Fast && std::is_same<C, float>::value) return erf_as7128(x);
    else return m_erf(x);
}
// a / b.  The narrow form multiplies by the hardware reciprocal
// (rcp.approx.f32, relative error below 2^-22 over the whole range including
// subnormal results), which keeps 0/0, x/0 and x/inf IEEE-like.
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <bool Fast, typename C>
__device__ __forceinline__ C f_div(C a, C b) {
    if constexpr (Fast && std::is_same<C, float>::value) return a * rcp_approx(b);
    else return a / b;
}

template <typename C, bool Fast = false>
__device__ __forceinline__ C bin_apply(int op, C a, C b, C alpha) {
    switch (op) {
        case TPB_ADD: return a + alpha * b;
        case TPB_SUB: return a - alpha * b;
        case TPB_MUL: return a * b;
        case TPB_DIV:
            if constexpr (std::is_integral<C>::value) return b == 0 ? C(0) : a / b;
            else return f_div<Fast>(a, b);
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

template <typename C, bool Fast = false>
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
            case TPB_EXP: return f_exp<Fast>(x);
            case TPB_LOG: return f_log<Fast>(x);
            case TPB_SQRT: return m_sqrt(x);
            case TPB_RSQRT: return C(1) / m_sqrt(x);
            case TPB_NEG: return -x;
            case TPB_ABS: return m_abs(x);
            case TPB_POW: return pow_apply(x, p);
            case TPB_RELU: return (x > C(0) || x != x) ? x : C(0);
            case TPB_SIGMOID: return f_div<Fast>(C(1), C(1) + f_exp<Fast>(-x));
            case TPB_TANH: return f_tanh<Fast>(x);
            case TPB_SILU: return f_div<Fast>(x, C(1) + f_exp<Fast>(-x));
            case TPB_GELU:
                if constexpr (Fast && std::is_same<C, float>::value) return x * phi_narrow(x);
                else return C(0.5) * x * (C(1) + f_erf<Fast>(x * C(0.70710678118654752440)));
            case TPB_GELU_TANH: {
                const C k_beta = C(0.79788456080286535588);  // sqrt(2/pi)
                const C inner = k_beta * (x + C(0.044715) * x * x * x);
                return C(0.5) * x * (C(1) + f_tanh<Fast>(inner));
            }
            default: return x * x;  // TPB_SQUARE
        }
    }
}

// Derivatives of the activations (standard calculus; the gelu forms follow
// the two definitions above).
template <typename C, bool Fast = false>
__device__ __forceinline__ C unary_backward_apply(int op, C dy, C z, C p) {
    switch (op) {
        case TPB_THRESHOLD_BACKWARD: return z <= p ? C(0) : dy;
        case TPB_SIGMOID_BACKWARD: return dy * (C(1) - z) * z;
        case TPB_TANH_BACKWARD: return dy * (C(1) - z * z);
        case TPB_GELU_BACKWARD: {
            if constexpr (std::is_integral<C>::value) return dy;
            else if constexpr (Fast && std::is_same<C, float>::value) {
                // Phi(z) + z phi(z), phi(z) = exp2(-z^2 log2(e) / 2) / sqrt(2 pi)
                float e;
                asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(z * z * -0.72134752044448170368f));
                return dy * fmaf(z * 0.39894228040143267794f, e, phi_narrow(z));
            } else {
                const C cdf = C(0.5) * (C(1) + f_erf<Fast>(z * C(0.70710678118654752440)));
                const C pdf = f_exp<Fast>(C(-0.5) * z * z) * C(0.39894228040143267794);  // 1/sqrt(2pi)
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
                const C t = f_tanh<Fast>(inner);
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
                const C s = f_div<Fast>(C(1), C(1) + f_exp<Fast>(-z));
                return dy * s * (C(1) + z * (C(1) - s));
            }
        }
    }
}

// Functors with the common shape C f(C a, C b).
template <typename C, bool Fast>
struct BinaryF {
    int op;
    C alpha;
    __device__ __forceinline__ C operator()(C a, C b) const { return bin_apply<C, Fast>(op, a, b, alpha); }
};
template <typename C, bool Fast>
struct ScalarF {
    int op;
    C s, alpha;
    __device__ __forceinline__ C operator()(C a, C) const { return bin_apply<C, Fast>(op, a, s, alpha); }
};
template <typename C, bool Fast>
struct UnaryF {
    int op;
    C p;
    __device__ __forceinline__ C operator()(C a, C) const { return unary_apply<C, Fast>(op, a, p); }
};
template <typename C, bool Fast>
struct UnaryBackwardF {
    int op;
    C p;
    __device__ __forceinline__ C operator()(C dy, C z) const {
        return unary_backward_apply<C, Fast>(op, dy, z, p);
    }
};

// The same ops with the operator fixed at compile time.
template <typename C, bool Fast, int OP>
struct BinaryCt {
    C alpha;
    __device__ __forceinline__ C operator()(C a, C b) const { return bin_apply<C, Fast>(OP, a, b, alpha); }
};
template <typename C, bool Fast, int OP>
struct ScalarCt {
    C s, alpha;
    __device__ __forceinline__ C operator()(C a, C) const { return bin_apply<C, Fast>(OP, a, s, alpha); }
};
template <typename C, bool Fast, int OP>
struct UnaryCt {
    C p;
    // gelu on 16-bit storage: x * Phi(x) two lanes at a time.
    static constexpr bool kPair = Fast && std::is_same<C, float>::value && OP == TPB_GELU;
    __device__ __forceinline__ C operator()(C a, C) const { return unary_apply<C, Fast>(OP, a, p); }
    __device__ __forceinline__ float2 pair(float2 a, float2) const { return __fmul2_rn(a, phi_narrow2(a)); }
};
template <typename C, bool Fast, int OP>
struct UnaryBackwardCt {
    C p;
    __device__ __forceinline__ C operator()(C dy, C z) const {
        return unary_backward_apply<C, Fast>(OP, dy, z, p);
    }
};

// ------------------------------------------------------------ kernels --

// All operands dense: V-element vectors (V = 16 bytes / element size, or 1
// when a pointer is not 16-byte aligned), kUnroll vectors per thread.
template <typename T, int V, int NIN, typename F>
__global__ void __launch_bounds__(kThreads) ew_contig(T* __restrict__ out, const T* __restrict__ a,
                                                      const T* __restrict__ b, int64_t n, F f) {
    pdl_entry();
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
            C x[V], y[V], r[V];
            unpack_vec(va[u], x);
            if constexpr (NIN > 1) {
                unpack_vec(vb[u], y);
            } else {
#pragma unroll
                for (int j = 0; j < V; ++j) y[j] = C(0);
            }
            if constexpr (PairOf<F>::value && V % 2 == 0) {
#pragma unroll
                for (int j = 0; j < V; j += 2) {
                    const float2 p = f.pair(make_float2(x[j], x[j + 1]), make_float2(y[j], y[j + 1]));
                    r[j] = p.x;
                    r[j + 1] = p.y;
                }
            } else {
#pragma unroll
                for (int j = 0; j < V; ++j) r[j] = f(x[j], y[j]);
            }
            VT vo;
            pack_vec(r, vo);
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
    pdl_entry();
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
            C x[V], y[V], r[V];
            unpack_vec(vf, x);
            if (single) {
#pragma unroll
                for (int j = 0; j < V; ++j) y[j] = single_value;
            } else {
                unpack_vec(vr, y);
            }
#pragma unroll
            for (int j = 0; j < V; ++j) r[j] = row_first ? f(y[j], x[j]) : f(x[j], y[j]);
            VT vo;
            pack_vec(r, vo);
            reinterpret_cast<VT*>(out)[i] = vo;
        }
    }
}

// Row broadcast over rows of at least kThreads vectors: block (x, y) owns
// kThreads column vectors of kRowsPerBlock consecutive outer rows; a thread
// loads its row vector once and reuses it for each row (no index division,
// one row read per kRowsPerBlock outputs).
constexpr int kRowsPerBlock = 4;

template <typename T, int V, bool ROW_FIRST, typename F>
__global__ void __launch_bounds__(kThreads) ew_rowbcast2d(T* __restrict__ out, const T* __restrict__ full,
                                                          const T* __restrict__ row, int64_t outer,
                                                          int64_t inner_v, F f) {
    pdl_entry();
    using C = typename Compute<T>::type;
    using VT = Vec<T, V>;
    const int64_t c = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (c >= inner_v) return;
    const int64_t o0 = int64_t(blockIdx.y) * kRowsPerBlock;
    C y[V];
    unpack_vec(reinterpret_cast<const VT*>(row)[c], y);
    VT vf[kRowsPerBlock];
#pragma unroll
    for (int u = 0; u < kRowsPerBlock; ++u) {
        if (o0 + u < outer) vf[u] = reinterpret_cast<const VT*>(full)[(o0 + u) * inner_v + c];
    }
#pragma unroll
    for (int u = 0; u < kRowsPerBlock; ++u) {
        if (o0 + u < outer) {
            C x[V], r[V];
            unpack_vec(vf[u], x);
#pragma unroll
            for (int j = 0; j < V; ++j) r[j] = ROW_FIRST ? f(y[j], x[j]) : f(x[j], y[j]);
            VT vo;
            pack_vec(r, vo);
            reinterpret_cast<VT*>(out)[(o0 + u) * inner_v + c] = vo;
        }
    }
}

// Any strides.
template <typename T, int NIN, typename F, typename Calc, typename Index>
__global__ void __launch_bounds__(kThreads) ew_general(T* out, const T* a, const T* b, Index n,
                                                       Calc calc, F f) {
    pdl_entry();
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

// `fct`: the op as a compile-time functor (dense shapes); `frt`: the same op
// chosen at run time (general shape).
template <typename T, int NIN, typename Fct, typename Frt>
void launch_elementwise(const char* what, T* out, const T* a, const T* b, const Layout& L, Fct fct,
                        Frt frt, int dev, cudaStream_t stream) {
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
            launch_pdl(ew_contig<T, V, NIN, Fct>, grid, kThreads, 0, stream, out, a, b, n, fct);
        } else {
            const unsigned grid = blocks_for(n, kThreads * kUnroll);
            launch_pdl(ew_contig<T, 1, NIN, Fct>, grid, kThreads, 0, stream, out, a, b, n, fct);
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
            if (!single && inner / V >= kThreads / 2) {
                const int64_t iv = inner / V, outer = n / inner;
                const dim3 grid2(static_cast<unsigned>((iv + kThreads - 1) / kThreads),
                                 static_cast<unsigned>((outer + kRowsPerBlock - 1) / kRowsPerBlock));
                if (grid2.y <= 65535u) {
                    if (which == 1) {
                        launch_pdl(ew_rowbcast2d<T, V, true, Fct>, grid2, kThreads, 0, stream, out, full, row, outer, iv, fct);
                    } else {
                        launch_pdl(ew_rowbcast2d<T, V, false, Fct>, grid2, kThreads, 0, stream, out, full, row, outer, iv, fct);
                    }
                    check_launch(what);
                    return;
                }
            }
            const unsigned grid = blocks_for(n / V, kThreads * kUnroll);
            const uint32_t inner_v = static_cast<uint32_t>(single ? 1 : inner / V);
            launch_pdl(ew_rowbcast<T, V, Fct>, grid, kThreads, 0, stream, out, full, row, n, FastDiv(inner_v),
                       inner_v, single, which == 1, fct);
            check_launch(what);
            return;
        }
    }
    const int which[3] = {0, 1, 2};
    const unsigned grid = static_cast<unsigned>(
        std::min<int64_t>(blocks_for(n, kThreads), int64_t(num_sms(dev)) * 16));
    if (n < (int64_t(1) << 32)) {
        auto calc = OffsetCalc<NIN + 1>::make(L, which);
        launch_pdl(ew_general<T, NIN, Frt, decltype(calc), uint32_t>, grid, kThreads, 0, stream, out, a, b,
                   static_cast<uint32_t>(n), calc, frt);
    } else {
        auto calc = OffsetCalc64<NIN + 1>::make(L, which);
        launch_pdl(ew_general<T, NIN, Frt, decltype(calc), int64_t>, grid, kThreads, 0, stream, out, a, b, n, calc,
                   frt);
    }
    check_launch(what);
}

}  // namespace
}  // namespace tpb
