// Layer normalisation and negative log-likelihood, forward and backward
// (tensorplay-mlu: NNKernels.cpp:59-161 and :304-397, cnnlLayerNormForward /
// cnnlLayerNormBackward_v2 / cnnlNlllossForward / cnnlNlllossBackward there).
//
// layer_norm: rows of D = prod(normalized_shape) contiguous elements.  A block
// owns a row held in registers (VPT 16-byte vectors per thread) for the mean,
// the variance (second pass over the registers, not E[x^2] - E[x]^2) and the
// write; rows too long for registers are read again from memory.  Statistics
// are accumulated in fp32 (fp64 for fp64 inputs) and returned in that type
// (NNKernels.cpp:53-57).  The backward's dx is per row; dweight / dbias are
// column sums over rows, split over blocks and combined in a fixed order.
//
// nll_loss: (N, C) log-probabilities with (N) class targets.  The reduction
// is deterministic: per-block partial sums of the losses and the weights,
// combined in block order by one block.  A target outside [0, C) that is not
// ignore_index contributes nothing and sets the device error word
// (kErrNllTarget; tp_b200_take_device_error).

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.h"
#include "device.cuh"

namespace tpb {
namespace {

constexpr int kThreads = 256;
constexpr int kErrNllTarget = 0x7c21;

template <typename T> struct Stat { using type = float; };
template <> struct Stat<double> { using type = double; };

template <typename A>
__device__ __forceinline__ A block_sum(A v) {
    __shared__ A warp_vals[32];
    __shared__ A result;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) warp_vals[warp] = v;
    __syncthreads();
    if (warp == 0) {
        const int nwarps = (blockDim.x + 31) >> 5;
        A s = lane < nwarps ? warp_vals[lane] : A(0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) result = s;
    }
    __syncthreads();
    return result;
}

template <typename A>
__device__ __forceinline__ A inv_sqrt(A v) {
    if constexpr (std::is_same<A, double>::value) return 1.0 / sqrt(v);
    else return 1.0f / sqrtf(v);
}

// ----------------------------------------------------------- layer norm --

// Row in registers: VPT vectors of V elements per thread.  `w` / `b` may be
// null (1 / 0).
template <typename T, int V, int VPT>
__global__ void __launch_bounds__(kThreads) layer_norm_rows(const T* __restrict__ x, T* __restrict__ y,
                                                            typename Stat<T>::type* __restrict__ mean_out,
                                                            typename Stat<T>::type* __restrict__ rstd_out,
                                                            const T* __restrict__ w, const T* __restrict__ b,
                                                            int64_t D, double eps) {
    using A = typename Stat<T>::type;
    using VT = Vec<T, V>;
    const int64_t row = blockIdx.x;
    const T* xr = x + row * D;
    T* yr = y + row * D;
    A v[VPT][V];
    A s = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * kThreads + threadIdx.x) * V;
        if (idx < D) {
            unpack_vec(*reinterpret_cast<const VT*>(xr + idx), v[k]);
#pragma unroll
            for (int j = 0; j < V; ++j) s += v[k][j];
        }
    }
    const A mean = block_sum(s) / A(D);
    A q = 0;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * kThreads + threadIdx.x) * V;
        if (idx < D) {
#pragma unroll
            for (int j = 0; j < V; ++j) {
                const A d = v[k][j] - mean;
                q += d * d;
            }
        }
    }
    const A rstd = inv_sqrt(block_sum(q) / A(D) + A(eps));
    if (threadIdx.x == 0) {
        mean_out[row] = mean;
        rstd_out[row] = rstd;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t idx = (int64_t(k) * kThreads + threadIdx.x) * V;
        if (idx < D) {
            A wv[V], bv[V];
            if (w != nullptr) unpack_vec(*reinterpret_cast<const VT*>(w + idx), wv);
            if (b != nullptr) unpack_vec(*reinterpret_cast<const VT*>(b + idx), bv);
            A o[V];
#pragma unroll
            for (int j = 0; j < V; ++j) {
                A t = (v[k][j] - mean) * rstd;
                if (w != nullptr) t *= wv[j];
                if (b != nullptr) t += bv[j];
                o[j] = t;
            }
            VT out;
            pack_vec(o, out);
            *reinterpret_cast<VT*>(yr + idx) = out;
        }
    }
}

// Any row length, element-wise loads (rows too long for registers, or not
// vector-aligned): three passes over the row.
template <typename T>
__global__ void __launch_bounds__(kThreads) layer_norm_rows_loop(const T* __restrict__ x, T* __restrict__ y,
                                                                 typename Stat<T>::type* __restrict__ mean_out,
                                                                 typename Stat<T>::type* __restrict__ rstd_out,
                                                                 const T* __restrict__ w, const T* __restrict__ b,
                                                                 int64_t D, double eps) {
    using A = typename Stat<T>::type;
    const int64_t row = blockIdx.x;
    const T* xr = x + row * D;
    T* yr = y + row * D;
    A s = 0;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) s += load_as<A>(xr[i]);
    const A mean = block_sum(s) / A(D);
    A q = 0;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        const A d = load_as<A>(xr[i]) - mean;
        q += d * d;
    }
    const A rstd = inv_sqrt(block_sum(q) / A(D) + A(eps));
    if (threadIdx.x == 0) {
        mean_out[row] = mean;
        rstd_out[row] = rstd;
    }
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        A t = (load_as<A>(xr[i]) - mean) * rstd;
        if (w != nullptr) t *= load_as<A>(w[i]);
        if (b != nullptr) t += load_as<A>(b[i]);
        yr[i] = store_as<T>(t);
    }
}

// dx for one row: g = dy * w, xhat = (x - mean) * rstd,
// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)).
template <typename T>
__global__ void __launch_bounds__(kThreads) layer_norm_bwd_dx(const T* __restrict__ dy, const T* __restrict__ x,
                                                              const typename Stat<T>::type* __restrict__ mean,
                                                              const typename Stat<T>::type* __restrict__ rstd,
                                                              const T* __restrict__ w, T* __restrict__ dx,
                                                              int64_t D) {
    using A = typename Stat<T>::type;
    const int64_t row = blockIdx.x;
    const T* dyr = dy + row * D;
    const T* xr = x + row * D;
    const A m = mean[row], r = rstd[row];
    A s1 = 0, s2 = 0;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        A g = load_as<A>(dyr[i]);
        if (w != nullptr) g *= load_as<A>(w[i]);
        const A xh = (load_as<A>(xr[i]) - m) * r;
        s1 += g;
        s2 += g * xh;
    }
    const A mg = block_sum(s1) / A(D);
    const A mgx = block_sum(s2) / A(D);
    T* dxr = dx + row * D;
    for (int64_t i = threadIdx.x; i < D; i += kThreads) {
        A g = load_as<A>(dyr[i]);
        if (w != nullptr) g *= load_as<A>(w[i]);
        const A xh = (load_as<A>(xr[i]) - m) * r;
        dxr[i] = store_as<T>(r * (g - mg - xh * mgx));
    }
}

// dweight / dbias partial column sums: split s takes rows s, s + splits, ...;
// partial[s][j] for dweight, partial[splits + s][j] for dbias.
template <typename T>
__global__ void __launch_bounds__(kThreads) layer_norm_bwd_params(const T* __restrict__ dy, const T* __restrict__ x,
                                                                  const typename Stat<T>::type* __restrict__ mean,
                                                                  const typename Stat<T>::type* __restrict__ rstd,
                                                                  typename Stat<T>::type* __restrict__ partial,
                                                                  int64_t rows, int64_t D) {
    using A = typename Stat<T>::type;
    const int64_t j = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (j >= D) return;
    const int split = blockIdx.y, splits = gridDim.y;
    A sw = 0, sb = 0;
    for (int64_t r = split; r < rows; r += splits) {
        const A g = load_as<A>(dy[r * D + j]);
        sw += g * (load_as<A>(x[r * D + j]) - mean[r]) * rstd[r];
        sb += g;
    }
    partial[int64_t(split) * D + j] = sw;
    partial[int64_t(splits + split) * D + j] = sb;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) layer_norm_bwd_params_combine(
    const typename Stat<T>::type* __restrict__ partial, T* __restrict__ dw, T* __restrict__ db, int splits,
    int64_t D) {
    using A = typename Stat<T>::type;
    const int64_t j = int64_t(blockIdx.x) * kThreads + threadIdx.x;
    if (j >= D) return;
    A sw = 0, sb = 0;
    for (int s = 0; s < splits; ++s) {
        sw += partial[int64_t(s) * D + j];
        sb += partial[int64_t(splits + s) * D + j];
    }
    if (dw != nullptr) dw[j] = store_as<T>(sw);
    if (db != nullptr) db[j] = store_as<T>(sb);
}

// ------------------------------------------------------------- nll loss --

template <typename I>
__device__ __forceinline__ bool nll_target(const I* target, int64_t i, int64_t C, int64_t ignore, int* err,
                                           int64_t* t_out) {
    const int64_t t = static_cast<int64_t>(target[i]);
    *t_out = t;
    if (t == ignore) return false;
    if (t < 0 || t >= C) {
        atomicExch(err, kErrNllTarget);
        return false;
    }
    return true;
}

// reduction none: out[i] = -w[t_i] x[i, t_i].  Otherwise per-block partial
// (sum of -w x, sum of w) into partial[2 * block].
template <typename T, typename I>
__global__ void __launch_bounds__(kThreads) nll_forward(const T* __restrict__ x, const I* __restrict__ target,
                                                        const T* __restrict__ w, T* __restrict__ out,
                                                        typename Stat<T>::type* __restrict__ partial, int64_t N,
                                                        int64_t C, int64_t sx_n, int64_t sx_c, int64_t ignore,
                                                        int reduction, int* err) {
    using A = typename Stat<T>::type;
    A loss = 0, wsum = 0;
    for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < N; i += int64_t(gridDim.x) * kThreads) {
        int64_t t;
        A li = 0;
        if (nll_target(target, i, C, ignore, err, &t)) {
            const A wt = w != nullptr ? load_as<A>(w[t]) : A(1);
            li = -wt * load_as<A>(x[i * sx_n + t * sx_c]);
            wsum += wt;
        }
        if (reduction == 0) out[i] = store_as<T>(li);
        else loss += li;
    }
    if (reduction == 0) return;
    loss = block_sum(loss);
    wsum = block_sum(wsum);
    if (threadIdx.x == 0) {
        partial[2 * blockIdx.x] = loss;
        partial[2 * blockIdx.x + 1] = wsum;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) nll_combine(const typename Stat<T>::type* __restrict__ partial,
                                                        int blocks, T* __restrict__ out, T* __restrict__ total,
                                                        int reduction) {
    using A = typename Stat<T>::type;
    A loss = 0, wsum = 0;
    for (int b = threadIdx.x; b < blocks; b += kThreads) {
        loss += partial[2 * b];
        wsum += partial[2 * b + 1];
    }
    loss = block_sum(loss);
    wsum = block_sum(wsum);
    if (threadIdx.x == 0) {
        out[0] = store_as<T>(reduction == 1 ? loss / wsum : loss);
        *total = store_as<T>(wsum);
    }
}

// dx[i, c] = -w[t_i] * g_i at c = t_i (not ignored), 0 elsewhere; g_i = dy[i]
// (none), dy (sum) or dy / total_weight (mean).  One pass writes all of dx.
template <typename T, typename I>
__global__ void __launch_bounds__(kThreads) nll_backward(T* __restrict__ dx, const T* __restrict__ dy,
                                                         const I* __restrict__ target, const T* __restrict__ w,
                                                         const T* __restrict__ total, int64_t N, int64_t C,
                                                         int64_t ignore, int reduction) {
    using A = typename Stat<T>::type;
    const int64_t n = N * C;
    for (int64_t e = int64_t(blockIdx.x) * kThreads + threadIdx.x; e < n; e += int64_t(gridDim.x) * kThreads) {
        const int64_t i = e / C, c = e - i * C;
        const int64_t t = static_cast<int64_t>(target[i]);
        A v = 0;
        if (c == t && t != ignore) {
            A g = reduction == 0 ? load_as<A>(dy[i]) : load_as<A>(dy[0]);
            if (reduction == 1) g /= load_as<A>(total[0]);
            v = -(w != nullptr ? load_as<A>(w[t]) : A(1)) * g;
        }
        dx[e] = store_as<T>(v);
    }
}

// -------------------------------------------------------------- dropout --

// Philox-4x32-10, the counter-based generator of Salmon, Moraes, Dror and
// Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011): ten rounds
// of two 32x32 -> 64-bit products mixing a 128-bit counter under a 64-bit key
// bumped by the Weyl constants each round.  Element e of a launch draws
// word e % 4 of the block for counter (e / 4 + offset, 0, 0, 0).
struct Philox4 {
    uint32_t v[4];
};

__device__ __forceinline__ Philox4 philox4x32_10(uint64_t counter, uint64_t key) {
    uint32_t c0 = static_cast<uint32_t>(counter), c1 = static_cast<uint32_t>(counter >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return Philox4{{c0, c1, c2, c3}};
}

// out = keep ? x / (1 - p) : 0 with keep = u >= p, u uniform in [0, 1) on
// 24 bits; mask records keep.  Four elements per generator call.
template <typename T>
__global__ void __launch_bounds__(kThreads) dropout_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                           bool* __restrict__ mask, int64_t n, float p, float scale,
                                                           uint64_t seed, uint64_t offset) {
    using C = typename Stat<T>::type;
    const int64_t groups = (n + 3) / 4;
    for (int64_t g = int64_t(blockIdx.x) * kThreads + threadIdx.x; g < groups; g += int64_t(gridDim.x) * kThreads) {
        const Philox4 r = philox4x32_10(static_cast<uint64_t>(g) + offset, seed);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t e = g * 4 + j;
            if (e >= n) break;
            const float u = static_cast<float>(r.v[j] >> 8) * (1.0f / 16777216.0f);
            const bool keep = u >= p;
            mask[e] = keep;
            out[e] = store_as<T>(keep ? load_as<C>(x[e]) * C(scale) : C(0));
        }
    }
}

// dx = dy * mask * scale.
template <typename T>
__global__ void __launch_bounds__(kThreads) masked_scale_kernel(const T* __restrict__ dy, const bool* __restrict__ mask,
                                                                T* __restrict__ dx, int64_t n, double scale) {
    using C = typename Stat<T>::type;
    for (int64_t e = int64_t(blockIdx.x) * kThreads + threadIdx.x; e < n; e += int64_t(gridDim.x) * kThreads) {
        dx[e] = store_as<T>(mask[e] ? load_as<C>(dy[e]) * C(scale) : C(0));
    }
}

// ---------------------------------------------------------- host side --

const tpb_tensor* opt(const tpb_tensor* t) { return t != nullptr && t->data != nullptr ? t : nullptr; }

bool dense(const tpb_tensor& t) {
    int64_t expect = 1;
    for (int i = t.ndim - 1; i >= 0; --i) {
        if (t.sizes[i] != 1 && t.strides[i] != expect) return false;
        expect *= t.sizes[i];
    }
    return true;
}

void require_dense(const tpb_tensor* t, const char* what) {
    check_tensor(t, what);
    TPB_CHECK(dense(*t), "%s must be contiguous", what);
}

int stat_code(int dtype) { return dtype == TPB_F64 ? TPB_F64 : TPB_F32; }

void fill_or_throw(const tpb_tensor& t, double value, cudaStream_t s) {
    TPB_CHECK(tp_b200_fill(&t, value, 0, s) == 0, "%s", tp_b200_last_error());
}

template <typename T>
void layer_norm_launch(const T* x, T* y, typename Stat<T>::type* mean, typename Stat<T>::type* rstd, const T* w,
                       const T* b, int64_t rows, int64_t D, double eps, cudaStream_t s) {
    constexpr int V = VecWidth<T>::value;
    const bool vec = D % V == 0 && aligned16(x) && aligned16(y) && (w == nullptr || aligned16(w)) &&
                     (b == nullptr || aligned16(b));
    const unsigned grid = static_cast<unsigned>(rows);
    const int64_t nv = D / V;
    if (vec && nv <= kThreads) layer_norm_rows<T, V, 1><<<grid, kThreads, 0, s>>>(x, y, mean, rstd, w, b, D, eps);
    else if (vec && nv <= 2 * kThreads) layer_norm_rows<T, V, 2><<<grid, kThreads, 0, s>>>(x, y, mean, rstd, w, b, D, eps);
    else if (vec && nv <= 4 * kThreads) layer_norm_rows<T, V, 4><<<grid, kThreads, 0, s>>>(x, y, mean, rstd, w, b, D, eps);
    else layer_norm_rows_loop<T><<<grid, kThreads, 0, s>>>(x, y, mean, rstd, w, b, D, eps);
    check_launch("layer_norm");
}

template <typename Fn>
void with_index_type(int dtype, Fn fn) {
    if (dtype == TPB_I64) fn(static_cast<int64_t*>(nullptr));
    else if (dtype == TPB_I32) fn(static_cast<int32_t*>(nullptr));
    else TPB_CHECK(false, "nll_loss: targets must be int64 or int32");
}

}  // namespace
// Mean squared error with its gradient in one pass over (out, target):
//   diff = round(out - target); sq = round(diff * diff); grad = round(diff * s)
// (round: to the storage type, where the separate sub / pow / mul operators
// round), per-block fp32 sums of sq (fp64 for fp64), combined in block order
// by mse_finish: loss = round(sum / n).  V: elements per 16-byte vector (1
// when a pointer is not 16-byte aligned).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) mse_partials(const T* __restrict__ out, const T* __restrict__ target,
                                                         T* __restrict__ grad, typename Stat<T>::type* partial,
                                                         int64_t n, float grad_scale) {
    pdl_entry();
    using A = typename Stat<T>::type;
    using C = typename std::conditional<std::is_same<T, double>::value, double, float>::type;
    using VT = Vec<T, V>;
    A acc = A(0);
    const int64_t nvec = n / V;
    const int64_t stride = int64_t(gridDim.x) * kThreads;
    for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < nvec; i += stride) {
        const VT o = reinterpret_cast<const VT*>(out)[i];
        const VT t = reinterpret_cast<const VT*>(target)[i];
        C fo[V], ft[V], g[V];
        unpack_vec(o, fo);
        unpack_vec(t, ft);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const C d = load_as<C>(store_as<T>(fo[j] - ft[j]));
            acc += A(load_as<C>(store_as<T>(d * d)));
            g[j] = d * C(grad_scale);
        }
        if (grad != nullptr) {
            VT gv;
            pack_vec(g, gv);
            reinterpret_cast<VT*>(grad)[i] = gv;
        }
    }
    if (blockIdx.x == 0) {
        for (int64_t i = nvec * V + threadIdx.x; i < n; i += kThreads) {
            const C d = load_as<C>(store_as<T>(load_as<C>(out[i]) - load_as<C>(target[i])));
            acc += A(load_as<C>(store_as<T>(d * d)));
            if (grad != nullptr) grad[i] = store_as<T>(d * C(grad_scale));
        }
    }
    acc = block_sum(acc);
    if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) mse_finish(const typename Stat<T>::type* __restrict__ partial, int blocks,
                                                       T* __restrict__ loss, double n) {
    pdl_entry();
    using A = typename Stat<T>::type;
    A acc = A(0);
    for (int i = threadIdx.x; i < blocks; i += kThreads) acc += partial[i];
    acc = block_sum(acc);
    if (threadIdx.x == 0) loss[0] = store_as<T>(acc / A(n));
}

}  // namespace tpb

using namespace tpb;

extern "C" {

int tp_b200_layer_norm(const tpb_tensor* y, const tpb_tensor* mean, const tpb_tensor* rstd, const tpb_tensor* x,
                       const tpb_tensor* weight, const tpb_tensor* bias, int64_t normalized_numel, double eps,
                       void* stream) {
    return guarded([&] {
        require_dense(x, "layer_norm input");
        require_dense(y, "layer_norm result");
        require_dense(mean, "layer_norm mean");
        require_dense(rstd, "layer_norm rstd");
        const tpb_tensor* w = opt(weight);
        const tpb_tensor* b = opt(bias);
        if (w) require_dense(w, "layer_norm weight");
        if (b) require_dense(b, "layer_norm bias");
        TPB_CHECK(is_floating(x->dtype), "layer_norm: input must be floating, got %s", dtype_name(x->dtype));
        TPB_CHECK(y->dtype == x->dtype && (!w || w->dtype == x->dtype) && (!b || b->dtype == x->dtype),
                  "layer_norm: input, weight, bias and result must share one dtype");
        TPB_CHECK(mean->dtype == stat_code(x->dtype) && rstd->dtype == mean->dtype,
                  "layer_norm: statistics must be %s", dtype_name(stat_code(x->dtype)));
        const int64_t n = numel_of(*x);
        TPB_CHECK(normalized_numel > 0 && n % normalized_numel == 0, "layer_norm: bad normalized size");
        const int64_t rows = n / normalized_numel;
        TPB_CHECK(numel_of(*y) == n && numel_of(*mean) == rows && numel_of(*rstd) == rows,
                  "layer_norm: result / statistics sizes do not match the input");
        TPB_CHECK((!w || numel_of(*w) == normalized_numel) && (!b || numel_of(*b) == normalized_numel),
                  "layer_norm: weight / bias must have the normalized shape");
        TPB_CHECK(rows < (int64_t(1) << 31), "layer_norm: too many rows");
        if (n == 0) return;
        const int dev = device_of(x->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        TPB_DISPATCH_FLOAT(x->dtype, "layer_norm", {
            using A = typename Stat<scalar_t>::type;
            layer_norm_launch<scalar_t>(static_cast<const scalar_t*>(x->data), static_cast<scalar_t*>(y->data),
                                        static_cast<A*>(mean->data), static_cast<A*>(rstd->data),
                                        w ? static_cast<const scalar_t*>(w->data) : nullptr,
                                        b ? static_cast<const scalar_t*>(b->data) : nullptr, rows,
                                        normalized_numel, eps, s);
        });
    });
}

int tp_b200_layer_norm_backward(const tpb_tensor* dx, const tpb_tensor* dweight, const tpb_tensor* dbias,
                                const tpb_tensor* dy, const tpb_tensor* x, const tpb_tensor* mean,
                                const tpb_tensor* rstd, const tpb_tensor* weight, int64_t normalized_numel,
                                void* stream) {
    return guarded([&] {
        require_dense(dy, "layer_norm_backward grad");
        require_dense(x, "layer_norm_backward input");
        require_dense(mean, "layer_norm_backward mean");
        require_dense(rstd, "layer_norm_backward rstd");
        const tpb_tensor* w = opt(weight);
        const tpb_tensor* gx = opt(dx);
        const tpb_tensor* gw = opt(dweight);
        const tpb_tensor* gb = opt(dbias);
        if (w) require_dense(w, "layer_norm_backward weight");
        if (gx) require_dense(gx, "layer_norm_backward dx");
        if (gw) require_dense(gw, "layer_norm_backward dweight");
        if (gb) require_dense(gb, "layer_norm_backward dbias");
        const int dt = x->dtype;
        TPB_CHECK(is_floating(dt) && dy->dtype == dt && (!w || w->dtype == dt) && (!gx || gx->dtype == dt) &&
                      (!gw || gw->dtype == dt) && (!gb || gb->dtype == dt),
                  "layer_norm_backward: operands must share one floating dtype");
        TPB_CHECK(mean->dtype == stat_code(dt) && rstd->dtype == mean->dtype,
                  "layer_norm_backward: statistics must be %s", dtype_name(stat_code(dt)));
        const int64_t n = numel_of(*x);
        TPB_CHECK(normalized_numel > 0 && n % normalized_numel == 0, "layer_norm_backward: bad normalized size");
        const int64_t rows = n / normalized_numel, D = normalized_numel;
        TPB_CHECK(numel_of(*dy) == n && numel_of(*mean) == rows && numel_of(*rstd) == rows &&
                      (!gx || numel_of(*gx) == n) && (!w || numel_of(*w) == D) && (!gw || numel_of(*gw) == D) &&
                      (!gb || numel_of(*gb) == D),
                  "layer_norm_backward: sizes do not match");
        TPB_CHECK(rows < (int64_t(1) << 31), "layer_norm_backward: too many rows");
        if (n == 0) return;
        const int dev = device_of(x->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        TPB_DISPATCH_FLOAT(dt, "layer_norm_backward", {
            using A = typename Stat<scalar_t>::type;
            const scalar_t* dyp = static_cast<const scalar_t*>(dy->data);
            const scalar_t* xp = static_cast<const scalar_t*>(x->data);
            const A* mp = static_cast<const A*>(mean->data);
            const A* rp = static_cast<const A*>(rstd->data);
            if (gx) {
                layer_norm_bwd_dx<scalar_t><<<static_cast<unsigned>(rows), kThreads, 0, s>>>(
                    dyp, xp, mp, rp, w ? static_cast<const scalar_t*>(w->data) : nullptr,
                    static_cast<scalar_t*>(gx->data), D);
                check_launch("layer_norm_backward_dx");
            }
            if (gw || gb) {
                const int64_t col_blocks = (D + kThreads - 1) / kThreads;
                const int64_t want = int64_t(num_sms(dev)) * 8;
                int splits = static_cast<int>(std::max<int64_t>(
                    1, std::min<int64_t>({(want + col_blocks - 1) / col_blocks, rows, 1024})));
                Scratch partial(sizeof(A) * 2 * size_t(splits) * size_t(D), dev, s);
                layer_norm_bwd_params<scalar_t><<<dim3(static_cast<unsigned>(col_blocks), splits), kThreads, 0, s>>>(
                    dyp, xp, mp, rp, static_cast<A*>(partial.get()), rows, D);
                check_launch("layer_norm_backward_params");
                layer_norm_bwd_params_combine<scalar_t><<<static_cast<unsigned>(col_blocks), kThreads, 0, s>>>(
                    static_cast<const A*>(partial.get()), gw ? static_cast<scalar_t*>(gw->data) : nullptr,
                    gb ? static_cast<scalar_t*>(gb->data) : nullptr, splits, D);
                check_launch("layer_norm_backward_params_combine");
            }
        });
    });
}

int tp_b200_nll_loss(const tpb_tensor* out, const tpb_tensor* total_weight, const tpb_tensor* x,
                     const tpb_tensor* target, const tpb_tensor* weight, int reduction, int64_t ignore_index,
                     void* stream) {
    return guarded([&] {
        check_tensor(out, "nll_loss result");
        check_tensor(total_weight, "nll_loss total_weight");
        check_tensor(x, "nll_loss input");
        check_tensor(target, "nll_loss target");
        const tpb_tensor* w = opt(weight);
        if (w) require_dense(w, "nll_loss weight");
        TPB_CHECK(reduction >= 0 && reduction <= 2, "nll_loss: reduction must be 0 (none), 1 (mean) or 2 (sum)");
        TPB_CHECK(x->ndim == 2 && target->ndim == 1 && target->sizes[0] == x->sizes[0],
                  "nll_loss: input must be (N, C) with (N) targets");
        const int dt = x->dtype;
        TPB_CHECK(is_floating(dt) && out->dtype == dt && total_weight->dtype == dt && (!w || w->dtype == dt),
                  "nll_loss: input, weight and results must share one floating dtype");
        const int64_t N = x->sizes[0], C = x->sizes[1];
        TPB_CHECK(!w || numel_of(*w) == C, "nll_loss: weight must have C elements");
        TPB_CHECK(reduction == 0 ? (out->ndim == 1 && out->sizes[0] == N && out->strides[0] == 1)
                                 : numel_of(*out) == 1,
                  "nll_loss: result shape does not match the reduction");
        TPB_CHECK(target->strides[0] == 1 || N <= 1, "nll_loss: targets must be contiguous");
        const int dev = device_of(x->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        int* err = device_error_word(dev);
        TPB_DISPATCH_FLOAT(dt, "nll_loss", {
            using A = typename Stat<scalar_t>::type;
            scalar_t* o = static_cast<scalar_t*>(out->data);
            scalar_t* tw = static_cast<scalar_t*>(total_weight->data);
            const scalar_t* wp = w ? static_cast<const scalar_t*>(w->data) : nullptr;
            with_index_type(target->dtype, [&](auto tag) {
                using I = std::remove_pointer_t<decltype(tag)>;
                const I* tp = static_cast<const I*>(target->data);
                const int blocks = static_cast<int>(std::max<int64_t>(
                    1, std::min<int64_t>((N + kThreads - 1) / kThreads, int64_t(num_sms(dev)) * 2)));
                Scratch partial(reduction == 0 ? 0 : sizeof(A) * 2 * size_t(blocks), dev, s);
                if (N > 0) {
                    nll_forward<scalar_t, I><<<blocks, kThreads, 0, s>>>(
                        static_cast<const scalar_t*>(x->data), tp, wp, o, static_cast<A*>(partial.get()), N, C,
                        x->strides[0], x->strides[1], ignore_index, reduction, err);
                    check_launch("nll_loss");
                }
                if (reduction == 0) {
                    // A per-sample result reports no total (NNKernels.cpp:352-353).
                    fill_or_throw(*total_weight, 0.0, s);
                } else if (N > 0) {
                    nll_combine<scalar_t><<<1, kThreads, 0, s>>>(static_cast<const A*>(partial.get()), blocks,
                                                                  o, tw, reduction);
                    check_launch("nll_loss_combine");
                } else {
                    // No samples: sum 0, mean 0 / 0 = NaN, total 0.
                    fill_or_throw(*total_weight, 0.0, s);
                    fill_or_throw(*out, reduction == 1 ? NAN : 0.0, s);
                }
            });
        });
    });
}

int tp_b200_nll_loss_backward(const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* target,
                              const tpb_tensor* weight, const tpb_tensor* total_weight, int reduction,
                              int64_t ignore_index, void* stream) {
    return guarded([&] {
        require_dense(dx, "nll_loss_backward dx");
        check_tensor(dy, "nll_loss_backward grad");
        check_tensor(target, "nll_loss_backward target");
        check_tensor(total_weight, "nll_loss_backward total_weight");
        const tpb_tensor* w = opt(weight);
        if (w) require_dense(w, "nll_loss_backward weight");
        TPB_CHECK(reduction >= 0 && reduction <= 2, "nll_loss_backward: bad reduction %d", reduction);
        TPB_CHECK(dx->ndim == 2 && target->ndim == 1 && target->sizes[0] == dx->sizes[0],
                  "nll_loss_backward: dx must be (N, C) with (N) targets");
        const int dt = dx->dtype;
        TPB_CHECK(is_floating(dt) && dy->dtype == dt && total_weight->dtype == dt && (!w || w->dtype == dt),
                  "nll_loss_backward: operands must share one floating dtype");
        const int64_t N = dx->sizes[0], C = dx->sizes[1];
        TPB_CHECK(reduction == 0 ? numel_of(*dy) == N : numel_of(*dy) == 1,
                  "nll_loss_backward: grad shape does not match the reduction");
        TPB_CHECK(dy->ndim <= 1 && (dy->ndim == 0 || dy->strides[0] == 1 || N <= 1),
                  "nll_loss_backward: grad must be contiguous");
        TPB_CHECK(target->strides[0] == 1 || N <= 1, "nll_loss_backward: targets must be contiguous");
        if (N * C == 0) return;
        const int dev = device_of(dx->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        TPB_DISPATCH_FLOAT(dt, "nll_loss_backward", {
            with_index_type(target->dtype, [&](auto tag) {
                using I = std::remove_pointer_t<decltype(tag)>;
                const unsigned grid = static_cast<unsigned>(
                    std::min<int64_t>(blocks_for(N * C, kThreads), int64_t(num_sms(dev)) * 16));
                nll_backward<scalar_t, I><<<grid, kThreads, 0, s>>>(
                    static_cast<scalar_t*>(dx->data), static_cast<const scalar_t*>(dy->data),
                    static_cast<const I*>(target->data), w ? static_cast<const scalar_t*>(w->data) : nullptr,
                    static_cast<const scalar_t*>(total_weight->data), N, C, ignore_index, reduction);
                check_launch("nll_loss_backward");
            });
        });
    });
}

}  // extern "C"

extern "C" {

int tp_b200_dropout(const tpb_tensor* out, const tpb_tensor* mask, const tpb_tensor* x, double p, uint64_t seed,
                    uint64_t offset, void* stream) {
    return guarded([&] {
        require_dense(out, "dropout result");
        require_dense(mask, "dropout mask");
        require_dense(x, "dropout input");
        TPB_CHECK(is_floating(x->dtype) && out->dtype == x->dtype, "dropout: floating input and result of one dtype");
        TPB_CHECK(mask->dtype == TPB_BOOL, "dropout: the mask must be bool");
        TPB_CHECK(p >= 0.0 && p < 1.0, "dropout: probability must be in [0, 1)");
        const int64_t n = numel_of(*x);
        TPB_CHECK(numel_of(*out) == n && numel_of(*mask) == n, "dropout: sizes differ");
        if (n == 0) return;
        const int dev = device_of(x->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const unsigned grid = static_cast<unsigned>(
            std::max<int64_t>(1, std::min<int64_t>(blocks_for((n + 3) / 4, kThreads), int64_t(num_sms(dev)) * 8)));
        TPB_DISPATCH_FLOAT(x->dtype, "dropout", {
            dropout_kernel<scalar_t><<<grid, kThreads, 0, s>>>(
                static_cast<const scalar_t*>(x->data), static_cast<scalar_t*>(out->data),
                static_cast<bool*>(mask->data), n, static_cast<float>(p), static_cast<float>(1.0 / (1.0 - p)),
                seed, offset);
        });
        check_launch("dropout");
    });
}

int tp_b200_masked_scale(const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* mask, double scale,
                         void* stream) {
    return guarded([&] {
        require_dense(dx, "masked_scale result");
        require_dense(dy, "masked_scale grad");
        require_dense(mask, "masked_scale mask");
        TPB_CHECK(is_floating(dy->dtype) && dx->dtype == dy->dtype && mask->dtype == TPB_BOOL,
                  "masked_scale: floating grad and result of one dtype, bool mask");
        const int64_t n = numel_of(*dy);
        TPB_CHECK(numel_of(*dx) == n && numel_of(*mask) == n, "masked_scale: sizes differ");
        if (n == 0) return;
        const int dev = device_of(dy->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const unsigned grid = static_cast<unsigned>(
            std::max<int64_t>(1, std::min<int64_t>(blocks_for(n, kThreads), int64_t(num_sms(dev)) * 16)));
        TPB_DISPATCH_FLOAT(dy->dtype, "masked_scale", {
            masked_scale_kernel<scalar_t><<<grid, kThreads, 0, s>>>(
                static_cast<const scalar_t*>(dy->data), static_cast<const bool*>(mask->data),
                static_cast<scalar_t*>(dx->data), n, scale);
        });
        check_launch("masked_scale");
    });
}

// The MLP step's loss: mean((out - target)^2) into `loss` (one element of
// out's dtype) and, when `grad` is not NULL, grad = (out - target) *
// grad_scale (2 / n for d loss / d out), one read of out and target.
int tp_b200_mse_loss(const tpb_tensor* loss, const tpb_tensor* grad, const tpb_tensor* out,
                     const tpb_tensor* target, double grad_scale, void* stream) {
    return guarded([&] {
        require_dense(out, "mse_loss input");
        require_dense(target, "mse_loss target");
        require_dense(loss, "mse_loss result");
        if (grad != nullptr) require_dense(grad, "mse_loss gradient");
        TPB_CHECK(is_floating(out->dtype) && target->dtype == out->dtype && loss->dtype == out->dtype &&
                      (grad == nullptr || grad->dtype == out->dtype),
                  "mse_loss: floating operands of one dtype");
        const int64_t n = numel_of(*out);
        TPB_CHECK(numel_of(*target) == n && (grad == nullptr || numel_of(*grad) == n),
                  "mse_loss: input, target and gradient sizes differ");
        TPB_CHECK(numel_of(*loss) == 1, "mse_loss: the result is one element");
        TPB_CHECK(n > 0, "mse_loss: empty input");
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const int blocks = static_cast<int>(std::max<int64_t>(
            1, std::min<int64_t>(blocks_for((n + 7) / 8, kThreads), int64_t(num_sms(dev)) * 4)));
        TPB_DISPATCH_FLOAT(out->dtype, "mse_loss", {
            using A = typename Stat<scalar_t>::type;
            constexpr int V = VecWidth<scalar_t>::value;
            Scratch partial(sizeof(A) * size_t(blocks), dev, s);
            const scalar_t* o = static_cast<const scalar_t*>(out->data);
            const scalar_t* t = static_cast<const scalar_t*>(target->data);
            scalar_t* g = grad != nullptr ? static_cast<scalar_t*>(grad->data) : nullptr;
            const bool vec = aligned16(o) && aligned16(t) && (g == nullptr || aligned16(g));
            if (vec) {
                launch_pdl(mse_partials<scalar_t, V>, blocks, kThreads, 0, s, o, t, g,
                           static_cast<A*>(partial.get()), n, static_cast<float>(grad_scale));
            } else {
                launch_pdl(mse_partials<scalar_t, 1>, blocks, kThreads, 0, s, o, t, g,
                           static_cast<A*>(partial.get()), n, static_cast<float>(grad_scale));
            }
            check_launch("mse_partials");
            launch_pdl(mse_finish<scalar_t>, 1, kThreads, 0, s, static_cast<const A*>(partial.get()), blocks,
                       static_cast<scalar_t*>(loss->data), static_cast<double>(n));
            check_launch("mse_finish");
        });
    });
}

}  // extern "C"
