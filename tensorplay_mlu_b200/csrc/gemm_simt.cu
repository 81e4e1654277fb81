// CUDA-core matrix product for the problems the tensor-core path does not
// take: exact fp32 (the "highest" float32 matmul precision,
// BlasKernels.cpp:63-66), float64, integer types, and 16-bit operands whose
// strides or alignment TMA cannot describe.
//
// Classic register-blocked SGEMM structure: a block computes a BM x BN tile,
// staging BK-deep slices of A and B in shared memory (double-buffered
// through registers), each thread accumulating a TM x TN sub-tile split into
// 2 x 2 quadrants so its shared-memory reads are 16-byte and conflict-free.
// Operands are read through their strides, so a transposed view costs only
// coalescing on the load, never a copy.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.h"
#include "device.cuh"
#include "gemm.h"

namespace tpb {

namespace {

template <typename T> struct GemmAcc { using type = float; };
template <> struct GemmAcc<double> { using type = double; };
template <> struct GemmAcc<int8_t> { using type = int64_t; };
template <> struct GemmAcc<uint8_t> { using type = int64_t; };
template <> struct GemmAcc<int16_t> { using type = int64_t; };
template <> struct GemmAcc<int32_t> { using type = int64_t; };
template <> struct GemmAcc<int64_t> { using type = int64_t; };
template <> struct GemmAcc<bool> { using type = int64_t; };

template <typename A, typename T>
__device__ __forceinline__ A gload(const T* p, int64_t off, bool ok) {
    return ok ? load_as<A>(p[off]) : A(0);
}

template <typename To, typename A>
__device__ __forceinline__ To gstore(A v) {
    if constexpr (std::is_same<To, __half>::value || std::is_same<To, __nv_bfloat16>::value) {
        return store_as<To, float>(static_cast<float>(v));
    } else if constexpr (std::is_same<To, bool>::value) {
        return v != A(0);
    } else {
        return static_cast<To>(v);
    }
}

// BM = BN = 16 * TM (256 threads as a 16 x 16 grid), TM even.
//
// Split K (splits > 1, for products too small to fill the device): blockIdx.z
// is batch * splits + split, the block sums K range [split * kchunk,
// (split + 1) * kchunk) and stores its raw accumulator tile into
// partial[(batch * splits + split)][M][N]; gemm_simt_combine adds the splits
// in split order (deterministic) and applies alpha / beta.
template <typename T, int TM, int BK>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmProblem p, int splits, int64_t kchunk,
                                                        typename GemmAcc<T>::type* __restrict__ partial) {
    using A = typename GemmAcc<T>::type;
    constexpr int BM = 16 * TM, BN = 16 * TM;
    constexpr int H = TM / 2;  // quadrant size
    constexpr int LA = BM * BK / 256;  // elements of A each thread loads per slice
    __shared__ __align__(16) A As[2][BK][BM];
    __shared__ __align__(16) A Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int64_t batch = blockIdx.z / splits;
    const int split = blockIdx.z % splits;
    const int64_t k_begin = int64_t(split) * kchunk;
    const int64_t k_end = k_begin + kchunk < p.K ? k_begin + kchunk : p.K;
    const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
    const T* a = static_cast<const T*>(p.a) + batch * p.sa_b;
    const T* b = static_cast<const T*>(p.b) + batch * p.sb_b;

    // Load mapping: along the operand's unit-stride side when it has one.
    const bool a_kmajor = p.sa_k == 1;
    const bool b_nmajor = p.sb_n == 1;
    A ra[LA], rb[LA];
    auto load_slice = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < LA; ++i) {
            const int e = tid + i * 256;
            int mm, kk;
            if (a_kmajor) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
            const int64_t gm = m0 + mm, gk = k0 + kk;
            ra[i] = gload<A>(a, gm * p.sa_m + gk * p.sa_k, gm < p.M && gk < k_end);
            int nn;
            if (b_nmajor) { nn = e % BN; kk = e / BN; } else { kk = e % BK; nn = e / BK; }
            const int64_t gn = n0 + nn, gk2 = k0 + kk;
            rb[i] = gload<A>(b, gk2 * p.sb_k + gn * p.sb_n, gn < p.N && gk2 < k_end);
        }
    };
    auto store_slice = [&](int buf) {
#pragma unroll
        for (int i = 0; i < LA; ++i) {
            const int e = tid + i * 256;
            int mm, kk;
            if (a_kmajor) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
            As[buf][kk][mm] = ra[i];
            int nn;
            if (b_nmajor) { nn = e % BN; kk = e / BN; } else { kk = e % BK; nn = e / BK; }
            Bs[buf][kk][nn] = rb[i];
        }
    };

    A acc[TM][TM];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TM; ++j) acc[i][j] = A(0);

    const int64_t ktiles = (k_end - k_begin + BK - 1) / BK;
    load_slice(k_begin);
    store_slice(0);
    __syncthreads();
    for (int64_t kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) load_slice(k_begin + (kt + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            A fa[TM], fb[TM];
#pragma unroll
            for (int i = 0; i < H; ++i) {
                fa[i] = As[buf][k][ty * H + i];
                fa[H + i] = As[buf][k][BM / 2 + ty * H + i];
                fb[i] = Bs[buf][k][tx * H + i];
                fb[H + i] = Bs[buf][k][BN / 2 + tx * H + i];
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TM; ++j) acc[i][j] += fa[i] * fb[j];
        }
        if (kt + 1 < ktiles) {
            store_slice(buf ^ 1);
        }
        __syncthreads();
    }

    if (splits > 1) {
        A* part = partial + (batch * splits + split) * p.M * p.N;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int64_t gm = m0 + (i < H ? ty * H + i : BM / 2 + ty * H + (i - H));
            if (gm >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TM; ++j) {
                const int64_t gn = n0 + (j < H ? tx * H + j : BN / 2 + tx * H + (j - H));
                if (gn < p.N) part[gm * p.N + gn] = acc[i][j];
            }
        }
        return;
    }
    T* c = static_cast<T*>(p.c) + batch * p.sc_b;
    const T* cin = static_cast<const T*>(p.cin);
    const A alpha = static_cast<A>(p.alpha), beta = static_cast<A>(p.beta);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int64_t gm = m0 + (i < H ? ty * H + i : BM / 2 + ty * H + (i - H));
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TM; ++j) {
            const int64_t gn = n0 + (j < H ? tx * H + j : BN / 2 + tx * H + (j - H));
            if (gn >= p.N) continue;
            A v = alpha * acc[i][j];
            if (cin != nullptr) {
                v += beta * load_as<A>(cin[batch * p.sci_b + gm * p.sci_m + gn * p.sci_n]);
            }
            c[gm * p.sc_m + gn] = gstore<T>(v);
        }
    }
}

// out[b][m][n] = alpha * sum over splits (in split order) + beta * cin.
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_combine(GemmProblem p, int splits,
                                                         const typename GemmAcc<T>::type* __restrict__ partial) {
    using A = typename GemmAcc<T>::type;
    const int64_t mn = p.M * p.N;
    const int64_t total = mn * p.batch;
    const A alpha = static_cast<A>(p.alpha), beta = static_cast<A>(p.beta);
    const T* cin = static_cast<const T*>(p.cin);
    for (int64_t i = int64_t(blockIdx.x) * 256 + threadIdx.x; i < total; i += int64_t(gridDim.x) * 256) {
        const int64_t batch = i / mn, r = i - batch * mn, m = r / p.N, n = r - m * p.N;
        const A* src = partial + batch * splits * mn + r;
        A v = src[0];
        for (int s = 1; s < splits; ++s) v += src[int64_t(s) * mn];
        v = alpha * v;
        if (cin != nullptr) v += beta * load_as<A>(cin[batch * p.sci_b + m * p.sci_m + n * p.sci_n]);
        static_cast<T*>(p.c)[batch * p.sc_b + m * p.sc_m + n] = gstore<T>(v);
    }
}

template <typename T, int TM>
void launch_tiles(const GemmProblem& p, int splits, int64_t kchunk, typename GemmAcc<T>::type* partial,
                  cudaStream_t stream) {
    constexpr int BM = 16 * TM;
    dim3 grid(static_cast<unsigned>((p.N + BM - 1) / BM), static_cast<unsigned>((p.M + BM - 1) / BM),
              static_cast<unsigned>(p.batch * splits));
    TPB_CHECK(grid.y < 65536 && grid.z < 65536, "gemm: problem too large for the CUDA-core kernel");
    gemm_simt_kernel<T, TM, 8><<<grid, 256, 0, stream>>>(p, splits, kchunk, partial);
    check_launch("gemm_simt");
}

// Tile size and K splits.  Large problems: 128 x 128 tiles (64 x 64 for
// 8-byte accumulators), one pass.  Problems whose tiles do not cover the
// SMs -- the small, latency-bound products -- take 64 x 64 tiles and split K
// into chunks of at least 64 until about two blocks per SM are busy, then
// combine the splits in a second, element-wise pass.
template <typename T>
void launch_simt(const GemmProblem& p, int dev, cudaStream_t stream) {
    using A = typename GemmAcc<T>::type;
    constexpr bool wide = sizeof(A) == 8;
    const int64_t sms = num_sms(dev);
    auto tiles = [&](int64_t bm) { return ((p.M + bm - 1) / bm) * ((p.N + bm - 1) / bm) * p.batch; };
    if (!wide && tiles(128) >= sms) {
        launch_tiles<T, 8>(p, 1, p.K, nullptr, stream);
        return;
    }
    const int64_t t64 = tiles(64);
    int splits = 1;
    if (t64 < sms) {
        const int64_t want = (2 * sms + t64 - 1) / t64;
        splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({want, p.K / 64, 32})));
    }
    if (splits == 1 || p.batch * splits >= 65536) {
        launch_tiles<T, 4>(p, 1, p.K, nullptr, stream);
        return;
    }
    const int64_t kchunk = ((p.K + splits - 1) / splits + 7) / 8 * 8;
    splits = static_cast<int>((p.K + kchunk - 1) / kchunk);
    Scratch partial(sizeof(A) * size_t(splits) * size_t(p.batch) * size_t(p.M) * size_t(p.N), dev, stream);
    launch_tiles<T, 4>(p, splits, kchunk, static_cast<A*>(partial.get()), stream);
    const int64_t total = p.M * p.N * p.batch;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, sms * 8));
    gemm_simt_combine<T><<<grid, 256, 0, stream>>>(p, splits, static_cast<const A*>(partial.get()));
    check_launch("gemm_simt_combine");
}

}  // namespace

void gemm_simt(const GemmProblem& p, int dev, cudaStream_t stream) {
    TPB_DISPATCH_ALL(p.dtype, "gemm", { launch_simt<scalar_t>(p, dev, stream); });
}

}  // namespace tpb
