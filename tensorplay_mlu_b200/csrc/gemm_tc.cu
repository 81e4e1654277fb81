// Tensor-core matrix product for sm_100a: tcgen05.mma with TMEM accumulators,
// operands staged by TMA into 128-byte-swizzled shared memory, and a
// persistent, warp-specialised CTA per SM (tensorplay-mlu runs these
// products on cnnlMatMul_v2 / cnnlStrideBatchMatMul_v3, BlasKernels.cpp:202-242).
//
// CTA layout (320 threads, one CTA per SM):
//   warp 0      TMA producer: one elected thread fills a ring of kStages
//               shared-memory stages (A: 128 x 64 bf16, B: BN x 64 bf16) and
//               arms each stage's "full" mbarrier with the byte count;
//   warp 1      MMA issuer: allocates TMEM (2 accumulators of 128 x BN fp32),
//               one elected thread issues 4 x tcgen05.mma (K = 16 each) per
//               stage and releases the stage with tcgen05.commit on its
//               "empty" mbarrier; after a tile's last stage it commits to the
//               accumulator's "full" barrier;
//   warps 2..9  epilogue: two warps per TMEM lane quadrant (the lanes a
//               warp may access), each taking half of the columns:
//               tcgen05.ld 32 columns at a time (the next chunk's load
//               issued before the current one is stored), apply
//               alpha/beta/addend, convert and store; then release the
//               accumulator.
// Two accumulators let the epilogue of tile i overlap the mainloop of
// tile i+1.  Tiles are visited in groups of kGroupM row-tiles so the CTAs in
// flight share A and B panels in L2.
//
// Transposed operands are read in place: an operand whose unit stride is on
// the M (or N) side is loaded as 64-element MN-major chunks and described to
// the MMA as MN-major (the instruction descriptor's transpose bits), the way
// as_operand (BlasKernels.cpp:40-54) passes a transpose flag.
//
// Every wait is bounded (kWaitNs): a role that gives up records an error
// code in the library's device error word, tells the other roles through
// shared memory, drains what it has in flight and leaves; the host reports
// it through tp_b200_take_device_error.  No TMA multicast is used.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>

#include "common.h"
#include "device.cuh"
#include "ew_common.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace tpb {

void copy_impl(const tpb_tensor& dst, const tpb_tensor& src, cudaStream_t stream, int dev);

namespace {

constexpr int kTcThreads = 320;  // warp 0 producer, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpilogueWarps = 8;
constexpr int kBM = 128;
constexpr int kGroupM = 16;

// Error codes written to the device error word (role that gave up).
constexpr int kErrProducer = 0x7c01;
constexpr int kErrMma = 0x7c02;
constexpr int kErrEpilogue = 0x7c03;

// ------------------------------------------------------- PTX wrappers --

// Wait for the phase of parity `parity` to complete.  False when it did not
// within kWaitNs, or when another role has already given up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - start > kWaitNs) {
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

template <bool TF32>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                     uint32_t accumulate) {
    if constexpr (TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns of TMEM into 32 registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format: start
// address, leading / stride byte offsets in 16-byte units, version 1 at bit
// 46, layout type 2 = SWIZZLE_128B at bits 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// ------------------------------------------------------------ kernel --

struct TcParams {
    int M, N, K, batch;
    int m_tiles, n_tiles, k_blocks, num_tiles;
    int a_mn, b_mn;   // operand stored MN-major (unit stride on M / N)
    int batched;      // 3-D tensor maps
    uint32_t idesc;
    void* c;
    int64_t sc_b, sc_m;
    const void* cin;
    int64_t sci_b, sci_m, sci_n;
    float alpha, beta;
    int vec_store;    // 16-byte stores allowed
    int tma_store;    // result written through the C tensor map (TMA stores)
    const void* aux;  // kEpiGeluBackward: the activation's input h [M x N], row stride saux_m
    int64_t saux_m;
    // CTA-pair kernel: tiles claimed at run time from this counter word (see
    // next_pair_tile), or in a fixed order when null.
    unsigned long long* sched;
    uint32_t epoch;
    // L2 eviction priority (CTA-pair kernel): 0 the plain (unhinted)
    // instructions; l2_operands 1 keeps A / B panels (evict_last);
    // l2_stream 1 lets the epilogue's result stores and activation-input
    // loads go first (evict_first); 2 the hinted instructions with
    // evict_normal (A/B measurements).
    int l2_operands, l2_stream;
    int* err;
};

// Epilogue forms (template argument of the CTA-pair kernel).
//   kEpiPlain         C = alpha * acc + beta * addend
//   kEpiGelu          v = alpha * acc + beta * addend; the aux map receives v
//                     rounded to T, C receives gelu of that rounded v
//   kEpiGeluBackward  d = alpha * acc rounded to T; C = gelu_backward(d, h),
//                     h read from p.aux
// The activation math is the elementwise kernels' own (unary_apply /
// unary_backward_apply, narrow-type fast forms), applied to the same rounded
// values, so a fused product gives the bits of the product followed by the
// separate activation kernel.
constexpr int kEpiPlain = 0;
constexpr int kEpiGelu = 1;
constexpr int kEpiGeluBackward = 2;

// Element traits: 128 bytes of K per stage row in every case.
template <typename T> struct TcElem;
template <> struct TcElem<__nv_bfloat16> {
    static constexpr int kES = 2;
    static constexpr bool kTF32 = false;
};
template <> struct TcElem<__half> {
    static constexpr int kES = 2;
    static constexpr bool kTF32 = false;
};
template <> struct TcElem<float> {
    static constexpr int kES = 4;
    static constexpr bool kTF32 = true;
};

template <int BN> struct TcShape {
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kTmemCols = 2 * BN;  // two accumulators (power of two)
};

// One operand's share of a pipeline stage: `rows` rows (M or N) by kEPR
// K-elements, written in the 128-byte-swizzled layout the MMA descriptors
// describe.  K-major: 64-row boxes (dst row r at r * 128 B).  MN-major: boxes
// of kEPR (MN) x kEPR (K), one per kEPR-wide MN chunk (chunk j at j * kChunk).
// The layout and batching are compile-time so the producer's loop is
// straight-line code.
constexpr int kBoxRows = 64;

template <int ES, bool MN, bool BATCHED, bool PAIR>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap* map, uint32_t bar, int mn0, int k0,
                                             int b, int rows) {
    constexpr int kEPR = 128 / ES;
    constexpr uint32_t kChunk = kEPR * 128;
    if constexpr (MN) {
        for (int j = 0; j < rows / kEPR; ++j) {
            if constexpr (PAIR) {
                if constexpr (BATCHED) tma_load_3d_pair(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0, b);
                else tma_load_2d_pair(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0);
            } else {
                if constexpr (BATCHED) tma_load_3d(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0, b);
                else tma_load_2d(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0);
            }
        }
    } else {
        for (int j = 0; j < rows / kBoxRows; ++j) {
            if constexpr (PAIR) {
                if constexpr (BATCHED) tma_load_3d_pair(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows, b);
                else tma_load_2d_pair(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows);
            } else {
                if constexpr (BATCHED) tma_load_3d(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows, b);
                else tma_load_2d(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows);
            }
        }
    }
}

// The CTA-pair form of load_operand with an L2 eviction-priority policy.
template <int ES, bool MN, bool BATCHED>
__device__ __forceinline__ void load_operand_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int mn0, int k0,
                                                  int b, int rows, uint64_t policy, bool hinted) {
    if (!hinted) {
        load_operand<ES, MN, BATCHED, true>(dst, map, bar, mn0, k0, b, rows);
        return;
    }
    constexpr int kEPR = 128 / ES;
    constexpr uint32_t kChunk = kEPR * 128;
    if constexpr (MN) {
        for (int j = 0; j < rows / kEPR; ++j) {
            if constexpr (BATCHED) tma_load_3d_pair_hint(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0, b, policy);
            else tma_load_2d_pair_hint(dst + j * kChunk, map, bar, mn0 + j * kEPR, k0, policy);
        }
    } else {
        for (int j = 0; j < rows / kBoxRows; ++j) {
            if constexpr (BATCHED) tma_load_3d_pair_hint(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows, b,
                                                         policy);
            else tma_load_2d_pair_hint(dst + j * kBoxRows * 128, map, bar, k0, mn0 + j * kBoxRows, policy);
        }
    }
}

// Per epilogue warp: one 32 x 32 tile of the result type, staged for a TMA
// store (64-byte-swizzled rows for 16-bit types, 128-byte for fp32).
template <typename T>
__host__ __device__ constexpr size_t staging_bytes() {
    return size_t(32) * 32 * sizeof(T);
}

template <typename T, int BN>
constexpr size_t tc_smem_bytes() {
    return size_t(TcShape<BN>::kStages) * (kBM * 128 + BN * 128) + kEpilogueWarps * staging_bytes<T>() + 1024 + 256;
}

__device__ __forceinline__ void tile_coords(const TcParams& p, int tile, int& b, int& mt, int& nt) {
    const int per_batch = p.m_tiles * p.n_tiles;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group = kGroupM * p.n_tiles;
    const int g = r / group;
    const int first_m = g * kGroupM;
    const int gsize = min(p.m_tiles - first_m, kGroupM);
    const int q = r - g * group;
    mt = first_m + q % gsize;
    nt = q / gsize;
}

// v[j] += beta * addend[n_base + j] for one 32-column chunk of a row.  An
// addend with unit column stride whose chunk lies inside N on a 16-byte
// boundary is read as 16-byte vectors (for a bias row every lane reads the
// same address: a broadcast), not element by element; the arithmetic is the
// same FFMA either way.
template <typename T>
__device__ __forceinline__ void add_addend_chunk(const TcParams& p, const T* crow_in, int64_t n_base, float (&v)[32]) {
    constexpr int kPer = 16 / int(sizeof(T));
    if (p.sci_n == 1 && n_base + 32 <= p.N && (reinterpret_cast<uintptr_t>(crow_in + n_base) & 15u) == 0) {
        const Vec<T, kPer>* src = reinterpret_cast<const Vec<T, kPer>*>(crow_in + n_base);
#pragma unroll
        for (int q = 0; q < 32 / kPer; ++q) {
            float f[kPer];
            unpack_vec(src[q], f);
#pragma unroll
            for (int j = 0; j < kPer; ++j) v[q * kPer + j] = fmaf(p.beta, f[j], v[q * kPer + j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (n_base + j < p.N) v[j] = fmaf(p.beta, load_as<float>(crow_in[(n_base + j) * p.sci_n]), v[j]);
        }
    }
}

// The epilogue of one accumulator: this warp's 32 rows (its TMEM lane
// quadrant, t_rows = TMEM address of row 0 / column 0 of the accumulator)
// for columns [col0, col0 + NCOL).  The load of chunk c + 1 is issued before
// chunk c is converted and stored, so TMEM reads overlap the global stores.
template <typename T, int NCOL>
__device__ __forceinline__ void store_accumulator(const TcParams& p, uint32_t t_rows, int col0, int b, int64_t gm,
                                                  int64_t n_tile0, bool row_ok) {
    constexpr int kChunks = NCOL / 32;
    T* crow = static_cast<T*>(p.c) + b * p.sc_b + gm * p.sc_m;
    const T* cin = static_cast<const T*>(p.cin);
    uint32_t r[2][32];
    __syncwarp();
    tmem_ld32(t_rows + col0, r[0]);
#pragma unroll
    for (int chunk = 0; chunk < kChunks; ++chunk) {
        tmem_wait_ld();
        if (chunk + 1 < kChunks) tmem_ld32(t_rows + col0 + (chunk + 1) * 32, r[(chunk + 1) & 1]);
        const uint32_t* rc = r[chunk & 1];
        const int64_t n_base = n_tile0 + col0 + chunk * 32;
        if (row_ok && n_base < p.N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(rc[j]);
            if (cin != nullptr) add_addend_chunk<T>(p, cin + b * p.sci_b + gm * p.sci_m, n_base, v);
            if (p.vec_store && n_base + 32 <= p.N) {
                constexpr int V = 16 / sizeof(T);
#pragma unroll
                for (int j = 0; j < 32; j += V) {
                    Vec<T, V> o;
#pragma unroll
                    for (int q = 0; q < V; ++q) o.v[q] = store_as<T>(v[j + q]);
                    *reinterpret_cast<Vec<T, V>*>(crow + n_base + j) = o;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (n_base + j < p.N) crow[n_base + j] = store_as<T>(v[j]);
                }
            }
        }
    }
}

// h[n_base .. n_base + 32) of one row of the activation input, as floats
// (16-byte vectors when the chunk is inside N on a 16-byte boundary; zero
// past N).
template <typename T>
__device__ __forceinline__ void load_aux_chunk(const TcParams& p, const T* row, int64_t n_base, float (&z)[32],
                                               uint64_t policy, bool hinted) {
    constexpr int kPer = 16 / int(sizeof(T));
    if (n_base + 32 <= p.N && (reinterpret_cast<uintptr_t>(row + n_base) & 15u) == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(row + n_base);
#pragma unroll
        for (int q = 0; q < 32 / kPer; ++q) {
            const uint4 raw = hinted ? ld_global_v4_hint(src + q, policy) : src[q];
            float f[kPer];
            unpack_vec(*reinterpret_cast<const Vec<T, kPer>*>(&raw), f);
#pragma unroll
            for (int j = 0; j < kPer; ++j) z[q * kPer + j] = f[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] = n_base + j < p.N ? load_as<float>(row[n_base + j]) : 0.0f;
    }
}

// gelu_backward on two lanes: the scalar narrow-type form of
// unary_backward_apply (Phi(z) + z phi(z) with phi from ex2.approx), each
// multiply and fused multiply-add as its two-lane instruction, which rounds
// each lane exactly as the scalar one does.
__device__ __forceinline__ float2 gelu_backward_narrow2(float2 dy, float2 z) {
    float2 t = __fmul2_rn(z, z);
    t = __fmul2_rn(t, f2(-0.72134752044448170368f));
    float2 e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(t.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(t.y));
    const float2 u = __fmul2_rn(z, f2(0.39894228040143267794f));
    return __fmul2_rn(dy, __ffma2_rn(u, e, phi_narrow2(z)));
}

// One 32 x 32 chunk into a warp's staging tile, rows swizzled the way the C
// tensor map expects (64-byte rows for 16-bit types, 128-byte for fp32), so
// the 32 lanes' 16-byte writes hit distinct banks.
template <typename T>
__device__ __forceinline__ void stage_chunk(uint8_t* stage, int lane, const Vec<T, 32>& packed) {
    constexpr int kRowBytes = 32 * int(sizeof(T));
    constexpr int kVecs = kRowBytes / 16;
    const uint4* src = reinterpret_cast<const uint4*>(&packed);
    uint8_t* row = stage + lane * kRowBytes;
#pragma unroll
    for (int q = 0; q < kVecs; ++q) {
        const int phys = kRowBytes == 64 ? (q ^ ((lane >> 1) & 3)) : (q ^ (lane & 7));
        *reinterpret_cast<uint4*>(row + phys * 16) = src[q];
    }
}

// The same through shared memory and a TMA store: each chunk of 32 rows x
// 32 columns is converted into this warp's staging tile, then one lane
// stores the whole tile asynchronously in full lines.  TMA clips the tile at
// M and N.  row0: the warp's first row in C.  EPI selects the epilogue form
// (kEpiGelu also stores the pre-activation through tmAux, from a second
// staging tile at stage2).
template <typename T, int NCOL, bool BATCHED, int EPI = kEpiPlain>
__device__ __forceinline__ void store_accumulator_tma(const TcParams& p, const CUtensorMap* tmC, uint8_t* stage,
                                                      uint32_t t_rows, int col0, int b, int64_t gm, int64_t row0,
                                                      int64_t n_tile0, bool row_ok,
                                                      const CUtensorMap* tmAux = nullptr,
                                                      uint8_t* stage2 = nullptr) {
    constexpr int kChunks = NCOL / 32;
    constexpr bool kFast = Narrow<T>::value;
    const int lane = threadIdx.x & 31;
    const T* cin = static_cast<const T*>(p.cin);
    const T* aux_row = nullptr;
    if constexpr (EPI == kEpiGeluBackward) aux_row = static_cast<const T*>(p.aux) + gm * p.saux_m;
    const bool hint = p.l2_stream != 0;
    const uint64_t pol = p.l2_stream == 1 ? l2_policy_evict_first() : l2_policy_evict_normal();
    uint32_t r[2][32];
    __syncwarp();
    tmem_ld32(t_rows + col0, r[0]);
#pragma unroll
    for (int chunk = 0; chunk < kChunks; ++chunk) {
        tmem_wait_ld();
        if (chunk + 1 < kChunks) tmem_ld32(t_rows + col0 + (chunk + 1) * 32, r[(chunk + 1) & 1]);
        const uint32_t* rc = r[chunk & 1];
        const int64_t n_base = n_tile0 + col0 + chunk * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = p.alpha * __uint_as_float(rc[j]);
        if (cin != nullptr && row_ok) add_addend_chunk<T>(p, cin + b * p.sci_b + gm * p.sci_m, n_base, v);
        Vec<T, 32> packed;
        Vec<T, 32> packed2;
        if constexpr (EPI == kEpiGelu) {
            // packed2: the pre-activation, rounded; packed: gelu of it.
            pack_vec(v, packed2);
            float h[32];
            unpack_vec(packed2, h);
            if constexpr (kFast) {
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 x = make_float2(h[j], h[j + 1]);
                    const float2 g = __fmul2_rn(x, phi_narrow2(x));
                    v[j] = g.x;
                    v[j + 1] = g.y;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = unary_apply<float, kFast>(TPB_GELU, h[j], 0.0f);
            }
        } else if constexpr (EPI == kEpiGeluBackward) {
            pack_vec(v, packed2);
            float d[32], z[32];
            unpack_vec(packed2, d);
            if (row_ok) {
                load_aux_chunk<T>(p, aux_row, n_base, z, pol, hint);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) z[j] = 0.0f;
            }
            if constexpr (kFast) {
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float2 g = gelu_backward_narrow2(make_float2(d[j], d[j + 1]), make_float2(z[j], z[j + 1]));
                    v[j] = g.x;
                    v[j + 1] = g.y;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    v[j] = unary_backward_apply<float, kFast>(TPB_GELU_BACKWARD, d[j], z[j], 0.0f);
                }
            }
        }
        pack_vec(v, packed);
        // The previous stores from this warp's staging tiles have finished
        // reading them.
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
        stage_chunk<T>(stage, lane, packed);
        if constexpr (EPI == kEpiGelu) stage_chunk<T>(stage2, lane, packed2);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && n_base < p.N && row0 < p.M) {
            if (hint) {
                if constexpr (BATCHED) tma_store_3d_hint(tmC, smem_addr(stage), int(n_base), int(row0), b, pol);
                else tma_store_2d_hint(tmC, smem_addr(stage), int(n_base), int(row0), pol);
                if constexpr (EPI == kEpiGelu) tma_store_2d_hint(tmAux, smem_addr(stage2), int(n_base), int(row0), pol);
            } else {
                if constexpr (BATCHED) tma_store_3d(tmC, smem_addr(stage), int(n_base), int(row0), b);
                else tma_store_2d(tmC, smem_addr(stage), int(n_base), int(row0));
                if constexpr (EPI == kEpiGelu) tma_store_2d(tmAux, smem_addr(stage2), int(n_base), int(row0));
            }
            bulk_commit_group();
        }
    }
}

template <typename T, int BN, bool A_MN, bool B_MN, bool BATCHED>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC,
                   const TcParams p) {
    using E = TcElem<T>;
    constexpr int kStages = TcShape<BN>::kStages;
    constexpr int kTmemCols = TcShape<BN>::kTmemCols;
    constexpr int kEPR = 128 / E::kES;             // elements per 128-byte row (K per stage)
    constexpr int kUmmaK = 32 / E::kES;            // K per instruction
    constexpr int kKSteps = kEPR / kUmmaK;         // instructions per stage (4)
    constexpr uint32_t kABytes = kBM * 128;        // A stage bytes
    constexpr uint32_t kBBytes = BN * 128;         // B stage bytes
    constexpr uint32_t kChunk = kEPR * 128;        // one MN-major chunk: kEPR rows of K x 128 B

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + kStages * kABytes;
    uint8_t* staging = smem_b + kStages * kBBytes;  // kEpilogueWarps tiles for TMA stores
    uint64_t* bars = reinterpret_cast<uint64_t*>(staging + kEpilogueWarps * staging_bytes<T>());
    uint64_t* full = bars;
    uint64_t* empty = bars + kStages;
    uint64_t* acc_full = bars + 2 * kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_addr(&acc_full[a]), 1);
            mbar_init(smem_addr(&acc_empty[a]), kEpilogueWarps);
        }
        mbar_init(smem_addr(drain), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(const_cast<uint32_t*>(tmem_slot)), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // set-up above overlaps the previous kernel; memory access starts here

    if (warp == 0) {
        // ---------------------------------------------------- producer --
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
                int b, mt, nt;
                tile_coords(p, tile, b, mt, nt);
                const int m0 = mt * kBM, n0 = nt * BN;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = smem_addr(&full[stage]);
                    mbar_expect_tx(fb, kABytes + kBBytes);
                    const uint32_t da = smem_addr(smem_a + stage * kABytes);
                    const uint32_t db = smem_addr(smem_b + stage * kBBytes);
                    const int k0 = kb * kEPR;
                    load_operand<E::kES, A_MN, BATCHED, false>(da, &tmA, fb, m0, k0, b, kBM);
                    load_operand<E::kES, B_MN, BATCHED, false>(db, &tmB, fb, n0, k0, b, BN);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                atomicExch(p.err, kErrProducer);
                // Let the loads already issued land before the CTA leaves:
                // every stage's most recent phase completes once its bytes do.
                for (int s = 0; s < kStages; ++s) {
                    const uint64_t start = global_ns();
                    while (!mbar_try_wait(smem_addr(&full[s]), (s < stage) ? phase : phase ^ 1)) {
                        if (global_ns() - start > kWaitNs) break;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA issuer --
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            constexpr uint32_t a_lbo = A_MN ? kChunk : 16;
            constexpr uint32_t b_lbo = B_MN ? kChunk : 16;
            constexpr uint32_t a_kstep = A_MN ? kUmmaK * 128 : 32;
            constexpr uint32_t b_kstep = B_MN ? kUmmaK * 128 : 32;
            for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(smem_addr(&acc_empty[acc]), acc_phase ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(smem_addr(&full[stage]), phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(smem_a + stage * kABytes);
                    const uint32_t sb = smem_addr(smem_b + stage * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kKSteps; ++kk) {
                        const uint64_t ad = sw128_desc(sa + kk * a_kstep, a_lbo, 1024);
                        const uint64_t bd = sw128_desc(sb + kk * b_kstep, b_lbo, 1024);
                        umma<E::kTF32>(d_tmem, ad, bd, p.idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(smem_addr(&empty[stage]));
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(smem_addr(&acc_full[acc]));
            }
            if (!ok) atomicExch(p.err, kErrMma);
            // Drain: every MMA issued by this thread completes before TMEM
            // is released.
            umma_commit(smem_addr(drain));
            const uint64_t start = global_ns();
            while (!mbar_try_wait(smem_addr(drain), 0)) {
                if (global_ns() - start > kWaitNs) break;
            }
        }
    } else {
        // --------------------------------------------------- epilogue --
        // Warps 2-9: lane quadrant warp & 3 (the TMEM lanes a warp may read),
        // column half (warp - 2) / 4.
        const int quad = warp & 3;
        const int half = (warp - 2) / 4;
        const int row_in_tile = quad * 32 + lane;
        int local = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(smem_addr(&acc_full[acc]), acc_phase, abort_flag)) {
                if (lane == 0) atomicExch(p.err, kErrEpilogue);
                break;
            }
            tc_fence_after();
            int b, mt, nt;
            tile_coords(p, tile, b, mt, nt);
            const int64_t gm = int64_t(mt) * kBM + row_in_tile;
            const uint32_t t_rows = tmem_base + (uint32_t(quad * 32) << 16) + acc * BN;
            if (p.tma_store) {
                store_accumulator_tma<T, BN / 2, BATCHED>(p, &tmC, staging + (warp - 2) * staging_bytes<T>(), t_rows,
                                                          half * (BN / 2), b, gm, gm - lane, int64_t(nt) * BN,
                                                          gm < p.M);
            } else {
                store_accumulator<T, BN / 2>(p, t_rows, half * (BN / 2), b, gm, int64_t(nt) * BN, gm < p.M);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(smem_addr(&acc_empty[acc]));
        }
        // The TMA stores this warp issued are complete before the CTA leaves.
        if (lane == 0) bulk_wait_group0();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------- 2-SM (CTA pair) kernel --
//
// A cluster of two CTAs on two SMs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA stages its own 128 rows of A
// and its own 128 columns of B (32 KiB per 64-deep K step instead of 48 KiB
// for a 128 x 256 tile on one SM, so 6 stages fit and L2 traffic per flop
// drops by a third), the leader CTA's single MMA thread drives both SMs'
// tensor cores, and each CTA's TMEM holds its 128 output rows.
//   * Both CTAs' TMA loads (.cta_group::2, no multicast) complete on the
//     leader's "full" barrier, which only the leader arms, with the pair's
//     total bytes.
//   * The leader's commits are multicast to the same barrier in both CTAs:
//     "empty" (the stage may be refilled in both) and "acc_full".
//   * Both CTAs' epilogue warps arrive on the leader's "acc_empty" (count 16).
// Waits are bounded as in the 1-SM kernel; teardown is a cluster barrier
// followed by the paired TMEM release.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared::cluster address of the variable at `local_addr` in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}


__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

template <bool TF32>
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    if constexpr (TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrive on the barrier at `bar`'s offset in both CTAs of the pair once the
// MMAs issued so far are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(mask)
        : "memory");
}

constexpr int kPairStages = 6;
constexpr int kPairBM = 256;  // rows per CTA pair (128 per CTA)
constexpr int kPairBN = 256;  // columns per CTA pair (each CTA stages 128 of B)

// Staging tiles per epilogue warp: two when the epilogue writes two results.
template <int EPI>
__host__ __device__ constexpr int staging_tiles() {
    return EPI == kEpiGelu ? 2 : 1;
}

template <typename T, int EPI = kEpiPlain>
constexpr size_t tc2_smem_bytes() {
    return size_t(kPairStages) * (128 * 128 + 128 * 128) + kEpilogueWarps * staging_tiles<EPI>() * staging_bytes<T>() +
           1024 + 512;
}

// Tile scheduling of the CTA-pair kernel.  In the fixed order every role
// computes the sequence itself.  With run-time claims the leader CTA's
// scheduler thread decides which tile the pair computes next and publishes
// it through a ring
// of kSchedDepth slots (in both CTAs' shared memory) to its consumers: both
// CTAs' producers, the leader's MMA thread and both CTAs' epilogue warps; -1
// ends the sequence.  Each slot's "empty" barrier (the leader's) counts
// those consumers' arrivals.
constexpr int kSchedDepth = 4;
constexpr int kSchedConsumers = 2 + 1 + 2 * kEpilogueWarps;
// The CTA-pair kernel's warps: 0 TMA producer, 1 MMA issuer, 2-9 epilogue,
// 10 tile scheduler (leader CTA).  352 threads take the same register
// allocation as 320 (12-warp granularity).
constexpr int kTc2Threads = 352;
constexpr int kSchedWarp = 10;
// Run-time claims are made just in time: the leader's producer asks for the
// next tile kClaimLead k-blocks before the end of its current one, so a
// claim's round trip to L2 is hidden behind those loads while the tiles in
// flight across the device stay one wave of consecutive claims (claiming
// further ahead spreads them over several waves' worth of operand panels
// and measured 10-16% slower from the lost L2 reuse).
constexpr int kClaimLead = 8;

// The next tile of a cluster: in a fixed order (cluster_id + iter *
// num_clusters) when p.sched is null; otherwise claimed from the counter word
// p.sched, whose high half holds the epoch of the launch that last claimed
// (each launch on the word has its own) and low half the claims made in that
// epoch, so a launch's first claim restarts the count whatever an earlier
// launch left behind.  Claims arrive in increasing order, so clusters that
// start late (SMs busy with a concurrent kernel, e.g. a collective) take
// fewer tiles instead of holding back tiles assigned to them in advance.
__device__ __forceinline__ int next_pair_tile(const TcParams& p, int cluster_id, int num_clusters, int iter) {
    if (p.sched == nullptr) {
        const int64_t t = int64_t(cluster_id) + int64_t(iter) * num_clusters;
        return t < p.num_tiles ? int(t) : -1;
    }
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(p.sched);
    unsigned long long assumed;
    uint32_t claim;
    do {
        assumed = old;
        claim = uint32_t(assumed >> 32) == p.epoch ? uint32_t(assumed) : 0u;
        const unsigned long long next = (static_cast<unsigned long long>(p.epoch) << 32) | (claim + 1u);
        old = atomicCAS(p.sched, assumed, next);
    } while (old != assumed);
    return claim < uint32_t(p.num_tiles) ? int(claim) : -1;
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait with cluster-scope acquire (the slot was written by the other
// CTA of the pair).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - start > kWaitNs) {
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void st_cluster_s32(uint32_t cluster_addr, int v) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void tile_coords_pair(const TcParams& p, int tile, int& b, int& mt, int& nt,
                                                 int group_m) {
    const int per_batch = p.m_tiles * p.n_tiles;
    b = tile / per_batch;
    const int r = tile - b * per_batch;
    const int group = group_m * p.n_tiles;
    const int g = r / group;
    const int first_m = g * group_m;
    const int gsize = min(p.m_tiles - first_m, group_m);
    const int q = r - g * group;
    mt = first_m + q % gsize;
    nt = q / gsize;
}

template <typename T, bool A_MN, bool B_MN, bool BATCHED, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTc2Threads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAux,
                    const TcParams p, const int group_m) {
    using E = TcElem<T>;
    constexpr int kStages = kPairStages;
    constexpr int kTmemCols = 2 * kPairBN;
    constexpr int kEPR = 128 / E::kES;
    constexpr int kUmmaK = 32 / E::kES;
    constexpr int kKSteps = kEPR / kUmmaK;
    constexpr uint32_t kABytes = 128 * 128;   // this CTA's 128 rows of A
    constexpr uint32_t kBBytes = 128 * 128;   // this CTA's 128 columns of B
    constexpr uint32_t kChunk = kEPR * 128;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + kStages * kABytes;
    // kEpilogueWarps x staging_tiles<EPI> tiles for TMA stores
    uint8_t* staging = smem_b + kStages * kBBytes;
    uint64_t* bars =
        reinterpret_cast<uint64_t*>(staging + kEpilogueWarps * staging_tiles<EPI>() * staging_bytes<T>());
    uint64_t* full = bars;
    uint64_t* empty = bars + kStages;
    uint64_t* acc_full = bars + 2 * kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* sched_full = drain + 1;
    uint64_t* sched_empty = sched_full + kSchedDepth;
    uint64_t* sched_req = sched_empty + kSchedDepth;
    volatile int* sched_tile = reinterpret_cast<volatile int*>(sched_req + 1);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sched_tile + kSchedDepth);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;
    // Run-time claims go through the tile ring; the fixed order needs none
    // (every role computes it), so short-K products pay no per-tile
    // synchronisation.
    const bool dynamic = p.sched != nullptr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&full[s]), 1);
            mbar_init(smem_addr(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_addr(&acc_full[a]), 1);
            mbar_init(smem_addr(&acc_empty[a]), 2 * kEpilogueWarps);
        }
        mbar_init(smem_addr(drain), 1);
        for (int d = 0; d < kSchedDepth; ++d) {
            mbar_init(smem_addr(&sched_full[d]), 1);
            mbar_init(smem_addr(&sched_empty[d]), kSchedConsumers);
        }
        mbar_init(smem_addr(sched_req), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(const_cast<uint32_t*>(tmem_slot)), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // set-up above overlaps the previous kernel; memory access starts here

    if (warp == 0) {
        // ---------------------------------------------------- producer --
        if (lane == 0) {
            const bool hint_ops = p.l2_operands != 0;
            const uint64_t pol_ops = p.l2_operands == 1 ? l2_policy_evict_last() : l2_policy_evict_normal();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int iter = 0; ok; ++iter) {
                int tile;
                if (!dynamic) {
                    tile = next_pair_tile(p, cluster_id, num_clusters, iter);
                } else {
                    const int slot = iter % kSchedDepth;
                    if (!mbar_wait_cluster(smem_addr(&sched_full[slot]), (iter / kSchedDepth) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tile = sched_tile[slot];
                    mbar_arrive_cluster(map_to_cta(smem_addr(&sched_empty[slot]), 0));
                }
                if (tile < 0) break;
                int b, mt, nt;
                tile_coords_pair(p, tile, b, mt, nt, group_m);
                const int m0 = mt * kPairBM + int(rank) * 128;
                const int n0 = nt * kPairBN + int(rank) * 128;
                const int kb_request = leader && p.sched != nullptr ? max(0, p.k_blocks - kClaimLead) : -1;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (kb == kb_request) mbar_arrive(smem_addr(sched_req));  // claim the next tile now
                    if (!mbar_wait(smem_addr(&empty[stage]), phase ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t own_full = smem_addr(&full[stage]);
                    if (leader) mbar_expect_tx(own_full, 2 * (kABytes + kBBytes));
                    const uint32_t fb = map_to_cta(own_full, 0);  // the leader's barrier
                    const uint32_t da = smem_addr(smem_a + stage * kABytes);
                    const uint32_t db = smem_addr(smem_b + stage * kBBytes);
                    const int k0 = kb * kEPR;
                    load_operand_pair<E::kES, A_MN, BATCHED>(da, &tmA, fb, m0, k0, b, 128, pol_ops, hint_ops);
                    load_operand_pair<E::kES, B_MN, BATCHED>(db, &tmB, fb, n0, k0, b, 128, pol_ops, hint_ops);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) atomicExch(p.err, kErrProducer);
        }
    } else if (warp == 1) {
        // ----------------------------------- MMA issuer (leader CTA only) --
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            constexpr uint32_t a_lbo = A_MN ? kChunk : 16;
            constexpr uint32_t b_lbo = B_MN ? kChunk : 16;
            constexpr uint32_t a_kstep = A_MN ? kUmmaK * 128 : 32;
            constexpr uint32_t b_kstep = B_MN ? kUmmaK * 128 : 32;
            for (int iter = 0; ok; ++iter, ++local) {
                int tile;
                if (!dynamic) {
                    tile = next_pair_tile(p, cluster_id, num_clusters, iter);
                } else {
                    const int slot = iter % kSchedDepth;
                    if (!mbar_wait(smem_addr(&sched_full[slot]), (iter / kSchedDepth) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tile = sched_tile[slot];
                    mbar_arrive(smem_addr(&sched_empty[slot]));
                }
                if (tile < 0) break;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(smem_addr(&acc_empty[acc]), acc_phase ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kPairBN;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(smem_addr(&full[stage]), phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(smem_a + stage * kABytes);
                    const uint32_t sb = smem_addr(smem_b + stage * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kKSteps; ++kk) {
                        const uint64_t ad = sw128_desc(sa + kk * a_kstep, a_lbo, 1024);
                        const uint64_t bd = sw128_desc(sb + kk * b_kstep, b_lbo, 1024);
                        umma_pair<E::kTF32>(d_tmem, ad, bd, p.idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit_pair(smem_addr(&empty[stage]));
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit_pair(smem_addr(&acc_full[acc]));
            }
            if (!ok) atomicExch(p.err, kErrMma);
            // Drain with a commit of the same CTA-group as the MMAs (it also
            // arrives, unobserved, on the peer's drain barrier).
            umma_commit_pair(smem_addr(drain));
            const uint64_t start = global_ns();
            while (!mbar_try_wait(smem_addr(drain), 0)) {
                if (global_ns() - start > kWaitNs) break;
            }
        }
    } else if (warp == kSchedWarp) {
        // ------------------------------------ tile scheduler (leader CTA) --
        if (leader && lane == 0 && dynamic) {
            for (int iter = 0;; ++iter) {
                const int slot = iter % kSchedDepth;
                if (!mbar_wait(smem_addr(&sched_empty[slot]), ((iter / kSchedDepth) & 1) ^ 1, abort_flag)) {
                    atomicExch(p.err, kErrProducer);
                    break;
                }
                // Run-time claims wait for the producer's request (made while
                // it loads the previous tile's last k-blocks).
                if (p.sched != nullptr && iter > 0 &&
                    !mbar_wait(smem_addr(sched_req), (iter - 1) & 1, abort_flag)) {
                    atomicExch(p.err, kErrProducer);
                    break;
                }
                const int tile = next_pair_tile(p, cluster_id, num_clusters, iter);
                sched_tile[slot] = tile;
                st_cluster_s32(map_to_cta(smem_addr(const_cast<int*>(&sched_tile[slot])), 1), tile);
                mbar_arrive(smem_addr(&sched_full[slot]));
                mbar_arrive_cluster(map_to_cta(smem_addr(&sched_full[slot]), 1));
                if (tile < 0) break;
            }
        }
    } else {
        // ------------------------------------------ epilogue (both CTAs) --
        const int quad = warp & 3;
        const int half = (warp - 2) / 4;
        const int row_in_tile = int(rank) * 128 + quad * 32 + lane;
        int local = 0;
        const uint32_t leader_empty0 = map_to_cta(smem_addr(&acc_empty[0]), 0);
        const uint32_t leader_empty1 = map_to_cta(smem_addr(&acc_empty[1]), 0);
        for (int iter = 0;; ++iter, ++local) {
            int tile;
            if (!dynamic) {
                tile = next_pair_tile(p, cluster_id, num_clusters, iter);
            } else {
                const int slot = iter % kSchedDepth;
                if (!mbar_wait_cluster(smem_addr(&sched_full[slot]), (iter / kSchedDepth) & 1, abort_flag)) {
                    if (lane == 0) atomicExch(p.err, kErrEpilogue);
                    break;
                }
                tile = sched_tile[slot];
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_addr(&sched_empty[slot]), 0));
            }
            if (tile < 0) break;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(smem_addr(&acc_full[acc]), acc_phase, abort_flag)) {
                if (lane == 0) atomicExch(p.err, kErrEpilogue);
                break;
            }
            tc_fence_after();
            int b, mt, nt;
            tile_coords_pair(p, tile, b, mt, nt, group_m);
            const int64_t gm = int64_t(mt) * kPairBM + row_in_tile;
            const uint32_t t_rows = tmem_base + (uint32_t(quad * 32) << 16) + acc * kPairBN;
            if (p.tma_store) {
                uint8_t* stage = staging + (warp - 2) * staging_tiles<EPI>() * staging_bytes<T>();
                store_accumulator_tma<T, kPairBN / 2, BATCHED, EPI>(p, &tmC, stage, t_rows, half * (kPairBN / 2), b,
                                                                    gm, gm - lane, int64_t(nt) * kPairBN, gm < p.M,
                                                                    &tmAux, stage + staging_bytes<T>());
            } else {
                store_accumulator<T, kPairBN / 2>(p, t_rows, half * (kPairBN / 2), b, gm, int64_t(nt) * kPairBN,
                                                  gm < p.M);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(acc == 0 ? leader_empty0 : leader_empty1);
        }
        if (lane == 0) bulk_wait_group0();
    }

    // Teardown: every thread of both CTAs reaches this point (no early
    // returns), so the cluster barrier completes; TMEM is then released
    // pairwise.
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------ host side --

// Counter words of the run-time tile scheduler: one per (device, stream)
// slot; a launch's epoch (per slot, counted on the host) tells its claims
// from those of the launches before it.
constexpr int kSchedSlots = 64;
__device__ unsigned long long g_gemm_sched[kSchedSlots];

struct SchedSlot {
    unsigned long long* word;
    uint32_t epoch;
};

// Whether the CTA-pair products on a device claim tiles at run time
// (tp_b200_set_gemm_tile_order; TPB200_GEMM_SCHED=dynamic turns it on for
// every device).  The fixed order is the default: it keeps each wave's
// tiles on neighbouring panels, and claiming costs a round trip per tile.
std::atomic<bool> g_gemm_dynamic[64] = {};

// The counter word and a fresh epoch for a launch on `stream`, or a null
// word (fixed tile order) unless run-time claims are on for the device;
// also while the stream is being captured into a graph (every replay would
// reuse the recorded epoch), for the per-thread default stream (one handle,
// many streams) and when the slots are used up.
SchedSlot gemm_sched_slot(int dev, cudaStream_t stream) {
    static const bool env_dynamic = [] {
        const char* e = std::getenv("TPB200_GEMM_SCHED");
        return e != nullptr && std::strcmp(e, "dynamic") == 0;
    }();
    const bool dynamic = dev >= 0 && dev < 64 && (env_dynamic || g_gemm_dynamic[dev].load(std::memory_order_relaxed));
    if (!dynamic || stream == cudaStreamPerThread) return {nullptr, 0};
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    TPB_CUDA(cudaStreamIsCapturing(stream, &cap));
    if (cap != cudaStreamCaptureStatusNone) return {nullptr, 0};
    static std::mutex lock;
    static unsigned long long* base[64] = {};
    static std::map<std::pair<int, cudaStream_t>, std::pair<int, uint32_t>> slots;
    static int used[64] = {};
    std::lock_guard<std::mutex> g(lock);
    if (base[dev] == nullptr) {
        void* ptr = nullptr;
        TPB_CUDA(cudaGetSymbolAddress(&ptr, g_gemm_sched));
        base[dev] = static_cast<unsigned long long*>(ptr);
    }
    auto it = slots.find({dev, stream});
    if (it == slots.end()) {
        if (used[dev] >= kSchedSlots) return {nullptr, 0};
        it = slots.emplace(std::make_pair(dev, stream), std::make_pair(used[dev]++, 0u)).first;
    }
    uint32_t& epoch = it->second.second;
    if (++epoch == 0) epoch = 1;  // 0 is the words' initial value
    return {base[dev] + it->second.first, epoch};
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        TPB_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                                  cudaEnableDefault, &q));
        TPB_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr,
                  "cuTensorMapEncodeTiled is unavailable from the driver");
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// Tensor map over an operand seen as [batch][outer][inner] with unit stride
// on `inner`; box = kEPR x box_outer elements, 128-byte swizzle.
CUtensorMap make_map(const void* base, CUtensorMapDataType type, int es, int64_t inner, int64_t outer,
                     int64_t outer_stride, int64_t batch, int64_t batch_stride, uint32_t box_outer) {
    CUtensorMap map;
    const int rank = batch > 1 ? 3 : 2;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(outer_stride * es),
                             static_cast<cuuint64_t>(batch_stride * es)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&map, type, rank, const_cast<void*>(base), dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TPB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return map;
}

// The result's tensor map for the TMA-store epilogue: boxes of 32 x 32
// elements, 64-byte-swizzled rows for 16-bit types, 128-byte for fp32.
CUtensorMap make_c_map(void* base, CUtensorMapDataType type, int es, int64_t N, int64_t M, int64_t row_stride,
                       int64_t batch, int64_t batch_stride) {
    CUtensorMap map;
    const int rank = batch > 1 ? 3 : 2;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * es), static_cast<cuuint64_t>(batch_stride * es)};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = encode_fn()(&map, type, rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   es == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TPB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (result) failed (%d)", static_cast<int>(r));
    return map;
}

bool tma_ok(const void* p, int es, int64_t other_stride, int64_t batch, int64_t batch_stride) {
    if (!aligned16(p)) return false;
    if (other_stride <= 0 || (other_stride * es) % 16 != 0) return false;
    if (batch > 1 && (batch_stride <= 0 || (batch_stride * es) % 16 != 0)) return false;
    return true;
}

// Per-shape tile choice, computed once and cached (BlasKernels.cpp:70-104
// caches a CNNL plan per problem the same way).
int choose_bn(int64_t M, int64_t N, int64_t batch, int sms) {
    using Key = std::tuple<int64_t, int64_t, int64_t, int>;
    static std::mutex lock;
    static std::map<Key, int> cache;
    const Key key{M, N, batch, sms};
    {
        std::lock_guard<std::mutex> g(lock);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    // Cost in units of one 128 x 128 tile; a 128 x 256 tile costs a little
    // under two (better operand reuse per MMA).
    auto cost = [&](int bn) {
        const int64_t tiles = batch * ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
        const int64_t waves = (tiles + sms - 1) / sms;
        return static_cast<double>(waves) * (bn == 256 ? 1.9 : 1.0);
    };
    const int bn = N <= 128 ? 128 : (cost(256) <= cost(128) ? 256 : 128);
    std::lock_guard<std::mutex> g(lock);
    cache[key] = bn;
    return bn;
}

template <typename T, int BN, bool A_MN, bool B_MN, bool BATCHED>
void launch_tc(const GemmProblem& p, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
               TcParams& tp, int dev, cudaStream_t stream) {
    constexpr size_t smem = tc_smem_bytes<T, BN>();
    auto kern = gemm_tc_kernel<T, BN, A_MN, B_MN, BATCHED>;
    static bool configured[64] = {};
    if (!configured[dev]) {
        TPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        configured[dev] = true;
    }
    tp.m_tiles = static_cast<int>((p.M + kBM - 1) / kBM);
    tp.n_tiles = static_cast<int>((p.N + BN - 1) / BN);
    tp.num_tiles = static_cast<int>(p.batch) * tp.m_tiles * tp.n_tiles;
    // Instruction descriptor: fp32 accumulate (bit 4), A/B format (bits 7-9,
    // 10-12: f16 0, bf16 1, tf32 2), A/B MN-major (bits 15, 16), N >> 3
    // (bits 17-22), M >> 4 (bits 24-28).
    const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : std::is_same<T, float>::value ? 2u : 0u;
    tp.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(tp.a_mn) << 15) |
               (uint32_t(tp.b_mn) << 16) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
    const int grid = std::min(tp.num_tiles, gemm_sm_budget(dev));
    launch_pdl(kern, grid, kTcThreads, smem, stream, ma, mb, mc, tp);
    check_launch("gemm_tc");
}

template <typename T, bool A_MN, bool B_MN, bool BATCHED, int EPI = kEpiPlain>
void launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, TcParams& tp, int dev,
                cudaStream_t stream, const CUtensorMap* maux = nullptr) {
    constexpr size_t smem = tc2_smem_bytes<T, EPI>();
    static_assert(smem <= 232448, "shared memory per CTA");
    auto kern = gemm_tc2_kernel<T, A_MN, B_MN, BATCHED, EPI>;
    static bool configured[64] = {};
    if (!configured[dev]) {
        TPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        configured[dev] = true;
    }
    tp.m_tiles = (tp.M + kPairBM - 1) / kPairBM;
    tp.n_tiles = (tp.N + kPairBN - 1) / kPairBN;
    tp.num_tiles = tp.batch * tp.m_tiles * tp.n_tiles;
    const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : std::is_same<T, float>::value ? 2u : 0u;
    tp.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(tp.a_mn) << 15) |
               (uint32_t(tp.b_mn) << 16) | (uint32_t(kPairBN >> 3) << 17) | (uint32_t(kPairBM >> 4) << 24);
    // Row-tile groups sized so the group's A panels (~32 MiB, a quarter of L2:
    // the two dies each cache their own half) stay resident while B streams
    // past them.
    // TPB200_GEMM_GROUP_MB overrides the 32 MiB panel budget (A/B measurements).
    static const int64_t budget_mb = [] {
        const char* e = std::getenv("TPB200_GEMM_GROUP_MB");
        const long v = e != nullptr ? std::strtol(e, nullptr, 10) : 0;
        return v > 0 ? int64_t(v) : int64_t(32);
    }();
    const int64_t panel = int64_t(kPairBM) * tp.K * int64_t(sizeof(T));
    int group_m = static_cast<int>(std::max<int64_t>(1, (budget_mb << 20) / std::max<int64_t>(panel, 1)));
    group_m = std::min(group_m, tp.m_tiles);
    const int clusters = std::min(tp.num_tiles, gemm_sm_budget(dev) / 2);
    const SchedSlot slot = gemm_sched_slot(dev, stream);
    tp.sched = slot.word;
    tp.epoch = slot.epoch;
    // TPB200_GEMM_L2HINT=none|stream|both (A/B measurements): which accesses
    // carry an eviction-priority policy.  None by default: in the MLP step,
    // evict_first on the epilogue's streams measured 4.36 ms per step and
    // evict_last on the operands as well 4.27 ms, against 4.24 ms without.
    static const int l2hint = [] {
        const char* e = std::getenv("TPB200_GEMM_L2HINT");
        if (e == nullptr || std::strcmp(e, "none") == 0) return 0;
        if (std::strcmp(e, "both") == 0) return 2;
        if (std::strcmp(e, "normal") == 0) return 3;
        return 1;
    }();
    tp.l2_stream = l2hint == 3 ? 2 : l2hint >= 1 ? 1 : 0;
    tp.l2_operands = l2hint == 3 ? 2 : l2hint == 2 ? 1 : 0;
    launch_pdl(kern, 2 * clusters, kTc2Threads, smem, stream, ma, mb, mc, maux != nullptr ? *maux : mc, tp, group_m);
    check_launch("gemm_tc2");
}

// The kernel instance for the operands' layouts and batching.  fp32 (TF32)
// operands always arrive K-major, so only that instance is built for them.
template <typename T, bool A_MN, bool B_MN, bool BATCHED>
void launch_layout(bool pair, int bn, const GemmProblem& p, const CUtensorMap& ma, const CUtensorMap& mb,
                   const CUtensorMap& mc, TcParams& tp, int dev, cudaStream_t stream) {
    if (pair) launch_tc2<T, A_MN, B_MN, BATCHED>(ma, mb, mc, tp, dev, stream);
    else if (bn == 256) launch_tc<T, 256, A_MN, B_MN, BATCHED>(p, ma, mb, mc, tp, dev, stream);
    else launch_tc<T, 128, A_MN, B_MN, BATCHED>(p, ma, mb, mc, tp, dev, stream);
}

template <typename T>
void launch_any(bool pair, int bn, const GemmProblem& p, const CUtensorMap& ma, const CUtensorMap& mb,
                const CUtensorMap& mc, TcParams& tp, int dev, cudaStream_t stream) {
    const bool bt = tp.batched != 0;
    if constexpr (std::is_same<T, float>::value) {
        TPB_CHECK(!tp.a_mn && !tp.b_mn, "gemm: TF32 operands must be K-major");
        if (bt) launch_layout<T, false, false, true>(pair, bn, p, ma, mb, mc, tp, dev, stream);
        else launch_layout<T, false, false, false>(pair, bn, p, ma, mb, mc, tp, dev, stream);
    } else {
        const int code = (tp.a_mn ? 4 : 0) | (tp.b_mn ? 2 : 0) | (bt ? 1 : 0);
        switch (code) {
            case 0: launch_layout<T, false, false, false>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 1: launch_layout<T, false, false, true>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 2: launch_layout<T, false, true, false>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 3: launch_layout<T, false, true, true>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 4: launch_layout<T, true, false, false>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 5: launch_layout<T, true, false, true>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            case 6: launch_layout<T, true, true, false>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
            default: launch_layout<T, true, true, true>(pair, bn, p, ma, mb, mc, tp, dev, stream); break;
        }
    }
}

// Which kernel: the CTA-pair kernel for problems with at least one full
// 256 x 256 tile, the single-SM kernel otherwise; TPB200_GEMM_KERNEL=1sm|2sm
// overrides the choice (for A/B measurements).
bool use_pair_kernel(const GemmProblem& p) {
    static const char* force = std::getenv("TPB200_GEMM_KERNEL");
    if (force != nullptr && std::strcmp(force, "1sm") == 0) return false;
    if (force != nullptr && std::strcmp(force, "2sm") == 0) return true;
    return p.M >= kPairBM && p.N >= kPairBN;
}

// The fused-epilogue instances: bf16, unbatched, CTA-pair kernel.
template <typename T, int EPI>
void launch_epi(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& maux,
                TcParams& tp, int dev, cudaStream_t stream) {
    const int code = (tp.a_mn ? 2 : 0) | (tp.b_mn ? 1 : 0);
    switch (code) {
        case 0: launch_tc2<T, false, false, false, EPI>(ma, mb, mc, tp, dev, stream, &maux); break;
        case 1: launch_tc2<T, false, true, false, EPI>(ma, mb, mc, tp, dev, stream, &maux); break;
        case 2: launch_tc2<T, true, false, false, EPI>(ma, mb, mc, tp, dev, stream, &maux); break;
        default: launch_tc2<T, true, true, false, EPI>(ma, mb, mc, tp, dev, stream, &maux); break;
    }
}

template <typename T>
bool gemm_tc_typed(const GemmProblem& p_in, int dev, cudaStream_t stream, CUtensorMapDataType type) {
    constexpr int es = sizeof(T);
    GemmProblem p = p_in;
    if (p.epi != kEpiPlain) {
        // Fused epilogues: bf16 products with a full CTA-pair tile, no batch,
        // the result (and gelu's pre-activation) written by TMA stores.
        if constexpr (!std::is_same<T, __nv_bfloat16>::value) {
            return false;
        } else {
            if (p.batch != 1 || !use_pair_kernel(p) || p.aux == nullptr) return false;
            if (p.epi == kEpiGeluBackward && p.cin != nullptr) return false;
            if (p.epi == kEpiGelu && !(aligned16(p.aux) && p.saux_m > 0 && (p.saux_m * es) % 16 == 0)) return false;
            if (std::getenv("TPB200_NO_TMA_STORE") != nullptr) return false;
            if (!(aligned16(p.c) && p.sc_m > 0 && (p.sc_m * es) % 16 == 0)) return false;
        }
    }
    // TF32 operands must be K-major here: the 128-byte-swizzled MN-major
    // layout this kernel stages is defined for 16-bit elements only (32-bit
    // MN-major operands need the 32-byte-atom swizzle variant).  An MN-major
    // fp32 operand is first copied K-major (one transposing pass).
    std::unique_ptr<Scratch> a_copy, b_copy;
    if constexpr (std::is_same<T, float>::value) {
        if (!(p.sa_k == 1 || p.K == 1)) {
            a_copy.reset(new Scratch(sizeof(float) * p.batch * p.M * p.K, dev, stream));
            Scratch& tmp = *a_copy;
            tpb_tensor src{}, dst{};
            src.data = const_cast<void*>(p.a);
            src.dtype = dst.dtype = TPB_F32;
            src.ndim = dst.ndim = 3;
            const int64_t sizes[3] = {p.batch, p.M, p.K};
            const int64_t sstr[3] = {p.sa_b, p.sa_m, p.sa_k};
            const int64_t dstr[3] = {p.M * p.K, p.K, 1};
            for (int i = 0; i < 3; ++i) {
                src.sizes[i] = dst.sizes[i] = sizes[i];
                src.strides[i] = sstr[i];
                dst.strides[i] = dstr[i];
            }
            dst.data = tmp.get();
            copy_impl(dst, src, stream, dev);
            p.a = tmp.get();
            p.sa_b = p.batch > 1 ? p.M * p.K : 0;
            p.sa_m = p.K;
            p.sa_k = 1;
        }
        if (!(p.sb_k == 1 || p.K == 1)) {
            b_copy.reset(new Scratch(sizeof(float) * p.batch * p.N * p.K, dev, stream));
            Scratch& tmp = *b_copy;
            tpb_tensor src{}, dst{};
            src.data = const_cast<void*>(p.b);
            src.dtype = dst.dtype = TPB_F32;
            src.ndim = dst.ndim = 3;
            const int64_t sizes[3] = {p.batch, p.N, p.K};
            const int64_t sstr[3] = {p.sb_b, p.sb_n, p.sb_k};
            const int64_t dstr[3] = {p.N * p.K, p.K, 1};
            for (int i = 0; i < 3; ++i) {
                src.sizes[i] = dst.sizes[i] = sizes[i];
                src.strides[i] = sstr[i];
                dst.strides[i] = dstr[i];
            }
            dst.data = tmp.get();
            copy_impl(dst, src, stream, dev);
            p.b = tmp.get();
            p.sb_b = p.batch > 1 ? p.N * p.K : 0;
            p.sb_n = p.K;
            p.sb_k = 1;
        }
    }
    // A: K-major (unit stride along K) or M-major; same for B along K / N.
    const bool a_k = p.sa_k == 1 || p.K == 1;
    const bool a_m = !a_k && (p.sa_m == 1 || p.M == 1);
    const bool b_k = p.sb_k == 1 || p.K == 1;
    const bool b_n = !b_k && (p.sb_n == 1 || p.N == 1);
    if (!(a_k || a_m) || !(b_k || b_n)) return false;
    if (!tma_ok(p.a, es, a_k ? p.sa_m : p.sa_k, p.batch, p.sa_b)) return false;
    if (!tma_ok(p.b, es, b_k ? p.sb_n : p.sb_k, p.batch, p.sb_b)) return false;
    if (p.M >= (int64_t(1) << 31) || p.N >= (int64_t(1) << 31) || p.K >= (int64_t(1) << 31)) return false;
    const int sms = gemm_sm_budget(dev);
    const bool pair = use_pair_kernel(p);
    const int bn = pair ? 128 : choose_bn(p.M, p.N, p.batch, sms);  // B rows staged per CTA
    constexpr int kEPR = 128 / es;
    // Boxes: K-major operands kEPR (K) x kBoxRows rows (a stage takes 128 /
    // kBoxRows, or bn / kBoxRows, of them); MN-major operands kEPR (MN) x kEPR
    // (K) chunks.
    const CUtensorMap ma = a_k ? make_map(p.a, type, es, p.K, p.M, p.sa_m, p.batch, p.sa_b, kBoxRows)
                               : make_map(p.a, type, es, p.M, p.K, p.sa_k, p.batch, p.sa_b, kEPR);
    const CUtensorMap mb = b_k ? make_map(p.b, type, es, p.K, p.N, p.sb_n, p.batch, p.sb_b, kBoxRows)
                               : make_map(p.b, type, es, p.N, p.K, p.sb_k, p.batch, p.sb_b, kEPR);
    TcParams tp{};
    tp.M = static_cast<int>(p.M);
    tp.N = static_cast<int>(p.N);
    tp.K = static_cast<int>(p.K);
    tp.batch = static_cast<int>(p.batch);
    tp.k_blocks = static_cast<int>((p.K + kEPR - 1) / kEPR);
    tp.a_mn = a_k ? 0 : 1;
    tp.b_mn = b_k ? 0 : 1;
    tp.batched = p.batch > 1 ? 1 : 0;
    tp.c = p.c;
    tp.sc_b = p.sc_b;
    tp.sc_m = p.sc_m;
    tp.cin = p.cin;
    tp.sci_b = p.sci_b;
    tp.sci_m = p.sci_m;
    tp.sci_n = p.sci_n;
    tp.alpha = static_cast<float>(p.alpha);
    tp.beta = static_cast<float>(p.beta);
    tp.vec_store = aligned16(p.c) && (p.sc_m * es) % 16 == 0 && (p.batch == 1 || (p.sc_b * es) % 16 == 0);
    tp.aux = p.aux;
    tp.saux_m = p.saux_m;
    tp.err = device_error_word(dev);
    // The result through a C tensor map (TMA stores) when its layout allows.
    // TPB200_NO_TMA_STORE=1 keeps the direct-store epilogue (A/B measurements).
    static const bool no_tma_store = std::getenv("TPB200_NO_TMA_STORE") != nullptr;
    const bool c_tma = !no_tma_store && aligned16(p.c) && p.sc_m > 0 && (p.sc_m * es) % 16 == 0 &&
                       (p.batch == 1 || (p.sc_b > 0 && (p.sc_b * es) % 16 == 0));
    tp.tma_store = c_tma ? 1 : 0;
    const CUtensorMap mc = c_tma ? make_c_map(p.c, type, es, p.N, p.M, p.sc_m, p.batch, p.sc_b) : ma;
    if (p.epi != kEpiPlain) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            TPB_CHECK(pair && c_tma, "gemm: fused epilogue without the CTA-pair TMA-store kernel");
            if (p.epi == kEpiGelu) {
                const CUtensorMap maux = make_c_map(p.aux, type, es, p.N, p.M, p.saux_m, 1, 0);
                launch_epi<T, kEpiGelu>(ma, mb, mc, maux, tp, dev, stream);
            } else {
                launch_epi<T, kEpiGeluBackward>(ma, mb, mc, mc, tp, dev, stream);
            }
        }
        return true;
    }
    launch_any<T>(pair, bn, p, ma, mb, mc, tp, dev, stream);
    return true;
}

// ---------------------------------------------- fp32 through 3 x TF32 --
//
// Without TF32 permission an fp32 product keeps fp32 accuracy by the
// split-precision ("3xTF32") method: every operand element x is split into
// hi = tf32(x) and lo = tf32(x - hi), both exact TF32 values (low 13
// mantissa bits zero, so the tensor core's reading of an fp32 word as TF32
// changes nothing), and A.B ~= Alo.Bhi + Ahi.Blo + Ahi.Bhi.  The dropped
// Alo.Blo term and the rounding of lo are both ~2^-22 relative to |a b|.
// The three products run as TF32 tensor-core GEMMs over K-concatenated
// operands, K in chunks of kSplitChunk:
//   A' chunk j = [Alo_j | Ahi_j | Ahi_j],   B' chunk j = [Bhi_j ; Blo_j ; Bhi_j]
// (both K-major; the small correction terms come first, while the
// accumulator is still small).  The tensor core adds into its accumulator
// with truncation after alignment, an error that grows with the number of
// additions; so each chunk is one GEMM launch whose epilogue adds its
// result into the output in fp32 with round-to-nearest (beta = 1 after the
// first chunk), keeping every accumulator chain short.
// A non-finite element (inf, NaN) has lo = 0, and inf * 0 in a cross term
// would turn an fp32 inf into NaN; the split marks such rows of A / columns
// of B and a fix-up pass recomputes the outputs in them with plain fp32 dot
// products.
constexpr int64_t kSplitChunk = 1024;

// Round to the nearest TF32 value (ties away from zero); a rounding that
// would overflow truncates instead; inf and NaN are returned unchanged.
__device__ __forceinline__ float tf32_round(float x) {
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    uint32_t r = (u + 0x1000u) & 0xffffe000u;
    if ((r & 0x7f800000u) == 0x7f800000u) r = u & 0xffffe000u;
    return __uint_as_float(r);
}

// Rows of a K-major operand (row `row` of batch `row / R` at
// src + (row / R) * s_b + (row % R) * s_r) into rows of `ld` floats, chunk j
// of K at j * 3 * kSplitChunk holding its three parts back to back (each
// K_j = min(kSplitChunk, K - j * kSplitChunk) wide): [lo | hi | hi] for A
// (b_side 0), [hi | lo | hi] for B (b_side 1).  flags[row] is set when the
// row holds a non-finite element.
__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                         int64_t rows, int64_t R, int64_t K, int64_t s_b,
                                                         int64_t s_r, int64_t ld, int b_side,
                                                         unsigned* __restrict__ flags) {
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        const float* s = src + (row / R) * s_b + (row % R) * s_r;
        float* d = dst + row * ld;
        int bad = 0;
        for (int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; k < K;
             k += int64_t(gridDim.x) * blockDim.x) {
            const float x = s[k];
            const float hi = tf32_round(x);
            const bool finite = isfinite(x);
            const float lo = finite ? tf32_round(x - hi) : 0.0f;
            bad |= !finite;
            const int64_t j = k / kSplitChunk, kk = k % kSplitChunk;
            const int64_t kj = K - j * kSplitChunk < kSplitChunk ? K - j * kSplitChunk : kSplitChunk;
            float* c = d + j * 3 * kSplitChunk + kk;
            c[0] = b_side ? hi : lo;
            c[kj] = b_side ? lo : hi;
            c[2 * kj] = hi;
        }
        if (__syncthreads_or(bad) && threadIdx.x == 0) flags[row] = 1u;
    }
}

struct FixupParams {
    const float* a;
    int64_t sa_b, sa_m, sa_k;
    const float* b;
    int64_t sb_b, sb_k, sb_n;
    float* c;
    int64_t sc_b, sc_m;
    const float* cin;
    int64_t sci_b, sci_m, sci_n;
    float alpha, beta;
    int64_t M, N, K, batch;
    int64_t a_rows_per_batch, b_rows_per_batch;  // 0 when that operand is broadcast over the batch
};

__device__ __forceinline__ void fixup_one(const FixupParams& p, int64_t bt, int64_t i, int64_t j) {
    const float* a = p.a + bt * p.sa_b + i * p.sa_m;
    const float* b = p.b + bt * p.sb_b + j * p.sb_n;
    float acc = 0.0f;
    for (int64_t k = 0; k < p.K; ++k) acc = fmaf(a[k * p.sa_k], b[k * p.sb_k], acc);
    float v = p.alpha * acc;
    if (p.cin != nullptr) v += p.beta * p.cin[bt * p.sci_b + i * p.sci_m + j * p.sci_n];
    p.c[bt * p.sc_b + i * p.sc_m + j] = v;
}

// Block per (batch, row of A) / (batch, column of B): recompute the flagged
// ones.  Unflagged blocks leave at once.
__global__ void __launch_bounds__(256) fixup_rows_kernel(FixupParams p, const unsigned* __restrict__ a_flags) {
    const int64_t bt = blockIdx.y, i = blockIdx.x;
    if (!a_flags[(p.a_rows_per_batch ? bt : 0) * p.M + i]) return;
    for (int64_t j = threadIdx.x; j < p.N; j += blockDim.x) fixup_one(p, bt, i, j);
}

__global__ void __launch_bounds__(256) fixup_cols_kernel(FixupParams p, const unsigned* __restrict__ b_flags) {
    const int64_t bt = blockIdx.y, j = blockIdx.x;
    if (!b_flags[(p.b_rows_per_batch ? bt : 0) * p.N + j]) return;
    for (int64_t i = threadIdx.x; i < p.M; i += blockDim.x) fixup_one(p, bt, i, j);
}

// A K-major view of an operand: `rows` rows of K floats at base + b*s_b + r*s_r.
struct KMajor {
    const float* base;
    int64_t s_b, s_r;
};

// Split one operand ([batches, R, K] with strides sb_, sr, sk) into a
// [batches * R, ld] scratch of split rows; MN-major operands are first
// copied K-major.
void split_operand(const float* src, int64_t batches, int64_t R, int64_t K, int64_t s_b, int64_t s_r,
                   int64_t s_k, int b_side, float* dst, int64_t ld, unsigned* flags,
                   std::unique_ptr<Scratch>& kmajor, int dev, cudaStream_t stream) {
    KMajor v{src, s_b, s_r};
    if (!(s_k == 1 || K == 1)) {
        kmajor.reset(new Scratch(sizeof(float) * batches * R * K, dev, stream));
        tpb_tensor s{}, d{};
        s.data = const_cast<float*>(src);
        s.dtype = d.dtype = TPB_F32;
        s.ndim = d.ndim = 3;
        const int64_t sizes[3] = {batches, R, K};
        const int64_t sstr[3] = {s_b, s_r, s_k};
        const int64_t dstr[3] = {R * K, K, 1};
        for (int i = 0; i < 3; ++i) {
            s.sizes[i] = d.sizes[i] = sizes[i];
            s.strides[i] = sstr[i];
            d.strides[i] = dstr[i];
        }
        d.data = kmajor->get();
        copy_impl(d, s, stream, dev);
        v = KMajor{static_cast<const float*>(kmajor->get()), R * K, K};
    }
    const int64_t rows = batches * R;
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((K + 255) / 256, 64)),
              static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
    split_tf32_kernel<<<grid, 256, 0, stream>>>(v.base, dst, rows, R, K, v.s_b, v.s_r, ld, b_side, flags);
    check_launch("split_tf32");
}

// Problems this large take the split path; smaller ones stay on the CUDA
// cores, where the three-fold operand traffic and launches would not pay.
bool use_split_tf32(const GemmProblem& p) {
    static const char* force = std::getenv("TPB200_GEMM_F32");
    if (force != nullptr && std::strcmp(force, "simt") == 0) return false;
    if (3 * p.K >= (int64_t(1) << 31) || p.M >= (int64_t(1) << 31) || p.N >= (int64_t(1) << 31)) return false;
    if (p.batch > 65535) return false;  // the fix-up grids' y extent
    // An operand broadcast over the batch (batch stride 0) has no batched
    // tensor map; such products take the CUDA-core kernel, as TF32 ones do.
    if (p.batch > 1 && (p.sa_b == 0 || p.sb_b == 0)) return false;
    return p.M >= 128 && p.N >= 128 && p.K >= 16 && p.M * p.N * p.K * p.batch >= (int64_t(1) << 27);
}

bool gemm_f32_split(const GemmProblem& p, int dev, cudaStream_t stream) {
    if (!use_split_tf32(p)) return false;
    const int64_t chunks = (p.K + kSplitChunk - 1) / kSplitChunk;
    const int64_t ld = chunks * 3 * kSplitChunk;  // a multiple of 4: 16-byte row pitch
    const int64_t a_batches = p.sa_b == 0 ? 1 : p.batch;
    const int64_t b_batches = p.sb_b == 0 ? 1 : p.batch;
    Scratch a3(sizeof(float) * a_batches * p.M * ld, dev, stream);
    Scratch b3(sizeof(float) * b_batches * p.N * ld, dev, stream);
    const int64_t nflags = a_batches * p.M + b_batches * p.N;
    Scratch flags(sizeof(unsigned) * nflags, dev, stream);
    TPB_CUDA(cudaMemsetAsync(flags.get(), 0, sizeof(unsigned) * nflags, stream));
    unsigned* a_flags = static_cast<unsigned*>(flags.get());
    unsigned* b_flags = a_flags + a_batches * p.M;
    std::unique_ptr<Scratch> a_k, b_k;
    split_operand(static_cast<const float*>(p.a), a_batches, p.M, p.K, p.sa_b, p.sa_m, p.sa_k, 0,
                  static_cast<float*>(a3.get()), ld, a_flags, a_k, dev, stream);
    split_operand(static_cast<const float*>(p.b), b_batches, p.N, p.K, p.sb_b, p.sb_n, p.sb_k, 1,
                  static_cast<float*>(b3.get()), ld, b_flags, b_k, dev, stream);
    a_k.reset();
    b_k.reset();
    for (int64_t j = 0; j < chunks; ++j) {
        const int64_t kj = std::min(kSplitChunk, p.K - j * kSplitChunk);
        GemmProblem q = p;
        q.K = 3 * kj;
        q.a = static_cast<const float*>(a3.get()) + j * 3 * kSplitChunk;
        q.sa_k = 1;
        q.sa_m = ld;
        q.sa_b = a_batches > 1 ? p.M * ld : 0;
        q.b = static_cast<const float*>(b3.get()) + j * 3 * kSplitChunk;
        q.sb_k = 1;
        q.sb_n = ld;
        q.sb_b = b_batches > 1 ? p.N * ld : 0;
        q.flags = p.flags | TPB_GEMM_ALLOW_TF32;
        if (j > 0) {  // out = alpha * A_j.B_j + out
            q.cin = p.c;
            q.sci_b = p.sc_b;
            q.sci_m = p.sc_m;
            q.sci_n = 1;
            q.beta = 1.0;
        }
        TPB_CHECK(gemm_tc_typed<float>(q, dev, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT32),
                  "gemm: the split-TF32 operands were not accepted by the tensor-core kernel");
    }
    FixupParams f{};
    f.a = static_cast<const float*>(p.a);
    f.sa_b = p.sa_b;
    f.sa_m = p.sa_m;
    f.sa_k = p.sa_k;
    f.b = static_cast<const float*>(p.b);
    f.sb_b = p.sb_b;
    f.sb_k = p.sb_k;
    f.sb_n = p.sb_n;
    f.c = static_cast<float*>(p.c);
    f.sc_b = p.sc_b;
    f.sc_m = p.sc_m;
    f.cin = static_cast<const float*>(p.cin);
    f.sci_b = p.sci_b;
    f.sci_m = p.sci_m;
    f.sci_n = p.sci_n;
    f.alpha = static_cast<float>(p.alpha);
    f.beta = static_cast<float>(p.beta);
    f.M = p.M;
    f.N = p.N;
    f.K = p.K;
    f.batch = p.batch;
    f.a_rows_per_batch = a_batches > 1 ? p.M : 0;
    f.b_rows_per_batch = b_batches > 1 ? p.N : 0;
    fixup_rows_kernel<<<dim3(static_cast<unsigned>(p.M), static_cast<unsigned>(p.batch)), 256, 0, stream>>>(
        f, a_flags);
    check_launch("gemm_f32_fixup_rows");
    fixup_cols_kernel<<<dim3(static_cast<unsigned>(p.N), static_cast<unsigned>(p.batch)), 256, 0, stream>>>(
        f, b_flags);
    check_launch("gemm_f32_fixup_cols");
    return true;
}

}  // namespace

bool gemm_tc(const GemmProblem& p, int dev, cudaStream_t stream) {
    if (p.M == 0 || p.N == 0 || p.K == 0) return false;
    if (p.epi != kEpiPlain && p.dtype != TPB_BF16) return false;
    switch (p.dtype) {
        case TPB_BF16: return gemm_tc_typed<__nv_bfloat16>(p, dev, stream, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
        case TPB_F16: return gemm_tc_typed<__half>(p, dev, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
        case TPB_F32:
            if (!(p.flags & TPB_GEMM_ALLOW_TF32)) return gemm_f32_split(p, dev, stream);
            return gemm_tc_typed<float>(p, dev, stream, CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
        default: return false;
    }
}

}  // namespace tpb

extern "C" int tp_b200_set_gemm_tile_order(int dev, int dynamic) {
    return tpb::guarded([&] {
        TPB_CHECK(dev >= 0 && dev < 64, "invalid device index %d", dev);
        tpb::g_gemm_dynamic[dev].store(dynamic != 0, std::memory_order_relaxed);
    });
}
