/*
 * mlp.c -- CPU port of one training step of the BASELINE MLP (Linear 4096 ->
 * 16384, GELU, Linear 16384 -> 4096, MSE, SGD).  TEST AND BASELINE
 * INFRASTRUCTURE ONLY: bench.py times it as the CPU path of the workload
 * (cpu_baseline / --impl reference) on the host cores, and tests/ use it to
 * check the device step; the product never calls it.
 *
 * It performs the same operator sequence TensorPlay's autograd engine would
 * run on its CPU kernels for this model (linear, gelu, sub, pow, mean,
 * mm on transposed views, sum over dim 0, gelu_backward, add_), in the
 * precision those kernels use for bf16 tensors: values stored as bf16
 * between operators, fp32 arithmetic inside each (the accumulation type of
 * the reference's kernels, BinaryKernels.cpp:76, ReduceKernels.cpp:34,
 * BlasKernels.cpp:113).
 *
 * The five products run through a cache-blocked matrix product in the
 * standard packed-panel organisation (the GotoBLAS / BLIS scheme): a KC x NC
 * panel of B is packed once into NR-wide strips shared by all threads, each
 * thread packs MC x KC blocks of A into MR-high strips, and a register-
 * blocked MR x NR micro-kernel (8 x 32 with AVX-512, 6 x 16 with AVX2, chosen
 * at run time) accumulates in fp32.  Packing converts bf16 operands to fp32
 * on the way, so no full-size fp32 copy of a weight is made.  Threads:
 * OpenMP, with the count set explicitly (orc_set_num_threads) because
 * torchrun exports OMP_NUM_THREADS=1.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float bf(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static uint16_t tobf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static float rbf(float f) { return bf(tobf(f)); }

static float gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678f)); }
static float gelu_grad(float x) {
    const float cdf = 0.5f * (1.0f + erff(x * 0.70710678f));
    const float pdf = expf(-0.5f * x * x) * 0.39894228f;
    return cdf + x * pdf;
}

/* ------------------------------------------------------ blocked product -- */

/* A matrix operand: element (r, c) at p[r * rs + c * cs], bf16 or fp32. */
typedef struct {
    const void* p;
    int bf16;
    int64_t rs, cs;
} Mat;

static inline float mat_at(const Mat* m, int64_t r, int64_t c) {
    const int64_t o = r * m->rs + c * m->cs;
    return m->bf16 ? bf(((const uint16_t*)m->p)[o]) : ((const float*)m->p)[o];
}

enum { KC = 256, MC = 128, NC = 4096 };

/* micro-kernel: C[mr x nr] (+)= A strip (kc x MR, k-major) . B strip (kc x NR) */
typedef void (*kern_fn)(int64_t kc, const float* A, const float* B, float* C, int64_t ldc, int acc);

typedef float v16 __attribute__((vector_size(64)));
typedef float v16u __attribute__((vector_size(64), aligned(4)));
typedef float v8 __attribute__((vector_size(32)));
typedef float v8u __attribute__((vector_size(32), aligned(4)));

#define BCAST16(x) ((v16){x, x, x, x, x, x, x, x, x, x, x, x, x, x, x, x})
#define BCAST8(x) ((v8){x, x, x, x, x, x, x, x})

#define K512_ROW(i) v16 c##i##0 = z, c##i##1 = z;
#define K512_FMA(i)                        \
    {                                      \
        const float s_ = A[k * 8 + (i)];   \
        const v16 a = BCAST16(s_);         \
        c##i##0 += a * b0;                 \
        c##i##1 += a * b1;                 \
    }
#define K512_STORE(i)                                                  \
    {                                                                  \
        v16u* r = (v16u*)(C + (i) * ldc);                              \
        if (acc) { r[0] += c##i##0; r[1] += c##i##1; }                 \
        else { r[0] = c##i##0; r[1] = c##i##1; }                       \
    }

__attribute__((target("avx512f,fma"))) static void kern_8x32(int64_t kc, const float* A, const float* B, float* C,
                                                              int64_t ldc, int acc) {
    const v16 z = {0};
    K512_ROW(0) K512_ROW(1) K512_ROW(2) K512_ROW(3) K512_ROW(4) K512_ROW(5) K512_ROW(6) K512_ROW(7)
    for (int64_t k = 0; k < kc; ++k) {
        const v16 b0 = *(const v16*)(B + k * 32);
        const v16 b1 = *(const v16*)(B + k * 32 + 16);
        K512_FMA(0) K512_FMA(1) K512_FMA(2) K512_FMA(3) K512_FMA(4) K512_FMA(5) K512_FMA(6) K512_FMA(7)
    }
    K512_STORE(0) K512_STORE(1) K512_STORE(2) K512_STORE(3) K512_STORE(4) K512_STORE(5) K512_STORE(6)
    K512_STORE(7)
}

#define K256_ROW(i) v8 c##i##0 = z, c##i##1 = z;
#define K256_FMA(i)                        \
    {                                      \
        const float s_ = A[k * 6 + (i)];   \
        const v8 a = BCAST8(s_);           \
        c##i##0 += a * b0;                 \
        c##i##1 += a * b1;                 \
    }
#define K256_STORE(i)                                                  \
    {                                                                  \
        v8u* r = (v8u*)(C + (i) * ldc);                                \
        if (acc) { r[0] += c##i##0; r[1] += c##i##1; }                 \
        else { r[0] = c##i##0; r[1] = c##i##1; }                       \
    }

__attribute__((target("avx2,fma"))) static void kern_6x16(int64_t kc, const float* A, const float* B, float* C,
                                                           int64_t ldc, int acc) {
    const v8 z = {0};
    K256_ROW(0) K256_ROW(1) K256_ROW(2) K256_ROW(3) K256_ROW(4) K256_ROW(5)
    for (int64_t k = 0; k < kc; ++k) {
        const v8 b0 = *(const v8*)(B + k * 16);
        const v8 b1 = *(const v8*)(B + k * 16 + 8);
        K256_FMA(0) K256_FMA(1) K256_FMA(2) K256_FMA(3) K256_FMA(4) K256_FMA(5)
    }
    K256_STORE(0) K256_STORE(1) K256_STORE(2) K256_STORE(3) K256_STORE(4) K256_STORE(5)
}

typedef struct {
    int mr, nr;
    kern_fn kern;
} Kernel;

static Kernel pick_kernel(void) {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f")) return (Kernel){8, 32, kern_8x32};
    return (Kernel){6, 16, kern_6x16};
}

/* B[pc : pc + kc, jc + j0 : jc + j0 + NR] into a strip laid out [k][NR],
 * zero-padded past N. */
static void pack_b_strip(const Mat* B, int64_t pc, int64_t kc, int64_t col0, int64_t ncols, int NR, float* dst) {
    if (B->cs == 1 || ncols == 1) {
        for (int64_t k = 0; k < kc; ++k) {
            float* d = dst + k * NR;
            int64_t j = 0;
            if (B->bf16) {
                const uint16_t* s = (const uint16_t*)B->p + (pc + k) * B->rs + col0 * B->cs;
                for (; j < ncols; ++j) d[j] = bf(s[j * B->cs]);
            } else {
                const float* s = (const float*)B->p + (pc + k) * B->rs + col0 * B->cs;
                for (; j < ncols; ++j) d[j] = s[j * B->cs];
            }
            for (; j < NR; ++j) d[j] = 0.0f;
        }
    } else {
        for (int64_t j = 0; j < NR; ++j) {
            if (j >= ncols) {
                for (int64_t k = 0; k < kc; ++k) dst[k * NR + j] = 0.0f;
                continue;
            }
            if (B->bf16) {
                const uint16_t* s = (const uint16_t*)B->p + pc * B->rs + (col0 + j) * B->cs;
                for (int64_t k = 0; k < kc; ++k) dst[k * NR + j] = bf(s[k * B->rs]);
            } else {
                const float* s = (const float*)B->p + pc * B->rs + (col0 + j) * B->cs;
                for (int64_t k = 0; k < kc; ++k) dst[k * NR + j] = s[k * B->rs];
            }
        }
    }
}

/* A[ic : ic + mc, pc : pc + kc] into MR-high strips laid out [k][MR],
 * zero-padded past M. */
static void pack_a_block(const Mat* A, int64_t ic, int64_t mc, int64_t pc, int64_t kc, int MR, float* dst) {
    for (int64_t s0 = 0; s0 < mc; s0 += MR) {
        float* d = dst + s0 * kc;
        const int64_t rows = mc - s0 < MR ? mc - s0 : MR;
        if (A->rs == 1 && rows > 1) {
            for (int64_t k = 0; k < kc; ++k) {
                int64_t i = 0;
                for (; i < rows; ++i) d[k * MR + i] = mat_at(A, ic + s0 + i, pc + k);
                for (; i < MR; ++i) d[k * MR + i] = 0.0f;
            }
        } else {
            for (int64_t i = 0; i < MR; ++i) {
                if (i >= rows) {
                    for (int64_t k = 0; k < kc; ++k) d[k * MR + i] = 0.0f;
                    continue;
                }
                if (A->bf16) {
                    const uint16_t* s = (const uint16_t*)A->p + (ic + s0 + i) * A->rs + pc * A->cs;
                    for (int64_t k = 0; k < kc; ++k) d[k * MR + i] = bf(s[k * A->cs]);
                } else {
                    const float* s = (const float*)A->p + (ic + s0 + i) * A->rs + pc * A->cs;
                    for (int64_t k = 0; k < kc; ++k) d[k * MR + i] = s[k * A->cs];
                }
            }
        }
    }
}

/* C[M x N] (row-major, ldc) = A[M x K] . B[K x N], fp32 accumulation. */
static int gemm_f32(int64_t M, int64_t N, int64_t K, Mat A, Mat B, float* C, int64_t ldc) {
    const Kernel kn = pick_kernel();
    const int MR = kn.mr, NR = kn.nr;
    const int64_t nc_max = NC < N ? NC : N;
    const int64_t nc_pad = (nc_max + NR - 1) / NR * NR;
    float* Bp = aligned_alloc(64, (size_t)KC * nc_pad * sizeof(float) + 64);
    if (!Bp) return -1;
    int failed = 0;
#pragma omp parallel
    {
        float* Ap = aligned_alloc(64, (size_t)(MC + MR) * KC * sizeof(float) + 64);
        float* edge = aligned_alloc(64, (size_t)MR * NR * sizeof(float) + 64);
        if (!Ap || !edge) {
#pragma omp atomic write
            failed = 1;
        }
        for (int64_t jc = 0; jc < N; jc += NC) {
            const int64_t nc = N - jc < NC ? N - jc : NC;
            const int64_t strips = (nc + NR - 1) / NR;
            for (int64_t pc = 0; pc < K; pc += KC) {
                const int64_t kc = K - pc < KC ? K - pc : KC;
#pragma omp for schedule(static)
                for (int64_t s = 0; s < strips; ++s) {
                    const int64_t j0 = s * NR;
                    pack_b_strip(&B, pc, kc, jc + j0, nc - j0 < NR ? nc - j0 : NR, NR, Bp + s * NR * kc);
                }
                /* implicit barrier: the panel is complete */
#pragma omp for schedule(dynamic, 1)
                for (int64_t ic = 0; ic < M; ic += MC) {
                    if (!Ap || !edge) continue;
                    const int64_t mc = M - ic < MC ? M - ic : MC;
                    pack_a_block(&A, ic, mc, pc, kc, MR, Ap);
                    for (int64_t s = 0; s < strips; ++s) {
                        const int64_t j0 = s * NR;
                        const int64_t nr = nc - j0 < NR ? nc - j0 : NR;
                        const float* bs = Bp + s * NR * kc;
                        for (int64_t i0 = 0; i0 < mc; i0 += MR) {
                            const int64_t mr = mc - i0 < MR ? mc - i0 : MR;
                            float* c = C + (ic + i0) * ldc + jc + j0;
                            if (mr == MR && nr == NR) {
                                kn.kern(kc, Ap + i0 * kc, bs, c, ldc, pc > 0);
                            } else {
                                kn.kern(kc, Ap + i0 * kc, bs, edge, NR, 0);
                                for (int64_t i = 0; i < mr; ++i)
                                    for (int64_t j = 0; j < nr; ++j)
                                        c[i * ldc + j] = (pc > 0 ? c[i * ldc + j] : 0.0f) + edge[i * NR + j];
                            }
                        }
                    }
                }
                /* implicit barrier: the panel may be refilled */
            }
        }
        free(Ap);
        free(edge);
    }
    free(Bp);
    return failed ? -1 : 0;
}

/* ------------------------------------------------------------ the step -- */

/* One SGD step on `rows` samples; weights updated in place (bf16).
 * x, t: [rows, D]; w1: [H, D]; b1: [H]; w2: [D, H]; b2: [D]. */
int orc_mlp_step(int rows, int D, int H, const uint16_t* x, const uint16_t* t, uint16_t* w1,
                 uint16_t* b1, uint16_t* w2, uint16_t* b2, float lr, float* loss_out) {
    const int64_t RD = (int64_t)rows * D, RH = (int64_t)rows * H, HD = (int64_t)H * D;
    float* h = malloc(sizeof(float) * RH);
    float* a = malloc(sizeof(float) * RH);
    float* o = malloc(sizeof(float) * RD);
    float* dout = malloc(sizeof(float) * RD);
    float* dh = malloc(sizeof(float) * RH);
    float* dw = malloc(sizeof(float) * HD);
    int rc = 0;
    if (!h || !a || !o || !dout || !dh || !dw) {
        rc = -1;
        goto done;
    }
    /* h = x @ w1^T + b1 ; a = gelu(h)   (each result stored as bf16) */
    rc |= gemm_f32(rows, H, D, (Mat){x, 1, D, 1}, (Mat){w1, 1, 1, D}, h, H);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < RH; ++i) {
        const float hv = rbf(h[i] + bf(b1[i % H]));
        h[i] = hv;
        a[i] = rbf(gelu(hv));
    }
    /* o = a @ w2^T + b2 */
    rc |= gemm_f32(rows, D, H, (Mat){a, 0, H, 1}, (Mat){w2, 1, 1, H}, o, D);
    /* diff, loss = mean(diff^2), dout = 2 diff / numel */
    double loss = 0.0;
    const float scale = 2.0f / (float)RD;
#pragma omp parallel for schedule(static) reduction(+ : loss)
    for (int64_t i = 0; i < RD; ++i) {
        const float ov = rbf(o[i] + bf(b2[i % D]));
        const float d = rbf(ov - bf(t[i]));
        const float sq = rbf(d * d);
        loss += sq;
        dout[i] = rbf(d * scale);
    }
    *loss_out = (float)(loss / (double)RD);
    /* da = dout @ w2 ; dh = gelu'(h) * da   (w2 before its update) */
    rc |= gemm_f32(rows, H, D, (Mat){dout, 0, D, 1}, (Mat){w2, 1, H, 1}, dh, H);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < RH; ++i) dh[i] = rbf(rbf(dh[i]) * gelu_grad(h[i]));
    /* dW2 = dout^T a ; db2 = sum_r dout ; SGD on w2, b2 */
    rc |= gemm_f32(D, H, rows, (Mat){dout, 0, 1, D}, (Mat){a, 0, H, 1}, dw, H);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < HD; ++p) w2[p] = tobf(bf(w2[p]) - lr * rbf(dw[p]));
#pragma omp parallel for schedule(static)
    for (int i = 0; i < D; ++i) {
        float db = 0.0f;
        for (int r = 0; r < rows; ++r) db += dout[(int64_t)r * D + i];
        b2[i] = tobf(bf(b2[i]) - lr * rbf(db));
    }
    /* dW1 = dh^T x ; db1 = sum_r dh ; SGD on w1, b1 */
    rc |= gemm_f32(H, D, rows, (Mat){dh, 0, 1, H}, (Mat){x, 1, D, 1}, dw, D);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < HD; ++p) w1[p] = tobf(bf(w1[p]) - lr * rbf(dw[p]));
#pragma omp parallel for schedule(static)
    for (int j = 0; j < H; ++j) {
        float db = 0.0f;
        for (int r = 0; r < rows; ++r) db += dh[(int64_t)r * H + j];
        b1[j] = tobf(bf(b1[j]) - lr * rbf(db));
    }
done:
    free(h); free(a); free(o); free(dout); free(dh); free(dw);
    return rc;
}

/* The blocked product on its own (fp32 operands, any strides), so tests can
 * check it against a plain dot-product loop. */
int orc_gemm_blocked(int64_t M, int64_t N, int64_t K, const float* a, int64_t a_rs, int64_t a_cs,
                     const float* b, int64_t b_rs, int64_t b_cs, float* c) {
    return gemm_f32(M, N, K, (Mat){a, 0, a_rs, a_cs}, (Mat){b, 0, b_rs, b_cs}, c, N);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
