/*
 * mlp.c -- CPU port of one training step of the BASELINE MLP (Linear 4096 ->
 * 16384, GELU, Linear 16384 -> 4096, MSE, SGD).  TEST AND BASELINE
 * INFRASTRUCTURE ONLY: bench.py times it as the CPU path of the workload
 * (cpu_baseline / --impl reference) on a bounded sample of rows, and
 * tests/ use it to check the device step; the product never calls it.
 *
 * It performs the same operator sequence TensorPlay's autograd engine would
 * run on its CPU kernels for this model (linear, gelu, sub, pow, mean,
 * mm on transposed views, sum over dim 0, gelu_backward, add_), in the
 * precision those kernels use for bf16 tensors: values stored as bf16
 * between operators, fp32 arithmetic inside each (the accumulation type of
 * the reference's kernels, BinaryKernels.cpp:76, ReduceKernels.cpp:34,
 * BlasKernels.cpp:113).  Threads: OpenMP over rows / output features.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

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

/* One SGD step on `rows` samples; weights updated in place (bf16).
 * x, t: [rows, D]; w1: [H, D]; b1: [H]; w2: [D, H]; b2: [D]. */
int orc_mlp_step(int rows, int D, int H, const uint16_t* x, const uint16_t* t, uint16_t* w1,
                 uint16_t* b1, uint16_t* w2, uint16_t* b2, float lr, float* loss_out) {
    const int64_t RD = (int64_t)rows * D, RH = (int64_t)rows * H, HD = (int64_t)H * D;
    float* xf = malloc(sizeof(float) * RD);
    float* h = malloc(sizeof(float) * RH);
    float* a = malloc(sizeof(float) * RH);
    float* o = malloc(sizeof(float) * RD);
    float* dout = malloc(sizeof(float) * RD);
    float* da = malloc(sizeof(float) * RH);
    float* w1f = malloc(sizeof(float) * HD);
    float* w2f = malloc(sizeof(float) * HD);
    if (!xf || !h || !a || !o || !dout || !da || !w1f || !w2f) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < HD; ++i) {
        w1f[i] = bf(w1[i]);
        w2f[i] = bf(w2[i]);
    }
    for (int64_t i = 0; i < RD; ++i) xf[i] = bf(x[i]);
    /* h = x @ w1^T + b1 ; a = gelu(h)   (each result stored as bf16) */
#pragma omp parallel for collapse(2) schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int j = 0; j < H; ++j) {
            const float* xr = xf + (int64_t)r * D;
            const float* wr = w1f + (int64_t)j * D;
            float acc = 0.0f;
            for (int k = 0; k < D; ++k) acc += xr[k] * wr[k];
            const float hv = rbf(acc + bf(b1[j]));
            h[(int64_t)r * H + j] = hv;
            a[(int64_t)r * H + j] = rbf(gelu(hv));
        }
    }
    /* o = a @ w2^T + b2 */
#pragma omp parallel for collapse(2) schedule(static)
    for (int r = 0; r < rows; ++r) {
        for (int i = 0; i < D; ++i) {
            const float* ar = a + (int64_t)r * H;
            const float* wr = w2f + (int64_t)i * H;
            float acc = 0.0f;
            for (int j = 0; j < H; ++j) acc += ar[j] * wr[j];
            o[(int64_t)r * D + i] = rbf(acc + bf(b2[i]));
        }
    }
    /* diff, loss = mean(diff^2), dout = 2 diff / numel */
    double loss = 0.0;
    const float scale = 2.0f / (float)RD;
    for (int64_t i = 0; i < RD; ++i) {
        const float d = rbf(o[i] - bf(t[i]));
        const float sq = rbf(d * d);
        loss += sq;
        dout[i] = rbf(d * scale);
    }
    *loss_out = (float)(loss / (double)RD);
    /* da = dout @ w2 ; dh = gelu'(h) * da   (into da) */
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        float* dar = da + (int64_t)r * H;
        for (int j = 0; j < H; ++j) dar[j] = 0.0f;
        for (int i = 0; i < D; ++i) {
            const float g = dout[(int64_t)r * D + i];
            const float* wr = w2f + (int64_t)i * H;
            for (int j = 0; j < H; ++j) dar[j] += g * wr[j];
        }
        for (int j = 0; j < H; ++j) {
            const float dav = rbf(dar[j]);
            dar[j] = rbf(dav * gelu_grad(h[(int64_t)r * H + j]));
        }
    }
    /* dW2[i][j] = sum_r dout[r][i] a[r][j]; db2 = sum_r dout; SGD on w2, b2 */
#pragma omp parallel for schedule(static)
    for (int i = 0; i < D; ++i) {
        float* acc = malloc(sizeof(float) * H);
        for (int j = 0; j < H; ++j) acc[j] = 0.0f;
        float db = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const float g = dout[(int64_t)r * D + i];
            const float* ar = a + (int64_t)r * H;
            for (int j = 0; j < H; ++j) acc[j] += g * ar[j];
            db += g;
        }
        for (int j = 0; j < H; ++j) {
            const int64_t p = (int64_t)i * H + j;
            w2[p] = tobf(bf(w2[p]) - lr * rbf(acc[j]));
        }
        b2[i] = tobf(bf(b2[i]) - lr * rbf(db));
        free(acc);
    }
    /* dW1[j][k] = sum_r dh[r][j] x[r][k]; db1 = sum_r dh; SGD on w1, b1 */
#pragma omp parallel for schedule(static)
    for (int j = 0; j < H; ++j) {
        float* acc = malloc(sizeof(float) * D);
        for (int k = 0; k < D; ++k) acc[k] = 0.0f;
        float db = 0.0f;
        for (int r = 0; r < rows; ++r) {
            const float g = da[(int64_t)r * H + j];
            const float* xr = xf + (int64_t)r * D;
            for (int k = 0; k < D; ++k) acc[k] += g * xr[k];
            db += g;
        }
        for (int k = 0; k < D; ++k) {
            const int64_t p = (int64_t)j * D + k;
            w1[p] = tobf(bf(w1[p]) - lr * rbf(acc[k]));
        }
        b1[j] = tobf(bf(b1[j]) - lr * rbf(db));
        free(acc);
    }
    free(xf); free(h); free(a); free(o); free(dout); free(da); free(w1f); free(w2f);
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}
