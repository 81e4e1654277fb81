/*
 * oracle.c -- CPU restatement of the operator semantics the B200 backend
 * claims.  TEST INFRASTRUCTURE ONLY: it is the checker of the CUDA path
 * (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline / reference arm)
 * and is never linked into or called by the product library.
 *
 * What it restates.  tensorplay-mlu's host path is TensorPlay's own CPU kernels
 * (every claimed operator falls back to them for integers and float64,
 * tensorplay_mlu/csrc/BinaryKernels.cpp:148-151 and siblings); TensorPlay is
 * not installed here and its device arithmetic is inside the closed CNNL
 * library, so neither can be run.  This file restates the semantics those
 * kernels share (ATen-compatible operator schemas) from the reference's call
 * sites:
 *   - broadcasting and dtype handling: tensorplay_mlu/csrc/Cnnl.cpp:178-205;
 *   - add/sub with alpha, true division: BinaryKernels.cpp:44-87 (CNNL
 *     OpTensor ADD with alpha2 = +-alpha, cnnlDiv_v3 DIV_TRUE);
 *   - scalar forms as y = alpha*x + beta: BinaryKernels.cpp:204-248
 *     (restated as x (op) s -- mathematically the same, without the
 *     reference's float truncation of alpha and beta);
 *   - unary math, pow special cases, activations (exact / tanh gelu) and their
 *     backward formulas: UnaryKernels.cpp:48-287;
 *   - reductions with keepdim then view: ReduceKernels.cpp:21-95;
 *   - max-subtracted softmax / log_softmax and their backward over
 *     [outer, dim, inner]: ReduceKernels.cpp:146-199;
 *   - C = alpha*A@B + beta*C with transposed operands: BlasKernels.cpp:202-242;
 *   - casts: CopyKernels.cpp:42-220 (16-bit floats through fp32,
 *     float -> int truncation, != 0 for bool).
 * Arithmetic: floating values in double (one rounding to the output dtype at
 * the end, so the oracle is at least as accurate as any fp32 kernel),
 * integers in int64 wrapped to the dtype -- bit-exact for integer work.
 *
 * Pinning: against PyTorch 2.11 CPU outputs (same operator schemas) committed
 * as fixtures under tests/golden/ with the script that made them, and against
 * the exact-valued cases of the reference's own tests (round trips, x*3+1,
 * single-rank collectives).  TensorPlay's CPU kernels themselves are absent,
 * so float parity against them is pinned only through that stand-in.
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "tpb200.h"

/* ------------------------------------------------------------ scalars -- */

static float bits_to_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static uint32_t float_to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* bfloat16 = the high 16 bits of an IEEE single; round to nearest even. */
static float bf16_to_float(uint16_t h) { return bits_to_float((uint32_t)h << 16); }
static uint16_t float_to_bf16(float f) {
    uint32_t u = float_to_bits(f);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* IEEE half <-> single, round to nearest even (including subnormals). */
static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ff;
    if (exp == 0) {
        if (man == 0) return bits_to_float(sign);
        float v = (float)man / 1024.0f / 16384.0f; /* man * 2^-24 */
        return sign ? -v : v;
    }
    if (exp == 31) return bits_to_float(sign | 0x7f800000u | (man << 13));
    return bits_to_float(sign | ((exp + 112) << 23) | (man << 13));
}
static uint16_t float_to_half(float f) {
    const uint32_t u = float_to_bits(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const int32_t exp = (int32_t)((u >> 23) & 0xff);
    uint32_t man = u & 0x7fffff;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0));
    const int32_t e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

static int is_float_dtype(int d) { return d == TPB_F16 || d == TPB_F32 || d == TPB_BF16 || d == TPB_F64; }

static size_t esize(int d) {
    switch (d) {
        case TPB_U8: case TPB_I8: case TPB_BOOL: return 1;
        case TPB_I16: case TPB_F16: case TPB_BF16: return 2;
        case TPB_I32: case TPB_F32: return 4;
        default: return 8;
    }
}

/* Element access: floating values as double, integer values as int64. */
static double loadf(const tpb_tensor* t, int64_t off) {
    const char* p = (const char*)t->data + off * (int64_t)esize(t->dtype);
    switch (t->dtype) {
        case TPB_F32: return *(const float*)p;
        case TPB_F64: return *(const double*)p;
        case TPB_F16: return half_to_float(*(const uint16_t*)p);
        case TPB_BF16: return bf16_to_float(*(const uint16_t*)p);
        case TPB_U8: return *(const uint8_t*)p;
        case TPB_I8: return *(const int8_t*)p;
        case TPB_I16: return *(const int16_t*)p;
        case TPB_I32: return *(const int32_t*)p;
        case TPB_I64: return (double)*(const int64_t*)p;
        default: return *(const uint8_t*)p ? 1.0 : 0.0;
    }
}
static int64_t loadi(const tpb_tensor* t, int64_t off) {
    const char* p = (const char*)t->data + off * (int64_t)esize(t->dtype);
    switch (t->dtype) {
        case TPB_U8: return *(const uint8_t*)p;
        case TPB_I8: return *(const int8_t*)p;
        case TPB_I16: return *(const int16_t*)p;
        case TPB_I32: return *(const int32_t*)p;
        case TPB_I64: return *(const int64_t*)p;
        case TPB_BOOL: return *(const uint8_t*)p ? 1 : 0;
        default: return (int64_t)loadf(t, off); /* float -> int truncates */
    }
}
/* Store a double into any dtype: 16-bit floats via fp32, ints truncate. */
static void storef(const tpb_tensor* t, int64_t off, double v) {
    char* p = (char*)t->data + off * (int64_t)esize(t->dtype);
    switch (t->dtype) {
        case TPB_F32: *(float*)p = (float)v; break;
        case TPB_F64: *(double*)p = v; break;
        case TPB_F16: *(uint16_t*)p = float_to_half((float)v); break;
        case TPB_BF16: *(uint16_t*)p = float_to_bf16((float)v); break;
        case TPB_BOOL: *(uint8_t*)p = v != 0.0; break;
        case TPB_U8: *(uint8_t*)p = (uint8_t)(int64_t)v; break;
        case TPB_I8: *(int8_t*)p = (int8_t)(int64_t)v; break;
        case TPB_I16: *(int16_t*)p = (int16_t)(int64_t)v; break;
        case TPB_I32: *(int32_t*)p = (int32_t)(int64_t)v; break;
        default: *(int64_t*)p = (int64_t)v; break;
    }
}
static void storei(const tpb_tensor* t, int64_t off, int64_t v) {
    char* p = (char*)t->data + off * (int64_t)esize(t->dtype);
    switch (t->dtype) {
        case TPB_U8: *(uint8_t*)p = (uint8_t)v; break;
        case TPB_I8: *(int8_t*)p = (int8_t)v; break;
        case TPB_I16: *(int16_t*)p = (int16_t)v; break;
        case TPB_I32: *(int32_t*)p = (int32_t)v; break;
        case TPB_I64: *(int64_t*)p = v; break;
        case TPB_BOOL: *(uint8_t*)p = v != 0; break;
        default: storef(t, off, (double)v); break;
    }
}

/* ------------------------------------------------------------ shapes -- */

static int64_t numel(const tpb_tensor* t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->sizes[i];
    return n;
}

/* Strides of `t` seen at `out`'s shape (right-aligned broadcasting). */
static int bstrides(const tpb_tensor* t, const tpb_tensor* out, int64_t* st) {
    const int off = out->ndim - t->ndim;
    if (off < 0) return -1;
    for (int i = 0; i < out->ndim; ++i) {
        if (i < off) { st[i] = 0; continue; }
        const int64_t s = t->sizes[i - off];
        if (s != out->sizes[i] && s != 1) return -1;
        st[i] = (s == 1) ? 0 : t->strides[i - off];
    }
    return 0;
}

/* Offset of linear index `i` (row-major over `sizes`) with strides `st`. */
static int64_t offset_of(int64_t i, int ndim, const int64_t* sizes, const int64_t* st) {
    int64_t off = 0;
    for (int d = ndim - 1; d >= 0; --d) {
        const int64_t q = i / sizes[d];
        off += (i - q * sizes[d]) * st[d];
        i = q;
    }
    return off;
}

/* ----------------------------------------------------------- elementwise -- */

static double binf(int op, double a, double b, double alpha) {
    switch (op) {
        case TPB_ADD: return a + alpha * b;
        case TPB_SUB: return a - alpha * b;
        case TPB_MUL: return a * b;
        case TPB_DIV: return a / b;
        default: return b - alpha * a;
    }
}
static int64_t bini(int op, int64_t a, int64_t b, int64_t alpha) {
    /* two's-complement wrap: compute in uint64 */
    const uint64_t ua = (uint64_t)a, ub = (uint64_t)b, ual = (uint64_t)alpha;
    switch (op) {
        case TPB_ADD: return (int64_t)(ua + ual * ub);
        case TPB_SUB: return (int64_t)(ua - ual * ub);
        case TPB_MUL: return (int64_t)(ua * ub);
        case TPB_DIV: return b == 0 ? 0 : a / b;
        default: return (int64_t)(ub - ual * ua);
    }
}

int orc_copy(const tpb_tensor* dst, const tpb_tensor* src) {
    int64_t st[TPB_MAX_DIMS], sd[TPB_MAX_DIMS];
    if (bstrides(src, dst, st)) return -1;
    for (int i = 0; i < dst->ndim; ++i) sd[i] = dst->strides[i];
    const int64_t n = numel(dst);
    const int fsrc = is_float_dtype(src->dtype);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) {
        const int64_t od = offset_of(i, dst->ndim, dst->sizes, sd);
        const int64_t os = offset_of(i, dst->ndim, dst->sizes, st);
        if (fsrc) storef(dst, od, loadf(src, os));
        else storei(dst, od, loadi(src, os));
    }
    return 0;
}

int orc_fill(const tpb_tensor* dst, double v, int64_t iv) {
    const int64_t n = numel(dst);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t od = offset_of(i, dst->ndim, dst->sizes, dst->strides);
        if (is_float_dtype(dst->dtype)) storef(dst, od, v);
        else storei(dst, od, iv);
    }
    return 0;
}

int orc_binary(int op, const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b, double alpha) {
    int64_t sa[TPB_MAX_DIMS], sb[TPB_MAX_DIMS];
    if (bstrides(a, out, sa) || bstrides(b, out, sb)) return -1;
    const int64_t n = numel(out);
    const int fl = is_float_dtype(out->dtype);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) {
        const int64_t oo = offset_of(i, out->ndim, out->sizes, out->strides);
        const int64_t oa = offset_of(i, out->ndim, out->sizes, sa);
        const int64_t ob = offset_of(i, out->ndim, out->sizes, sb);
        if (fl) storef(out, oo, binf(op, loadf(a, oa), loadf(b, ob), alpha));
        else storei(out, oo, bini(op, loadi(a, oa), loadi(b, ob), (int64_t)alpha));
    }
    return 0;
}

int orc_binary_scalar(int op, const tpb_tensor* out, const tpb_tensor* a, double s, int64_t si,
                      double alpha) {
    int64_t sa[TPB_MAX_DIMS];
    if (bstrides(a, out, sa)) return -1;
    const int64_t n = numel(out);
    const int fl = is_float_dtype(out->dtype);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) {
        const int64_t oo = offset_of(i, out->ndim, out->sizes, out->strides);
        const int64_t oa = offset_of(i, out->ndim, out->sizes, sa);
        if (fl) storef(out, oo, binf(op, loadf(a, oa), s, alpha));
        else storei(out, oo, bini(op, loadi(a, oa), si, (int64_t)alpha));
    }
    return 0;
}

static double pow_special(double x, double p) {
    if (p == 2.0) return x * x;
    if (p == 1.0) return x;
    if (p == 0.0) return 1.0;
    if (p == 3.0) return x * x * x;
    if (p == 0.5) return sqrt(x);
    if (p == -0.5) return 1.0 / sqrt(x);
    if (p == -1.0) return 1.0 / x;
    if (p == -2.0) return 1.0 / (x * x);
    return pow(x, p);
}

static double unf(int op, double x, double p) {
    switch (op) {
        case TPB_EXP: return exp(x);
        case TPB_LOG: return log(x);
        case TPB_SQRT: return sqrt(x);
        case TPB_RSQRT: return 1.0 / sqrt(x);
        case TPB_NEG: return -x;
        case TPB_ABS: return fabs(x);
        case TPB_POW: return pow_special(x, p);
        case TPB_RELU: return (x > 0 || x != x) ? x : 0.0;
        case TPB_SIGMOID: return 1.0 / (1.0 + exp(-x));
        case TPB_TANH: return tanh(x);
        case TPB_SILU: return x / (1.0 + exp(-x));
        case TPB_GELU: return 0.5 * x * (1.0 + erf(x * 0.70710678118654752440));
        case TPB_GELU_TANH: {
            const double inner = 0.79788456080286535588 * (x + 0.044715 * x * x * x);
            return 0.5 * x * (1.0 + tanh(inner));
        }
        default: return x * x;
    }
}
static int64_t uni(int op, int64_t x, double p) {
    switch (op) {
        case TPB_NEG: return (int64_t)(0 - (uint64_t)x);
        case TPB_ABS: return x < 0 ? (int64_t)(0 - (uint64_t)x) : x;
        case TPB_RELU: return x > 0 ? x : 0;
        case TPB_SQUARE: return (int64_t)((uint64_t)x * (uint64_t)x);
        default: {
            uint64_t r = 1, b = (uint64_t)x;
            for (int64_t e = (int64_t)p; e > 0; e >>= 1) {
                if (e & 1) r *= b;
                b *= b;
            }
            return (int64_t)r;
        }
    }
}

int orc_unary(int op, const tpb_tensor* out, const tpb_tensor* x, double p) {
    const int64_t n = numel(out);
    const int fl = is_float_dtype(out->dtype);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) {
        const int64_t oo = offset_of(i, out->ndim, out->sizes, out->strides);
        const int64_t ox = offset_of(i, x->ndim, x->sizes, x->strides);
        if (fl) storef(out, oo, unf(op, loadf(x, ox), p));
        else storei(out, oo, uni(op, loadi(x, ox), p));
    }
    return 0;
}

static double ubf(int op, double dy, double z, double p) {
    switch (op) {
        case TPB_THRESHOLD_BACKWARD: return z <= p ? 0.0 : dy;
        case TPB_SIGMOID_BACKWARD: return dy * (1.0 - z) * z;
        case TPB_TANH_BACKWARD: return dy * (1.0 - z * z);
        case TPB_GELU_BACKWARD: {
            const double cdf = 0.5 * (1.0 + erf(z * 0.70710678118654752440));
            const double pdf = exp(-0.5 * z * z) * 0.39894228040143267794;
            return dy * (cdf + z * pdf);
        }
        case TPB_GELU_TANH_BACKWARD: {
            const double kb = 0.79788456080286535588, kk = 0.044715;
            const double x2 = z * z;
            const double t = tanh(kb * (z + kk * x2 * z));
            const double left = 0.5 * z, right = 1.0 + t;
            return dy * (0.5 * right + left * (1.0 - t * t) * kb * (1.0 + 3.0 * kk * x2));
        }
        default: {
            const double s = 1.0 / (1.0 + exp(-z));
            return dy * s * (1.0 + z * (1.0 - s));
        }
    }
}

int orc_unary_backward(int op, const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* z, double p) {
    const int64_t n = numel(dx);
    const int fl = is_float_dtype(dx->dtype);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t i = 0; i < n; ++i) {
        const int64_t o0 = offset_of(i, dx->ndim, dx->sizes, dx->strides);
        const int64_t o1 = offset_of(i, dy->ndim, dy->sizes, dy->strides);
        const int64_t o2 = offset_of(i, z->ndim, z->sizes, z->strides);
        if (fl) storef(dx, o0, ubf(op, loadf(dy, o1), loadf(z, o2), p));
        else storei(dx, o0, (op == TPB_THRESHOLD_BACKWARD && loadi(z, o2) <= (int64_t)p) ? 0 : loadi(dy, o1));
    }
    return 0;
}

/* ----------------------------------------------------------- reductions -- */

int orc_reduce(int op, const tpb_tensor* out, const tpb_tensor* x, uint32_t mask) {
    if (out->ndim != x->ndim) return -1;
    const int nd = x->ndim;
    int64_t rsizes[TPB_MAX_DIMS], rstr[TPB_MAX_DIMS], ksizes[TPB_MAX_DIMS], kstr[TPB_MAX_DIMS];
    int nr = 0, nk = 0;
    for (int i = 0; i < nd; ++i) {
        if ((mask >> i) & 1) { rsizes[nr] = x->sizes[i]; rstr[nr++] = x->strides[i]; }
        else { ksizes[nk] = x->sizes[i]; kstr[nk++] = x->strides[i]; }
    }
    int64_t R = 1, K = 1;
    for (int i = 0; i < nr; ++i) R *= rsizes[i];
    for (int i = 0; i < nk; ++i) K *= ksizes[i];
    const int fl = is_float_dtype(x->dtype);
    const int fout = is_float_dtype(out->dtype);
#pragma omp parallel for schedule(static) if (K > 16)
    for (int64_t k = 0; k < K; ++k) {
        const int64_t base = offset_of(k, nk, ksizes, kstr);
        double accf = op == TPB_AMAX ? -INFINITY : op == TPB_AMIN ? INFINITY : 0.0;
        int64_t acci = op == TPB_AMAX ? INT64_MIN : op == TPB_AMIN ? INT64_MAX : 0;
        int nan = 0;
        for (int64_t r = 0; r < R; ++r) {
            const int64_t off = base + offset_of(r, nr, rsizes, rstr);
            if (fl) {
                const double v = loadf(x, off);
                if (v != v) nan = 1;
                if (op == TPB_AMAX) accf = v > accf ? v : accf;
                else if (op == TPB_AMIN) accf = v < accf ? v : accf;
                else accf += v;
            } else {
                const int64_t v = loadi(x, off);
                if (op == TPB_AMAX) acci = v > acci ? v : acci;
                else if (op == TPB_AMIN) acci = v < acci ? v : acci;
                else acci = (int64_t)((uint64_t)acci + (uint64_t)v);
            }
        }
        if (nan && (op == TPB_AMAX || op == TPB_AMIN)) accf = NAN;
        /* out is keepdim-shaped and contiguous: its k-th element */
        if (fl) {
            if (op == TPB_MEAN) accf /= (double)R;
            storef(out, k, accf);
        } else if (op == TPB_MEAN) {
            storef(out, k, (double)acci / (double)R);
        } else if (fout) {
            storef(out, k, (double)acci);
        } else {
            storei(out, k, acci);
        }
    }
    return 0;
}

static void softmax_geometry(const tpb_tensor* t, int dim, int64_t* outer, int64_t* D, int64_t* inner) {
    const int nd = t->ndim == 0 ? 1 : t->ndim;
    if (dim < 0) dim += nd;
    *outer = 1;
    *inner = 1;
    *D = t->ndim == 0 ? 1 : t->sizes[dim];
    for (int i = 0; i < dim; ++i) *outer *= t->sizes[i];
    for (int i = dim + 1; i < t->ndim; ++i) *inner *= t->sizes[i];
}

/* Inputs and outputs are contiguous for the softmax family. */
int orc_softmax(int log_, const tpb_tensor* out, const tpb_tensor* x, int dim) {
    int64_t outer, D, inner;
    softmax_geometry(x, dim, &outer, &D, &inner);
#pragma omp parallel for schedule(static) if (outer * inner > 16)
    for (int64_t t = 0; t < outer * inner; ++t) {
        const int64_t o = t / inner, i = t % inner;
        const int64_t base = o * D * inner + i;
        double m = -INFINITY;
        for (int64_t d = 0; d < D; ++d) {
            const double v = loadf(x, base + d * inner);
            if (v > m || v != v) m = v;
        }
        double s = 0.0;
        for (int64_t d = 0; d < D; ++d) s += exp(loadf(x, base + d * inner) - m);
        for (int64_t d = 0; d < D; ++d) {
            const double v = loadf(x, base + d * inner);
            storef(out, base + d * inner, log_ ? v - m - log(s) : exp(v - m) / s);
        }
    }
    return 0;
}

int orc_softmax_backward(int log_, const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* y, int dim) {
    int64_t outer, D, inner;
    softmax_geometry(dy, dim, &outer, &D, &inner);
#pragma omp parallel for schedule(static) if (outer * inner > 16)
    for (int64_t t = 0; t < outer * inner; ++t) {
        const int64_t o = t / inner, i = t % inner;
        const int64_t base = o * D * inner + i;
        double acc = 0.0;
        for (int64_t d = 0; d < D; ++d) {
            const double g = loadf(dy, base + d * inner);
            acc += log_ ? g : g * loadf(y, base + d * inner);
        }
        for (int64_t d = 0; d < D; ++d) {
            const double g = loadf(dy, base + d * inner), w = loadf(y, base + d * inner);
            storef(dx, base + d * inner, log_ ? g - exp(w) * acc : w * (g - acc));
        }
    }
    return 0;
}

/* ------------------------------------------------------------------- NN -- */

/* native_layer_norm (tensorplay_mlu/csrc/NNKernels.cpp:59-107, the ATen
 * schema it registers): contiguous rows of D elements; mean, biased
 * variance, rstd = 1 / sqrt(var + eps), y = (x - mean) * rstd * w + b (w, b
 * NULL: 1, 0).  mean / rstd are stored per row. */
int orc_layer_norm(const tpb_tensor* y, const tpb_tensor* mean, const tpb_tensor* rstd, const tpb_tensor* x,
                   const tpb_tensor* w, const tpb_tensor* b, int64_t D, double eps) {
    const int64_t rows = numel(x) / D;
#pragma omp parallel for schedule(static) if (rows > 16)
    for (int64_t r = 0; r < rows; ++r) {
        double m = 0.0;
        for (int64_t j = 0; j < D; ++j) m += loadf(x, r * D + j);
        m /= (double)D;
        double v = 0.0;
        for (int64_t j = 0; j < D; ++j) {
            const double d = loadf(x, r * D + j) - m;
            v += d * d;
        }
        v /= (double)D;
        const double rs = 1.0 / sqrt(v + eps);
        storef(mean, r, m);
        storef(rstd, r, rs);
        for (int64_t j = 0; j < D; ++j) {
            double t = (loadf(x, r * D + j) - m) * rs;
            if (w) t *= loadf(w, j);
            if (b) t += loadf(b, j);
            storef(y, r * D + j, t);
        }
    }
    return 0;
}

/* native_layer_norm_backward (NNKernels.cpp:109-161) with the forward's
 * mean / rstd: g = dy * w, xhat = (x - mean) * rstd,
 * dx = rstd * (g - mean_j(g) - xhat * mean_j(g * xhat)),
 * dw_j = sum_r dy * xhat, db_j = sum_r dy.  Outputs may be NULL. */
int orc_layer_norm_backward(const tpb_tensor* dx, const tpb_tensor* dw, const tpb_tensor* db,
                            const tpb_tensor* dy, const tpb_tensor* x, const tpb_tensor* mean,
                            const tpb_tensor* rstd, const tpb_tensor* w, int64_t D) {
    const int64_t rows = numel(x) / D;
    if (dx) {
#pragma omp parallel for schedule(static) if (rows > 16)
        for (int64_t r = 0; r < rows; ++r) {
            const double m = loadf(mean, r), rs = loadf(rstd, r);
            double s1 = 0.0, s2 = 0.0;
            for (int64_t j = 0; j < D; ++j) {
                const double g = loadf(dy, r * D + j) * (w ? loadf(w, j) : 1.0);
                s1 += g;
                s2 += g * (loadf(x, r * D + j) - m) * rs;
            }
            s1 /= (double)D;
            s2 /= (double)D;
            for (int64_t j = 0; j < D; ++j) {
                const double g = loadf(dy, r * D + j) * (w ? loadf(w, j) : 1.0);
                const double xh = (loadf(x, r * D + j) - m) * rs;
                storef(dx, r * D + j, rs * (g - s1 - xh * s2));
            }
        }
    }
    if (dw || db) {
#pragma omp parallel for schedule(static) if (D > 16)
        for (int64_t j = 0; j < D; ++j) {
            double sw = 0.0, sb = 0.0;
            for (int64_t r = 0; r < rows; ++r) {
                const double g = loadf(dy, r * D + j);
                sw += g * (loadf(x, r * D + j) - loadf(mean, r)) * loadf(rstd, r);
                sb += g;
            }
            if (dw) storef(dw, j, sw);
            if (db) storef(db, j, sb);
        }
    }
    return 0;
}

/* nll_loss (NNKernels.cpp:322-360, ATen nll_loss_forward semantics): x is
 * (N, C) log-probabilities, target (N) classes, optional weight (C).
 * out_i = -w[t_i] * x[i, t_i], 0 where t_i == ignore; total = sum of w[t_i]
 * over the samples not ignored; reduction 0: per sample (total 0),
 * 1: sum / total, 2: sum.  Returns -1 for a target outside [0, C). */
int orc_nll_loss(const tpb_tensor* out, const tpb_tensor* total, const tpb_tensor* x, const tpb_tensor* target,
                 const tpb_tensor* w, int reduction, int64_t ignore) {
    const int64_t N = x->sizes[0], C = x->sizes[1];
    double loss = 0.0, wsum = 0.0;
    for (int64_t i = 0; i < N; ++i) {
        const int64_t t = loadi(target, i * target->strides[0]);
        double li = 0.0;
        if (t != ignore) {
            if (t < 0 || t >= C) return -1;
            const double wt = w ? loadf(w, t) : 1.0;
            li = -wt * loadf(x, i * x->strides[0] + t * x->strides[1]);
            wsum += wt;
        }
        if (reduction == 0) storef(out, i, li);
        else loss += li;
    }
    if (reduction == 0) storef(total, 0, 0.0);
    else {
        storef(out, 0, reduction == 1 ? loss / wsum : loss);
        storef(total, 0, wsum);
    }
    return 0;
}

/* nll_loss_backward (NNKernels.cpp:362-397): dx zero except
 * dx[i, t_i] = -w[t_i] * g with g = dy_i (none), dy (sum), dy / total (mean). */
int orc_nll_loss_backward(const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* target,
                          const tpb_tensor* w, const tpb_tensor* total, int reduction, int64_t ignore) {
    const int64_t N = dx->sizes[0], C = dx->sizes[1];
    for (int64_t e = 0; e < N * C; ++e) storef(dx, e, 0.0);
    for (int64_t i = 0; i < N; ++i) {
        const int64_t t = loadi(target, i * target->strides[0]);
        if (t == ignore) continue;
        if (t < 0 || t >= C) return -1;
        double g = reduction == 0 ? loadf(dy, i) : loadf(dy, 0);
        if (reduction == 1) g /= loadf(total, 0);
        storef(dx, i * C + t, -(w ? loadf(w, t) : 1.0) * g);
    }
    return 0;
}

/* -------------------------------------------------------------- dropout -- */

/* Philox-4x32-10 (Salmon, Moraes, Dror and Shaw, SC 2011): ten rounds, each
 * two 32x32 -> 64-bit products (multipliers 0xD2511F53, 0xCD9E8D57) mixing
 * the four counter words with the two key words, the key bumped by the Weyl
 * constants 0x9E3779B9, 0xBB67AE85 between rounds. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n1 = (uint32_t)p1;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1, n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* native_dropout (NNKernels.cpp:164-196) with the element -> random word
 * mapping of the device kernel: element e uses word e % 4 of Philox at
 * counter (e / 4 + offset) (low / high 32 bits, then 0, 0) under key
 * seed (low, high); keep when (word >> 8) / 2^24 >= p; out = x / (1 - p). */
int orc_dropout(const tpb_tensor* out, const tpb_tensor* mask, const tpb_tensor* x, double p, uint64_t seed,
                uint64_t offset) {
    const int64_t n = numel(x);
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    const float scale = (float)(1.0 / (1.0 - p));
    for (int64_t g = 0; g < (n + 3) / 4; ++g) {
        const uint64_t c = (uint64_t)g + offset;
        const uint32_t ctr[4] = {(uint32_t)c, (uint32_t)(c >> 32), 0u, 0u};
        uint32_t w[4];
        orc_philox4x32_10(ctr, key, w);
        for (int j = 0; j < 4 && g * 4 + j < n; ++j) {
            const int64_t e = g * 4 + j;
            const float u = (float)(w[j] >> 8) * (1.0f / 16777216.0f);
            const int keep = u >= (float)p;
            storei(mask, e, keep);
            /* x * scale rounded once into the storage type (the float scale
             * times a float / 16-bit value is exact in double) */
            storef(out, e, keep ? loadf(x, e) * (double)scale : 0.0);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- index -- */

/* Offset of the multi-index of linear position `i` over `sizes` with `st`. */
static int64_t coords_offset(int64_t i, int nd, const int64_t* sizes, const int64_t* st, int64_t* coord) {
    int64_t off = 0;
    for (int d = nd - 1; d >= 0; --d) {
        const int64_t c = sizes[d] ? i % sizes[d] : 0;
        i = sizes[d] ? i / sizes[d] : 0;
        if (coord) coord[d] = c;
        off += c * st[d];
    }
    return off;
}

static int resolve(int64_t k, int64_t size, int64_t* out) {
    if (k < 0) k += size;
    if (k < 0 || k >= size) return 0;
    *out = k;
    return 1;
}

/* gather (IndexKernels.cpp:45-69, ATen gather): out[c] = self[c, c[dim] <- index[c]]. */
int orc_gather(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index, int dim) {
    const int nd = index->ndim;
    const int64_t n = numel(index);
    int64_t coord[TPB_MAX_DIMS];
    for (int64_t i = 0; i < n; ++i) {
        const int64_t io = coords_offset(i, nd, index->sizes, index->strides, coord);
        const int64_t oo = coords_offset(i, nd, index->sizes, out->strides, NULL);
        int64_t k;
        if (!resolve(loadi(index, io), self->sizes[dim], &k)) return -1;
        int64_t so = 0;
        for (int d = 0; d < nd; ++d) so += (d == dim ? k : coord[d]) * self->strides[d];
        if (is_float_dtype(self->dtype)) storef(out, oo, loadf(self, so));
        else storei(out, oo, loadi(self, so));
    }
    return 0;
}

/* index_select (IndexKernels.cpp:184-209): contiguous self / out, 1-d index. */
int orc_index_select(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index, int dim) {
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < dim; ++d) outer *= self->sizes[d];
    for (int d = dim + 1; d < self->ndim; ++d) inner *= self->sizes[d];
    const int64_t S = self->sizes[dim], L = numel(index);
    const int64_t ist = index->ndim ? index->strides[0] : 0;
    for (int64_t o = 0; o < outer; ++o)
        for (int64_t l = 0; l < L; ++l) {
            int64_t k;
            if (!resolve(loadi(index, l * ist), S, &k)) return -1;
            for (int64_t j = 0; j < inner; ++j) {
                const int64_t so = (o * S + k) * inner + j, oo = (o * L + l) * inner + j;
                if (is_float_dtype(self->dtype)) storef(out, oo, loadf(self, so));
                else storei(out, oo, loadi(self, so));
            }
        }
    return 0;
}

/* Combine of the scatter modes: 1 add, 2 multiply, 3 amax, 4 amin (5 mean adds). */
static double combf(int mode, double a, double b) {
    switch (mode) {
        case 2: return a * b;
        case 3: return (a > b || a != a) ? a : b;
        case 4: return (a < b || a != a) ? a : b;
        default: return a + b;
    }
}
static int64_t combi(int mode, int64_t a, int64_t b) {
    switch (mode) {
        case 2: return (int64_t)((uint64_t)a * (uint64_t)b);
        case 3: return a > b ? a : b;
        case 4: return a < b ? a : b;
        default: return (int64_t)((uint64_t)a + (uint64_t)b);
    }
}

/* scatter family (IndexKernels.cpp:71-115, 221-275; ATen scatter /
 * scatter_add / scatter_reduce): `out` holds self on entry; in index order,
 * out[c, c[dim] <- index[c]] (op)= src[c].  include_self 0 starts each landed
 * element from the first value scattered into it; mean divides by the count
 * (+1 with self), floor division for integers.  Values combine in double
 * (floats) or int64 (integers) and are stored after every step, as a host
 * loop over the storage type does. */
int orc_scatter(const tpb_tensor* out, const tpb_tensor* index, const tpb_tensor* src, int dim, int mode,
                int include_self) {
    const int nd = index->ndim;
    const int64_t n = numel(index), on = numel(out);
    const int fl = is_float_dtype(out->dtype);
    int64_t* count = (int64_t*)calloc((size_t)(on > 0 ? on : 1), sizeof(int64_t));
    int64_t coord[TPB_MAX_DIMS];
    for (int64_t i = 0; i < n; ++i) {
        const int64_t io = coords_offset(i, nd, index->sizes, index->strides, coord);
        const int64_t so = coords_offset(i, nd, index->sizes, src->strides, NULL);
        int64_t k;
        if (!resolve(loadi(index, io), out->sizes[dim], &k)) {
            free(count);
            return -1;
        }
        int64_t oo = 0, lin = 0;
        for (int d = 0; d < nd; ++d) {
            const int64_t c = d == dim ? k : coord[d];
            oo += c * out->strides[d];
            lin = lin * out->sizes[d] + c;
        }
        if (mode == 0) {
            if (fl) storef(out, oo, loadf(src, so));
            else storei(out, oo, loadi(src, so));
            continue;
        }
        const int first = count[lin] == 0 && !include_self;
        ++count[lin];
        if (fl) storef(out, oo, first ? loadf(src, so) : combf(mode, loadf(out, oo), loadf(src, so)));
        else storei(out, oo, first ? loadi(src, so) : combi(mode, loadi(out, oo), loadi(src, so)));
    }
    if (mode == 5) {
        for (int64_t e = 0; e < on; ++e) {
            if (count[e] == 0) continue;
            const int64_t d = count[e] + (include_self ? 1 : 0);
            if (fl) storef(out, e, loadf(out, e) / (double)d);
            else {
                const int64_t v = loadi(out, e);
                int64_t q = v / d;
                if ((v % d != 0) && ((v < 0) != (d < 0))) --q;
                storei(out, e, q);
            }
        }
    }
    free(count);
    return 0;
}

/* index_add (index_select's backward, IndexKernels.cpp:211-219): contiguous
 * out [outer, S, inner] += src [outer, L, inner] at index[l]. */
int orc_index_add(const tpb_tensor* out, const tpb_tensor* src, const tpb_tensor* index, int dim) {
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < dim; ++d) outer *= out->sizes[d];
    for (int d = dim + 1; d < out->ndim; ++d) inner *= out->sizes[d];
    const int64_t S = out->sizes[dim], L = numel(index);
    const int64_t ist = index->ndim ? index->strides[0] : 0;
    for (int64_t o = 0; o < outer; ++o)
        for (int64_t l = 0; l < L; ++l) {
            int64_t k;
            if (!resolve(loadi(index, l * ist), S, &k)) return -1;
            for (int64_t j = 0; j < inner; ++j) {
                const int64_t oo = (o * S + k) * inner + j, so = (o * L + l) * inner + j;
                if (is_float_dtype(out->dtype)) storef(out, oo, loadf(out, oo) + loadf(src, so));
                else storei(out, oo, combi(1, loadi(out, oo), loadi(src, so)));
            }
        }
    return 0;
}

/* cumsum / cumprod (IndexKernels.cpp:123-149): inclusive, along dim, over
 * contiguous input and result of one dtype; double / int64 accumulation. */
int orc_scan(int product, const tpb_tensor* out, const tpb_tensor* x, int dim) {
    int64_t outer = 1, inner = 1;
    for (int d = 0; d < dim; ++d) outer *= x->sizes[d];
    for (int d = dim + 1; d < x->ndim; ++d) inner *= x->sizes[d];
    const int64_t D = x->ndim ? x->sizes[dim] : 1;
    const int fl = is_float_dtype(x->dtype);
    for (int64_t o = 0; o < outer; ++o)
        for (int64_t j = 0; j < inner; ++j) {
            double af = product ? 1.0 : 0.0;
            int64_t ai = product ? 1 : 0;
            for (int64_t d = 0; d < D; ++d) {
                const int64_t e = (o * D + d) * inner + j;
                if (fl) {
                    af = product ? af * loadf(x, e) : af + loadf(x, e);
                    storef(out, e, af);
                } else {
                    ai = combi(product ? 2 : 1, ai, loadi(x, e));
                    storei(out, e, ai);
                }
            }
        }
    return 0;
}

/* where.self (IndexKernels.cpp:313-349): out = cond ? a : b, broadcast. */
int orc_where(const tpb_tensor* out, const tpb_tensor* cond, const tpb_tensor* a, const tpb_tensor* b) {
    int64_t sc[TPB_MAX_DIMS], sa[TPB_MAX_DIMS], sb[TPB_MAX_DIMS];
    if (bstrides(cond, out, sc) || bstrides(a, out, sa) || bstrides(b, out, sb)) return -1;
    const int64_t n = numel(out);
    for (int64_t i = 0; i < n; ++i) {
        const int64_t oo = offset_of(i, out->ndim, out->sizes, out->strides);
        const int c = loadi(cond, offset_of(i, out->ndim, out->sizes, sc)) != 0;
        const int64_t src = offset_of(i, out->ndim, out->sizes, c ? sa : sb);
        const tpb_tensor* t = c ? a : b;
        if (is_float_dtype(out->dtype)) storef(out, oo, loadf(t, src));
        else storei(out, oo, loadi(t, src));
    }
    return 0;
}

/* ----------------------------------------------------------------- GEMM -- */

/* Round an fp32 value to TF32 (10 explicit mantissa bits, nearest-even). */
static double tf32_round(double v) {
    uint32_t u = float_to_bits((float)v);
    if ((u & 0x7f800000u) == 0x7f800000u) return v;
    u += 0xfffu + ((u >> 13) & 1u);
    u &= 0xffffe000u;
    return bits_to_float(u);
}

/* out[b][m][n] = alpha * sum_k a[b][m][k] b[b][k][n] + beta * c (broadcast),
 * accumulated in double (int64 for integer types). */
int orc_gemm(const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b, const tpb_tensor* c,
             double alpha, double beta, int flags) {
    const int nd = out->ndim;
    const int64_t M = out->sizes[nd - 2], N = out->sizes[nd - 1], K = a->sizes[nd - 1];
    const int64_t B = nd == 3 ? out->sizes[0] : 1;
    const int64_t sab = nd == 3 && a->sizes[0] != 1 ? a->strides[0] : 0;
    const int64_t sbb = nd == 3 && b->sizes[0] != 1 ? b->strides[0] : 0;
    int64_t sc[TPB_MAX_DIMS] = {0};
    const int use_c = c != NULL && beta != 0.0;
    if (use_c && bstrides(c, out, sc)) return -1;
    const int fl = is_float_dtype(out->dtype);
    const int tf32 = (flags & TPB_GEMM_ALLOW_TF32) && out->dtype == TPB_F32;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bb = 0; bb < B; ++bb) {
        for (int64_t m = 0; m < M; ++m) {
            for (int64_t n = 0; n < N; ++n) {
                const int64_t oo = (nd == 3 ? bb * out->strides[0] : 0) + m * out->strides[nd - 2] +
                                   n * out->strides[nd - 1];
                if (fl) {
                    double acc = 0.0;
                    for (int64_t k = 0; k < K; ++k) {
                        double x = loadf(a, bb * sab + m * a->strides[nd - 2] + k * a->strides[nd - 1]);
                        double y = loadf(b, bb * sbb + k * b->strides[nd - 2] + n * b->strides[nd - 1]);
                        if (tf32) { x = tf32_round(x); y = tf32_round(y); }
                        acc += x * y;
                    }
                    double v = alpha * acc;
                    if (use_c) v += beta * loadf(c, (nd == 3 ? bb * sc[0] : 0) + m * sc[nd - 2] + n * sc[nd - 1]);
                    storef(out, oo, v);
                } else {
                    uint64_t acc = 0;
                    for (int64_t k = 0; k < K; ++k) {
                        acc += (uint64_t)loadi(a, bb * sab + m * a->strides[nd - 2] + k * a->strides[nd - 1]) *
                               (uint64_t)loadi(b, bb * sbb + k * b->strides[nd - 2] + n * b->strides[nd - 1]);
                    }
                    uint64_t v = (uint64_t)(int64_t)alpha * acc;
                    if (use_c) v += (uint64_t)(int64_t)beta *
                                    (uint64_t)loadi(c, (nd == 3 ? bb * sc[0] : 0) + m * sc[nd - 2] + n * sc[nd - 1]);
                    storei(out, oo, (int64_t)v);
                }
            }
        }
    }
    return 0;
}

/* Selected outputs only (for problems too large to recompute in full):
 * idx holds `count` (batch, m, n) triples; vals receives alpha*acc + beta*c in
 * double, before any rounding to the output dtype. */
int orc_gemm_sampled(double* vals, const int64_t* idx, int64_t count, const tpb_tensor* a,
                     const tpb_tensor* b, const tpb_tensor* c, double alpha, double beta, int flags) {
    const int nd = a->ndim;
    const int64_t K = a->sizes[nd - 1];
    const int64_t sab = nd == 3 && a->sizes[0] != 1 ? a->strides[0] : 0;
    const int64_t sbb = nd == 3 && b->sizes[0] != 1 ? b->strides[0] : 0;
    const int tf32 = (flags & TPB_GEMM_ALLOW_TF32) && a->dtype == TPB_F32;
    int64_t sc[TPB_MAX_DIMS] = {0};
    const int use_c = c != NULL && beta != 0.0;
    tpb_tensor shape;
    if (use_c) {
        /* broadcast c against [.., M, N]; only its own strides matter */
        shape.ndim = nd;
        for (int i = 0; i < nd; ++i) shape.sizes[i] = 1 << 30;
        const int off = nd - c->ndim;
        for (int i = 0; i < nd; ++i) sc[i] = (i < off || c->sizes[i - off] == 1) ? 0 : c->strides[i - off];
    }
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < count; ++s) {
        const int64_t bb = idx[3 * s], m = idx[3 * s + 1], n = idx[3 * s + 2];
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            double x = loadf(a, bb * sab + m * a->strides[nd - 2] + k * a->strides[nd - 1]);
            double y = loadf(b, bb * sbb + k * b->strides[nd - 2] + n * b->strides[nd - 1]);
            if (tf32) { x = tf32_round(x); y = tf32_round(y); }
            acc += x * y;
        }
        double v = alpha * acc;
        if (use_c) v += beta * loadf(c, (nd == 3 ? bb * sc[0] : 0) + m * sc[nd - 2] + n * sc[nd - 1]);
        vals[s] = v;
    }
    (void)shape;
    return 0;
}
