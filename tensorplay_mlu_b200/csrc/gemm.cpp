// tp_b200_gemm: shape checks and the choice between the tensor-core and the
// CUDA-core kernel (tensorplay-mlu: gemm() in BlasKernels.cpp:202-242, which
// builds CNNL descriptors and a cached plan instead).

#include "common.h"
#include "gemm.h"

using namespace tpb;

extern "C" int tp_b200_gemm(const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b,
                            const tpb_tensor* c, double alpha, double beta, int flags, void* stream) {
    return guarded([&] {
        check_tensor(out, "gemm out");
        check_tensor(a, "gemm a");
        check_tensor(b, "gemm b");
        const int nd = out->ndim;
        TPB_CHECK(nd == 2 || nd == 3, "gemm: the result must be 2-d or 3-d, got %d-d", nd);
        TPB_CHECK(a->ndim == nd && b->ndim == nd, "gemm: operands must have the result's rank");
        TPB_CHECK(a->dtype == out->dtype && b->dtype == out->dtype,
                  "gemm: operand dtypes (%s, %s) must match the result (%s)", dtype_name(a->dtype),
                  dtype_name(b->dtype), dtype_name(out->dtype));
        GemmProblem p{};
        p.dtype = out->dtype;
        p.M = out->sizes[nd - 2];
        p.N = out->sizes[nd - 1];
        p.K = a->sizes[nd - 1];
        p.batch = nd == 3 ? out->sizes[0] : 1;
        TPB_CHECK(a->sizes[nd - 2] == p.M && b->sizes[nd - 2] == p.K && b->sizes[nd - 1] == p.N,
                  "gemm: shapes [%lld x %lld] and [%lld x %lld] cannot be multiplied into [%lld x %lld]",
                  (long long)a->sizes[nd - 2], (long long)a->sizes[nd - 1], (long long)b->sizes[nd - 2],
                  (long long)b->sizes[nd - 1], (long long)p.M, (long long)p.N);
        if (nd == 3) {
            TPB_CHECK(a->sizes[0] == p.batch || a->sizes[0] == 1, "gemm: batch sizes do not match");
            TPB_CHECK(b->sizes[0] == p.batch || b->sizes[0] == 1, "gemm: batch sizes do not match");
        }
        TPB_CHECK(out->strides[nd - 1] == 1 || p.N <= 1, "gemm: the result needs unit column stride");
        p.a = a->data;
        p.sa_m = a->strides[nd - 2];
        p.sa_k = a->strides[nd - 1];
        p.sa_b = nd == 3 && a->sizes[0] != 1 ? a->strides[0] : 0;
        p.b = b->data;
        p.sb_k = b->strides[nd - 2];
        p.sb_n = b->strides[nd - 1];
        p.sb_b = nd == 3 && b->sizes[0] != 1 ? b->strides[0] : 0;
        p.c = out->data;
        p.sc_m = out->strides[nd - 2];
        p.sc_b = nd == 3 ? out->strides[0] : 0;
        p.alpha = alpha;
        p.beta = beta;
        p.flags = flags;
        if (c != nullptr && beta != 0.0) {
            check_tensor(c, "gemm addend");
            TPB_CHECK(c->dtype == out->dtype, "gemm: addend dtype must match the result");
            int64_t st[TPB_MAX_DIMS];
            broadcast_strides(*c, *out, st);
            p.cin = c->data;
            p.sci_m = st[nd - 2];
            p.sci_n = st[nd - 1];
            p.sci_b = nd == 3 ? st[0] : 0;
        }
        if (p.M == 0 || p.N == 0 || p.batch == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        if (!gemm_tc(p, dev, s)) gemm_simt(p, dev, s);
    });
}

// tp_b200_gemm_epilogue: a product whose activation (or its derivative) is
// applied in the product's epilogue on the CTA-pair tcgen05 kernel.  Problems
// that kernel does not take (other dtypes, shapes below one 256 x 256 tile,
// layouts TMA cannot store) run as the plain product followed by the
// elementwise activation kernel, which gives the same bits.
extern "C" int tp_b200_gemm_epilogue(int epilogue, const tpb_tensor* out, const tpb_tensor* aux,
                                     const tpb_tensor* a, const tpb_tensor* b, const tpb_tensor* c,
                                     double alpha, double beta, int flags, void* stream) {
    return guarded([&] {
        TPB_CHECK(epilogue == TPB_EPI_GELU || epilogue == TPB_EPI_GELU_BACKWARD,
                  "gemm_epilogue: unknown epilogue %d", epilogue);
        check_tensor(out, "gemm_epilogue out");
        check_tensor(aux, "gemm_epilogue aux");
        check_tensor(a, "gemm_epilogue a");
        check_tensor(b, "gemm_epilogue b");
        TPB_CHECK(out->ndim == 2 && a->ndim == 2 && b->ndim == 2 && aux->ndim == 2,
                  "gemm_epilogue: 2-d operands and result");
        TPB_CHECK(aux->sizes[0] == out->sizes[0] && aux->sizes[1] == out->sizes[1],
                  "gemm_epilogue: aux must have the result's shape");
        TPB_CHECK(aux->dtype == out->dtype, "gemm_epilogue: aux dtype must match the result");
        TPB_CHECK(out->dtype == TPB_BF16 || out->dtype == TPB_F16 || out->dtype == TPB_F32 || out->dtype == TPB_F64,
                  "gemm_epilogue: the activation needs a floating dtype, got %s", dtype_name(out->dtype));
        TPB_CHECK(a->sizes[0] == out->sizes[0] && b->sizes[0] == a->sizes[1] && b->sizes[1] == out->sizes[1] &&
                      a->dtype == out->dtype && b->dtype == out->dtype,
                  "gemm_epilogue: operand shapes or dtypes do not match the result");
        TPB_CHECK(aux->strides[1] == 1 || out->sizes[1] <= 1, "gemm_epilogue: aux needs unit column stride");
        if (epilogue == TPB_EPI_GELU_BACKWARD) {
            TPB_CHECK(c == nullptr || beta == 0.0, "gemm_epilogue: gelu_backward takes no addend");
            TPB_CHECK(aux->data != out->data, "gemm_epilogue: gelu_backward's result cannot overwrite its input");
        } else {
            TPB_CHECK(aux->data != out->data, "gemm_epilogue: gelu's result and pre-activation must differ");
        }
        if (numel_of(*out) == 0) return;
        const int dev = device_of(out->data);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        if (out->dtype == TPB_BF16 && a->sizes[1] > 0) {
            GemmProblem p{};
            p.dtype = out->dtype;
            p.M = out->sizes[0];
            p.N = out->sizes[1];
            p.K = a->sizes[1];
            p.batch = 1;
            p.a = a->data;
            p.sa_m = a->strides[0];
            p.sa_k = a->strides[1];
            p.b = b->data;
            p.sb_k = b->strides[0];
            p.sb_n = b->strides[1];
            p.c = out->data;
            p.sc_m = out->strides[0];
            p.alpha = alpha;
            p.beta = beta;
            p.flags = flags;
            p.epi = epilogue;
            p.aux = aux->data;
            p.saux_m = aux->strides[0];
            if (c != nullptr && beta != 0.0) {
                check_tensor(c, "gemm_epilogue addend");
                TPB_CHECK(c->dtype == out->dtype, "gemm_epilogue: addend dtype must match the result");
                int64_t st[TPB_MAX_DIMS];
                broadcast_strides(*c, *out, st);
                p.cin = c->data;
                p.sci_m = st[0];
                p.sci_n = st[1];
            }
            if ((out->strides[1] == 1 || p.N <= 1) && gemm_tc(p, dev, s)) return;
        }
        // Decomposed: the product, then the activation kernel.
        if (epilogue == TPB_EPI_GELU) {
            TPB_CHECK(tp_b200_gemm(aux, a, b, c, alpha, beta, flags, s) == 0, "%s", tp_b200_last_error());
            TPB_CHECK(tp_b200_unary(TPB_GELU, out, aux, 0.0, s) == 0, "%s", tp_b200_last_error());
        } else {
            TPB_CHECK(tp_b200_gemm(out, a, b, nullptr, alpha, 0.0, flags, s) == 0, "%s", tp_b200_last_error());
            TPB_CHECK(tp_b200_unary_backward(TPB_GELU_BACKWARD, out, out, aux, 0.0, s) == 0, "%s",
                      tp_b200_last_error());
        }
    });
}
