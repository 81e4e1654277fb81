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
