// Broadcasting binary arithmetic and its scalar forms (tensorplay-mlu:
// BinaryKernels.cpp, cnnlOpTensor / cnnlDiv_v3 / cnnlTransform_v2 there).
// Each operator gets its own dense-path kernels (ew_common.cuh).

#include "ew_common.cuh"

using namespace tpb;

namespace {

// Launch `op` with the operator fixed at compile time for the dense shapes.
template <typename T, int NIN, typename C, template <typename, bool, int> class Ct, typename Rt,
          typename... Args>
void dispatch_binary(int op, const char* what, T* out, const T* a, const T* b, const Layout& L, Rt rt,
                     int dev, cudaStream_t s, Args... args) {
    constexpr bool Fast = Narrow<T>::value;
    switch (op) {
        case TPB_ADD: launch_elementwise<T, NIN>(what, out, a, b, L, Ct<C, Fast, TPB_ADD>{args...}, rt, dev, s); break;
        case TPB_SUB: launch_elementwise<T, NIN>(what, out, a, b, L, Ct<C, Fast, TPB_SUB>{args...}, rt, dev, s); break;
        case TPB_MUL: launch_elementwise<T, NIN>(what, out, a, b, L, Ct<C, Fast, TPB_MUL>{args...}, rt, dev, s); break;
        case TPB_DIV: launch_elementwise<T, NIN>(what, out, a, b, L, Ct<C, Fast, TPB_DIV>{args...}, rt, dev, s); break;
        default: launch_elementwise<T, NIN>(what, out, a, b, L, Ct<C, Fast, TPB_RSUB>{args...}, rt, dev, s); break;
    }
}

int tensor_device(const tpb_tensor& t) { return device_of(t.data); }

}  // namespace

extern "C" {

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
            const C al = static_cast<C>(std::is_integral<C>::value
                                            ? static_cast<double>(static_cast<int64_t>(alpha))
                                            : alpha);
            dispatch_binary<scalar_t, 2, C, BinaryCt>(op, "binary", static_cast<scalar_t*>(out->data),
                                                      static_cast<const scalar_t*>(a->data),
                                                      static_cast<const scalar_t*>(b->data), L,
                                                      BinaryF<C, Narrow<scalar_t>::value>{op, al}, dev, s, al);
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
            dispatch_binary<scalar_t, 1, C, ScalarCt>(op, "binary_scalar", static_cast<scalar_t*>(out->data),
                                                      static_cast<const scalar_t*>(a->data), nullptr, L,
                                                      ScalarF<C, Narrow<scalar_t>::value>{op, scalar, al}, dev, s, scalar, al);
        });
    });
}

}  // extern "C"
