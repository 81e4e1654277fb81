// Unary math, activations and their backward kernels (tensorplay-mlu:
// UnaryKernels.cpp, CNNL activation kernels there).  Each operator gets its
// own dense-path kernels (ew_common.cuh); 16-bit floats use the narrow-output
// math of ew_common.cuh.

#include "ew_common.cuh"

using namespace tpb;

namespace {

int tensor_device(const tpb_tensor& t) { return device_of(t.data); }

void require_same_shape(const tpb_tensor& a, const tpb_tensor& b, const char* what) {
    TPB_CHECK(a.ndim == b.ndim, "%s: rank mismatch (%d vs %d)", what, a.ndim, b.ndim);
    for (int i = 0; i < a.ndim; ++i) {
        TPB_CHECK(a.sizes[i] == b.sizes[i], "%s: size mismatch at dimension %d (%lld vs %lld)", what,
                  i, (long long)a.sizes[i], (long long)b.sizes[i]);
    }
}

#define TPB_UNARY_CASE(OPC)                                                                      \
    case OPC:                                                                                    \
        launch_elementwise<T, 1>("unary", out, x, nullptr, L, UnaryCt<C, Fast, OPC>{p},          \
                                 UnaryF<C, Fast>{op, p}, dev, s);                                \
        break;

template <typename T>
void dispatch_unary(int op, T* out, const T* x, const Layout& L, double pd, int dev, cudaStream_t s) {
    using C = typename Compute<T>::type;
    constexpr bool Fast = Narrow<T>::value;
    const C p = static_cast<C>(pd);
    if constexpr (std::is_integral<C>::value) {
        switch (op) {
            TPB_UNARY_CASE(TPB_NEG)
            TPB_UNARY_CASE(TPB_ABS)
            TPB_UNARY_CASE(TPB_RELU)
            TPB_UNARY_CASE(TPB_SQUARE)
            default: TPB_UNARY_CASE(TPB_POW)
        }
    } else {
        switch (op) {
            TPB_UNARY_CASE(TPB_EXP)
            TPB_UNARY_CASE(TPB_LOG)
            TPB_UNARY_CASE(TPB_SQRT)
            TPB_UNARY_CASE(TPB_RSQRT)
            TPB_UNARY_CASE(TPB_NEG)
            TPB_UNARY_CASE(TPB_ABS)
            TPB_UNARY_CASE(TPB_POW)
            TPB_UNARY_CASE(TPB_RELU)
            TPB_UNARY_CASE(TPB_SIGMOID)
            TPB_UNARY_CASE(TPB_TANH)
            TPB_UNARY_CASE(TPB_SILU)
            TPB_UNARY_CASE(TPB_GELU)
            TPB_UNARY_CASE(TPB_GELU_TANH)
            default: TPB_UNARY_CASE(TPB_SQUARE)
        }
    }
}
#undef TPB_UNARY_CASE

#define TPB_BACKWARD_CASE(OPC)                                                                   \
    case OPC:                                                                                    \
        launch_elementwise<T, 2>("unary_backward", dx, dy, z, L, UnaryBackwardCt<C, Fast, OPC>{p}, \
                                 UnaryBackwardF<C, Fast>{op, p}, dev, s);                        \
        break;

template <typename T>
void dispatch_backward(int op, T* dx, const T* dy, const T* z, const Layout& L, double pd, int dev,
                       cudaStream_t s) {
    using C = typename Compute<T>::type;
    constexpr bool Fast = Narrow<T>::value;
    const C p = static_cast<C>(pd);
    if constexpr (std::is_integral<C>::value) {
        switch (op) {
            default: TPB_BACKWARD_CASE(TPB_THRESHOLD_BACKWARD)
        }
    } else {
        switch (op) {
            TPB_BACKWARD_CASE(TPB_THRESHOLD_BACKWARD)
            TPB_BACKWARD_CASE(TPB_SIGMOID_BACKWARD)
            TPB_BACKWARD_CASE(TPB_TANH_BACKWARD)
            TPB_BACKWARD_CASE(TPB_GELU_BACKWARD)
            TPB_BACKWARD_CASE(TPB_GELU_TANH_BACKWARD)
            default: TPB_BACKWARD_CASE(TPB_SILU_BACKWARD)
        }
    }
}
#undef TPB_BACKWARD_CASE

}  // namespace

extern "C" {

int tp_b200_unary(int op, const tpb_tensor* out, const tpb_tensor* x, double p, void* stream) {
    return guarded([&] {
        check_tensor(out, "unary out");
        check_tensor(x, "unary x");
        TPB_CHECK(op >= TPB_EXP && op <= TPB_SQUARE, "unary: unknown op %d", op);
        TPB_CHECK(x->dtype == out->dtype, "unary: input and result dtypes differ");
        require_same_shape(*out, *x, "unary");
        const bool int_ok = op == TPB_NEG || op == TPB_ABS || op == TPB_RELU || op == TPB_SQUARE ||
                            (op == TPB_POW && p >= 0 && p == static_cast<double>(static_cast<int64_t>(p)));
        TPB_CHECK(is_floating(out->dtype) || int_ok,
                  "unary: op %d on %s needs a floating dtype; promote first", op, dtype_name(out->dtype));
        if (numel_of(*out) == 0) return;
        const int dev = tensor_device(*out);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[1] = {x};
        const Layout L = make_layout(*out, ins, 1);
        TPB_DISPATCH_ALL(out->dtype, "unary", {
            dispatch_unary<scalar_t>(op, static_cast<scalar_t*>(out->data),
                                     static_cast<const scalar_t*>(x->data), L, p, dev, s);
        });
    });
}

int tp_b200_unary_backward(int op, const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* z,
                           double p, void* stream) {
    return guarded([&] {
        check_tensor(dx, "backward dx");
        check_tensor(dy, "backward dy");
        check_tensor(z, "backward input");
        TPB_CHECK(op >= TPB_THRESHOLD_BACKWARD && op <= TPB_SILU_BACKWARD,
                  "unary_backward: unknown op %d", op);
        TPB_CHECK(dy->dtype == dx->dtype && z->dtype == dx->dtype,
                  "unary_backward: operands must share one dtype");
        TPB_CHECK(is_floating(dx->dtype) || op == TPB_THRESHOLD_BACKWARD,
                  "unary_backward: op %d needs a floating dtype", op);
        require_same_shape(*dx, *dy, "unary_backward");
        require_same_shape(*dx, *z, "unary_backward");
        if (numel_of(*dx) == 0) return;
        const int dev = tensor_device(*dx);
        DeviceGuard guard(dev);
        cudaStream_t s = resolve_stream(stream, dev);
        const tpb_tensor* ins[2] = {dy, z};
        const Layout L = make_layout(*dx, ins, 2);
        TPB_DISPATCH_ALL(dx->dtype, "unary_backward", {
            dispatch_backward<scalar_t>(op, static_cast<scalar_t*>(dx->data),
                                        static_cast<const scalar_t*>(dy->data),
                                        static_cast<const scalar_t*>(z->data), L, p, dev, s);
        });
    });
}

}  // extern "C"
