/*
 * tpb200.h -- C ABI of the B200 device backend for TensorPlay.
 *
 * Every entry point is `extern "C"`, takes plain pointers, sizes and codes,
 * and never lets a C++ exception cross the boundary.  Status convention (the
 * one tensorplay-mlu uses in tensorplay_mlu/csrc/Cncl.cpp:4-9 and
 * tensorplay_mlu/csrc/Module.cpp:15-22): an `int` return of 0 means success,
 * a negative value means failure, and the failure message is read from
 * tp_b200_last_error() (thread-local).
 *
 * Device pointers belong to the caller.  Every operator entry point is
 * asynchronous: it enqueues work on `stream` (a cudaStream_t; NULL is the CUDA
 * default stream) and returns.  Entry points whose reference signature has
 * no stream argument (the collectives) use the calling thread's current
 * stream of the device, set with tp_b200_set_stream.  Each operator
 * declaration names the tensorplay-mlu kernel it replaces (path within the
 * reference project, file:line).
 */
#ifndef TPB200_H
#define TPB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TPB_MAX_DIMS 8

/* Element-type codes.  0..7 are the codes tensorplay-mlu's collective ABI
 * uses (tensorplay_mlu/distributed.py:37-46, tensorplay_mlu/csrc/Cncl.cpp:32-44);
 * float64 and bool are added because every operator here covers them too. */
enum tpb_dtype {
    TPB_U8 = 0,
    TPB_I8 = 1,
    TPB_I16 = 2,
    TPB_I32 = 3,
    TPB_I64 = 4,
    TPB_F16 = 5,
    TPB_F32 = 6,
    TPB_BF16 = 7,
    TPB_F64 = 8,
    TPB_BOOL = 9
};

/* A strided view of device memory.  `data` points at element [0,..,0]
 * (storage offset already applied); `strides` count elements.  A 0-d tensor
 * has ndim 0 and one element. */
typedef struct tpb_tensor {
    void* data;
    int32_t dtype;
    int32_t ndim;
    int64_t sizes[TPB_MAX_DIMS];
    int64_t strides[TPB_MAX_DIMS];
} tpb_tensor;

/* ------------------------------------------------------------------------
 * Runtime (replaces tensorplay_mlu/csrc/Module.cpp:13-37,
 * tensorplay_mlu/csrc/MLURuntime.cpp:34-136, tensorplay_mlu/csrc/MLUHooks.cpp:14-53)
 * ---------------------------------------------------------------------- */

/* Module.cpp:15-22 tp_mlu_init.  Checks that the CUDA runtime answers and
 * that every visible device is sm_100 class.  0 on success (also when no
 * device is visible), 1 on failure. */
int tp_b200_init(void);
/* Module.cpp:24 tp_mlu_device_count.  0 when no driver is present. */
int tp_b200_device_count(void);
/* MLURuntime.cpp:46-56 current_device / set_device. */
int tp_b200_current_device(void);
int tp_b200_set_device(int dev);
/* MLURuntime.cpp:58-71 capability: packed major*10+minor, negative on error. */
int tp_b200_capability(int dev);
/* MLURuntime.cpp:107-110 synchronize: blocks until the device is idle. */
int tp_b200_synchronize(int dev);
/* MLURuntime.cpp:81-93 queue(index).  The stream the collectives of this
 * thread are ordered on for `dev`.  Defaults to the CUDA default stream (0),
 * the stream PyTorch also starts on. */
int tp_b200_set_stream(int dev, void* stream);
void* tp_b200_get_stream(int dev);
/* MLURuntime.cpp:112-136 copy_to_device / copy_to_host / copy_on_device and
 * MLUHooks.cpp:23-45 copy_bytes.  kind: 1 host->device, 2 device->host,
 * 3 device->device (peer-to-peer when `src_dev` differs from `dev`, over
 * NVLink instead of the reference's bounce through host memory).  When
 * `blocking` is non-zero the call returns after the bytes have landed, as
 * the reference's copies do. */
int tp_b200_memcpy(void* dst, const void* src, size_t nbytes, int kind, int dev, int src_dev,
                   void* stream, int blocking);
/* MLUHooks.cpp:47-53 memory_info: free and total bytes from the driver. */
int tp_b200_mem_get_info(int dev, size_t* free_bytes, size_t* total_bytes);
/* Module.cpp:13-37 error surface. */
const char* tp_b200_last_error(void);
/* Device-side failure word.  Kernels whose waits are bounded record a
 * non-zero code here instead of hanging; returns and clears it (0: none).
 * No reference counterpart: CNNL kernels never report this way. */
int tp_b200_take_device_error(int dev);
/* Number of kernels this library has launched since it was loaded (all
 * devices, all threads).  No reference counterpart: lets a benchmark state
 * how many of its kernels ran inside a timed region. */
int64_t tp_b200_launch_count(void);
/* Replayed recordings add the kernels one replay runs. */
/* SMs the persistent tensor-core GEMMs launched afterwards on `dev` may
 * occupy (rounded down to an even count, at least 2; sms <= 0 or >= the
 * device's count: all).  No reference counterpart: a data-parallel step
 * lowers it around a GEMM that overlaps a collective, so the collective's
 * kernels find free SMs instead of delaying the GEMM's statically
 * scheduled tiles.  Process-wide per device; affects launches, not
 * kernels already queued. */
int tp_b200_set_gemm_sm_limit(int dev, int sms);
/* Tile order of the CTA-pair tensor-core GEMMs launched afterwards on `dev`:
 * 0 (default) a fixed order (tile c + i * clusters to cluster c); non-zero
 * claimed at run time, each cluster taking the next tile when it is ready,
 * so clusters that start late (SMs held by a concurrent kernel such as a
 * collective) take fewer tiles.  Launches captured into a graph always use
 * the fixed order.  No reference counterpart (CNNL schedules internally). */
int tp_b200_set_gemm_tile_order(int dev, int dynamic);

/* ------------------------------------------------------------------------
 * Normalisation and loss (replaces tensorplay_mlu/csrc/NNKernels.cpp:59-161,
 * native_layer_norm(_backward), and :304-397, nll_loss(_backward)).
 * layer_norm: contiguous x of rows x normalized_numel; mean / rstd flat over
 * the rows in fp32 (fp64 for fp64 input); weight / bias / dx / dweight /
 * dbias may be NULL (absent / not wanted).  nll_loss: (N, C) input, (N)
 * int64 or int32 targets, optional (C) weight; reduction 0 none, 1 mean,
 * 2 sum; `out` is (N) for none, one element otherwise; total_weight one
 * element (0 for none).  A target outside [0, C) other than ignore_index
 * sets the device error word (tp_b200_take_device_error) and counts as
 * ignored.
 * ---------------------------------------------------------------------- */
int tp_b200_layer_norm(const tpb_tensor* y, const tpb_tensor* mean, const tpb_tensor* rstd,
                       const tpb_tensor* x, const tpb_tensor* weight, const tpb_tensor* bias,
                       int64_t normalized_numel, double eps, void* stream);
int tp_b200_layer_norm_backward(const tpb_tensor* dx, const tpb_tensor* dweight,
                                const tpb_tensor* dbias, const tpb_tensor* dy, const tpb_tensor* x,
                                const tpb_tensor* mean, const tpb_tensor* rstd,
                                const tpb_tensor* weight, int64_t normalized_numel, void* stream);
int tp_b200_nll_loss(const tpb_tensor* out, const tpb_tensor* total_weight, const tpb_tensor* x,
                     const tpb_tensor* target, const tpb_tensor* weight, int reduction,
                     int64_t ignore_index, void* stream);
int tp_b200_nll_loss_backward(const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* target,
                              const tpb_tensor* weight, const tpb_tensor* total_weight, int reduction,
                              int64_t ignore_index, void* stream);
/* native_dropout / native_dropout_backward (NNKernels.cpp:164-236): keep an
 * element with probability 1 - p (uniform on 24 bits from Philox-4x32-10 at
 * counter (element / 4 + offset), key seed) and scale it by 1 / (1 - p);
 * `mask` (bool) records the kept elements.  masked_scale: dx = dy * mask *
 * scale.  Contiguous operands; 0 <= p < 1 (p = 1 needs no kernel). */
int tp_b200_dropout(const tpb_tensor* out, const tpb_tensor* mask, const tpb_tensor* x, double p,
                    uint64_t seed, uint64_t offset, void* stream);
int tp_b200_masked_scale(const tpb_tensor* dx, const tpb_tensor* dy, const tpb_tensor* mask, double scale,
                         void* stream);
/* The mean-squared-error loss with its gradient in one pass (no single
 * counterpart in the reference: it is the autograd sequence sub -> pow -> mean
 * with mul for the gradient, BinaryKernels.cpp:148-248, UnaryKernels.cpp:140-186,
 * ReduceKernels.cpp:105-111): diff = out - target; loss (one element of out's
 * dtype) = mean(diff^2); grad (may be NULL) = diff * grad_scale.  diff,
 * diff^2 and grad are rounded to the dtype where those operators round;
 * the sum accumulates in fp32 (fp64 for float64) in a fixed order.
 * Contiguous operands of one floating dtype. */
int tp_b200_mse_loss(const tpb_tensor* loss, const tpb_tensor* grad, const tpb_tensor* out,
                     const tpb_tensor* target, double grad_scale, void* stream);

/* ------------------------------------------------------------------------
 * Indexing, scatter, scans, where (replaces tensorplay_mlu/csrc/
 * IndexKernels.cpp:45-352: gather, index_select, the scatter family,
 * cumsum / cumprod, where.self).  Index tensors are int64 or int32; negative
 * indices count from the end; an index outside the dimension writes nothing
 * and sets the device error word.
 *   gather:       out (index's shape) = self[.., index, ..] along dim.
 *   index_select: contiguous self / out, 0-d or 1-d index.
 *   index_add:    out[.., index[l], ..] += src[.., l, ..] (contiguous).
 *   scatter:      out (holding `self` on entry) at index along dim, over
 *                 index's shape: mode 0 replace, 1 add, 2 multiply, 3 amax,
 *                 4 amin, 5 mean (contiguous out); include_self 0 starts
 *                 the landed elements from the mode's identity.
 *   scan:         inclusive cumulative sum (product != 0: product) along
 *                 dim; contiguous input and result of one dtype.
 *   where:        out = cond ? a : b with broadcasting; cond bool.
 * ---------------------------------------------------------------------- */
int tp_b200_gather(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index, int dim,
                   void* stream);
int tp_b200_index_select(const tpb_tensor* out, const tpb_tensor* self, const tpb_tensor* index,
                         int dim, void* stream);
int tp_b200_index_add(const tpb_tensor* out, const tpb_tensor* src, const tpb_tensor* index, int dim,
                      void* stream);
int tp_b200_scatter(const tpb_tensor* out, const tpb_tensor* index, const tpb_tensor* src, int dim,
                    int mode, int include_self, void* stream);
int tp_b200_scan(int product, const tpb_tensor* out, const tpb_tensor* x, int dim, void* stream);
int tp_b200_where(const tpb_tensor* out, const tpb_tensor* cond, const tpb_tensor* a,
                  const tpb_tensor* b, void* stream);

/* ------------------------------------------------------------------------
 * Recording and replay (replaces tensorplay_mlu/csrc/GraphCapture.cpp:69-130,
 * tp_mlu_capture_*).  CUDA stream capture of the calling thread's current
 * stream of `dev` (tp_b200_set_stream; a created stream, not the default
 * one) into a graph, instantiated at the end and launched by invoke on the
 * thread's current stream.  Blocks the caching allocator hands out while
 * recording are held until reset.  One recording at a time.
 * ---------------------------------------------------------------------- */
int tp_b200_capture_ready(void);                 /* 1 when a recording can be invoked */
void tp_b200_capture_stats(int64_t out[2]);      /* blocks handed out while recording, blocks held */
int tp_b200_capture_begin(int dev);
int tp_b200_capture_end(int dev);
int tp_b200_capture_invoke(int dev);
int tp_b200_capture_reset(void);

/* ------------------------------------------------------------------------
 * Device timer for the profiler (replaces tensorplay_mlu/csrc/MLUProfiler.cpp:
 * 20-80, the prof::DeviceTimerHooks TensorPlay calls around each operation).
 * record() places a pooled timing event on the device's current library
 * stream; elapsed_ms() waits for `end` and returns 0 on success; release()
 * returns an event to the pool.  tp_b200_timer_pooled has no reference
 * counterpart (events the pool holds; for tests).
 * ---------------------------------------------------------------------- */
int tp_b200_timer_current_device(void);
void* tp_b200_timer_record(int dev);
int tp_b200_timer_elapsed_ms(void* start, void* end, float* ms);
void tp_b200_timer_release(void* event);
int64_t tp_b200_timer_pooled(void);

/* ------------------------------------------------------------------------
 * Caching allocator (replaces tensorplay_mlu/csrc/MLUAllocator.cpp:61-237 and
 * the memory entry points of tensorplay_mlu/csrc/Module.cpp:24-37)
 *
 * Stream-ordered: a freed block is tagged with the stream it was last used
 * on and goes back to that stream's pool; a block reused on another stream
 * is ordered behind an event recorded at free time.  The signatures of
 * tp_b200_malloc / tp_b200_free are the ones
 * torch.cuda.memory.CUDAPluggableAllocator loads, so the same allocator can
 * back every tensor of a host framework.
 * ---------------------------------------------------------------------- */

/* MLUAllocator.cpp:98-128 take(): rounding 512 B below 1 MiB, 2 MiB above;
 * reuse when cached <= 1.25 x request; on out-of-memory the cache is released
 * and the allocation retried once.  NULL on failure (message in last_error). */
void* tp_b200_malloc(size_t nbytes, int dev, void* stream);
/* MLUAllocator.cpp:131-141 give_back(). */
void tp_b200_free(void* ptr, size_t nbytes, int dev, void* stream);
/* Module.cpp:27-33 tp_mlu_memory_stats: allocated, reserved, peak
 * allocated, peak reserved (bytes). */
void tp_b200_memory_stats(int dev, int64_t out[4]);
/* Module.cpp:35 tp_mlu_reset_peak_memory_stats. */
void tp_b200_reset_peak_memory_stats(int dev);
/* Module.cpp:37 tp_mlu_empty_cache. */
void tp_b200_empty_cache(void);

/* ------------------------------------------------------------------------
 * Copy, cast and fill (replaces tensorplay_mlu/csrc/CopyKernels.cpp:123-345 and
 * strided_copy, tensorplay_mlu/csrc/Cnnl.cpp:127-176)
 * ---------------------------------------------------------------------- */

/* CopyKernels.cpp:222-264 device_to_device + Cnnl.cpp:153-176 strided_copy +
 * CopyKernels.cpp:123-142 cast_into: dst[i] = (dst dtype) src[i] on one
 * device, any strides, `src` broadcast to dst's shape, every dtype pair. */
int tp_b200_copy(const tpb_tensor* dst, const tpb_tensor* src, void* stream);
/* CopyKernels.cpp:266-299 fill_kernel, every dtype (float64 included).
 * Floating destinations take `value`, integer and bool ones `ivalue`. */
int tp_b200_fill(const tpb_tensor* dst, double value, int64_t ivalue, void* stream);

/* ------------------------------------------------------------------------
 * Elementwise arithmetic (replaces tensorplay_mlu/csrc/BinaryKernels.cpp:30-248)
 * ---------------------------------------------------------------------- */

enum tpb_binary_op {
    TPB_ADD = 0,  /* out = a + alpha * b   (add.Tensor, add.Scalar)     */
    TPB_SUB = 1,  /* out = a - alpha * b   (sub.Tensor, sub.Scalar)     */
    TPB_MUL = 2,  /* out = a * b                                        */
    TPB_DIV = 3,  /* out = a / b, true division                         */
    TPB_RSUB = 4  /* out = b - alpha * a   (rsub.Scalar)                */
};

/* BinaryKernels.cpp:44-146 launch_binary/binary: `a` and `b` are broadcast
 * to `out`'s shape (size-1 or stride-0 dimensions), all three of one dtype
 * (the host promotes first).  Floating types compute in fp32 (fp64 for
 * float64), integers in int64 with the result wrapped to the dtype. */
int tp_b200_binary(int op, const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b,
                   double alpha, void* stream);
/* BinaryKernels.cpp:204-248 the .Scalar forms (reference: one affine
 * transform): out = a (op) s.  Floating dtypes read `s`, integer ones `si`. */
int tp_b200_binary_scalar(int op, const tpb_tensor* out, const tpb_tensor* a, double s,
                          int64_t si, double alpha, void* stream);

/* ------------------------------------------------------------------------
 * Unary math and activations (replaces tensorplay_mlu/csrc/UnaryKernels.cpp:29-287)
 * ---------------------------------------------------------------------- */

enum tpb_unary_op {
    TPB_EXP = 0,
    TPB_LOG = 1,
    TPB_SQRT = 2,
    TPB_RSQRT = 3,
    TPB_NEG = 4,
    TPB_ABS = 5,
    TPB_POW = 6,        /* x ** p                                        */
    TPB_RELU = 7,
    TPB_SIGMOID = 8,
    TPB_TANH = 9,
    TPB_SILU = 10,
    TPB_GELU = 11,      /* exact (erf) form                              */
    TPB_GELU_TANH = 12, /* approximate="tanh"                            */
    TPB_SQUARE = 13
};

enum tpb_unary_backward_op {
    TPB_THRESHOLD_BACKWARD = 0, /* dx = x <= p ? 0 : dy      (z = x) */
    TPB_SIGMOID_BACKWARD = 1,   /* dx = dy * y * (1 - y)     (z = y) */
    TPB_TANH_BACKWARD = 2,      /* dx = dy * (1 - y * y)     (z = y) */
    TPB_GELU_BACKWARD = 3,      /* exact gelu'               (z = x) */
    TPB_GELU_TANH_BACKWARD = 4, /* tanh-approximated gelu'   (z = x) */
    TPB_SILU_BACKWARD = 5       /* silu'                     (z = x) */
};

/* UnaryKernels.cpp:29-50 unary<>, :52-80 activation, :140-186 pow.  `out`
 * and `x` have one shape and dtype; `p` is pow's exponent. */
int tp_b200_unary(int op, const tpb_tensor* out, const tpb_tensor* x, double p, void* stream);
/* UnaryKernels.cpp:82-104 activation_backward, :222-287 the *_backward
 * kernels.  `p` is threshold_backward's threshold. */
int tp_b200_unary_backward(int op, const tpb_tensor* dx, const tpb_tensor* dy,
                           const tpb_tensor* z, double p, void* stream);

/* ------------------------------------------------------------------------
 * Reductions and softmax (replaces tensorplay_mlu/csrc/ReduceKernels.cpp:21-263)
 * ---------------------------------------------------------------------- */

enum tpb_reduce_op { TPB_SUM = 0, TPB_MEAN = 1, TPB_AMAX = 2, TPB_AMIN = 3 };

/* ReduceKernels.cpp:21-95 launch_reduce/reduce: reduce `x` over the
 * dimensions whose bit is set in `dim_mask` into `out`, which has x's shape
 * with those dimensions set to 1 (keepdim layout, contiguous).  Floating
 * inputs accumulate in fp32 (fp64 for float64), integer ones in int64;
 * amax/amin are exact and propagate NaN.  `out`'s dtype may differ from
 * x's (sum of int32 into int64, sum(dtype=...)). */
int tp_b200_reduce(int op, const tpb_tensor* out, const tpb_tensor* x, uint32_t dim_mask,
                   void* stream);
/* No counterpart in the reference: tp_b200_reduce for callers that cannot
 * allocate device memory when they reduce (a process whose GPU memory is
 * reserved up front by its own pool, or a path that must not risk a
 * cudaMalloc on an allocator miss).  Same arguments, kernels, split policy
 * and results as tp_b200_reduce, but it allocates nothing: the per-block
 * partial results go to one static 8 MiB device array per GPU (held by every
 * GPU that loads the library until the process exits).  A reduction whose
 * partial results would exceed 8 MiB, whose input layout would need a
 * gathered copy, whose result dtype is neither the input's nor the
 * accumulator's, or which reduces columns under 65536 or more outer rows, is
 * rejected with an error (use tp_b200_reduce).  The first call on a device
 * is its one-time set-up: with that device current it looks up the array's
 * device address (cudaGetSymbolAddress) and loads every reduction kernel the
 * entry point can launch.  Under CUDA's lazy module loading that set-up is
 * where the array and the kernels' code take their device memory, so make
 * one call on each device before its memory is reserved by a pool, and
 * before any stream capture; no later call on that device allocates.  All
 * calls share the array, so calls whose work overlaps on the GPU race. */
int tp_b200_reduce_noalloc(int op, const tpb_tensor* out, const tpb_tensor* x, uint32_t dim_mask,
                           void* stream);
/* ReduceKernels.cpp:146-199 softmax_forward over dimension `dim`
 * (log != 0: log_softmax).  Max-subtracted, single read of the row. */
int tp_b200_softmax(int log, const tpb_tensor* out, const tpb_tensor* x, int dim, void* stream);
/* ReduceKernels.cpp:180-199 softmax_backward (_softmax_backward_data and
 * _log_softmax_backward_data): y is the forward output. */
int tp_b200_softmax_backward(int log, const tpb_tensor* dx, const tpb_tensor* dy,
                             const tpb_tensor* y, int dim, void* stream);

/* ------------------------------------------------------------------------
 * Matrix products (replaces tensorplay_mlu/csrc/BlasKernels.cpp:32-242)
 * ---------------------------------------------------------------------- */

#define TPB_GEMM_ALLOW_TF32 1  /* BlasKernels.cpp:63-66: fp32 may use TF32 */

/* BlasKernels.cpp:202-242 gemm: out = alpha * a @ b + beta * c.
 * a [M,K] or [B,M,K], b [K,N] or [B,K,N], out [M,N] or [B,M,N] with unit
 * column stride.  A transposed operand (unit stride on the M or N side) is
 * read in place, as as_operand (:40-54) does.  `c` may be NULL (beta
 * ignored), the output itself, or any tensor broadcastable to out (an addmm
 * bias [N] seen with strides (0,1)); it is read in the epilogue instead of
 * being copied into out first (:318-324).  bf16/f16 run on tcgen05 tensor
 * cores (fp32 accumulate); f32 runs exact fp32 unless TPB_GEMM_ALLOW_TF32;
 * f64 and integer types run on CUDA cores. */
int tp_b200_gemm(const tpb_tensor* out, const tpb_tensor* a, const tpb_tensor* b,
                 const tpb_tensor* c, double alpha, double beta, int flags, void* stream);

/* Epilogues that tp_b200_gemm_epilogue applies inside the product. */
enum tpb_gemm_epilogue { TPB_EPI_GELU = 1, TPB_EPI_GELU_BACKWARD = 2 };

/* A product with its activation fused into the epilogue (no single
 * counterpart in the reference: it is the sequence linear -> gelu
 * (BlasKernels.cpp:374-386 then UnaryKernels.cpp:52-80), or mm ->
 * gelu_backward (BlasKernels.cpp:250-262 then UnaryKernels.cpp:222-240), in
 * one pass over the result).  2-d operands, one floating dtype.
 *   TPB_EPI_GELU:          aux = alpha * a @ b + beta * c (the
 *                          pre-activation, kept for the backward pass),
 *                          out = gelu(aux);
 *   TPB_EPI_GELU_BACKWARD: out = gelu_backward(alpha * a @ b, aux), aux the
 *                          activation's input; no addend.
 * Each intermediate is rounded to the dtype exactly where the separate
 * operators round it, so the result has the bits of the two-operator
 * sequence.  bf16 products of at least one 256 x 256 tile run fused on the
 * tcgen05 CTA-pair kernel; others run as the two operators. */
int tp_b200_gemm_epilogue(int epilogue, const tpb_tensor* out, const tpb_tensor* aux,
                          const tpb_tensor* a, const tpb_tensor* b, const tpb_tensor* c,
                          double alpha, double beta, int flags, void* stream);

/* ------------------------------------------------------------------------
 * Collectives over NCCL (replaces tensorplay_mlu/csrc/Cncl.cpp:71-387; same
 * argument order, codes and status convention).  Each collective is ordered
 * on the calling thread's current stream of `dev` (tp_b200_set_stream).
 * Reduction codes: sum 0, prod 1, max 2, min 3.
 * ---------------------------------------------------------------------- */

const char* tp_b200_nccl_last_error(void);                       /* Cncl.cpp:74 */
int tp_b200_nccl_unique_id_bytes(void);                          /* Cncl.cpp:78 */
int tp_b200_nccl_get_unique_id(void* out);                       /* Cncl.cpp:82-96 */
int tp_b200_nccl_comm_init(int rank, int nranks, int dev, const void* id,
                           void** comm_out);                     /* Cncl.cpp:101-120 */
/* Same as tp_b200_nccl_comm_init, but the communicator is created
 * non-blocking and the call gives up after `timeout_ms` (abort + error)
 * instead of waiting for absent ranks.  No reference counterpart. */
int tp_b200_nccl_comm_init_timeout(int rank, int nranks, int dev, const void* id,
                                   int timeout_ms, void** comm_out);
/* tp_b200_nccl_comm_init_timeout with bounds on the CTAs (hence SMs) the
 * communicator's kernels occupy (ncclConfig_t minCTAs / maxCTAs; 0 keeps
 * NCCL's choice).  No reference counterpart: a data-parallel step whose
 * products leave a fixed number of SMs free beside a collective caps the
 * collective at that many. */
int tp_b200_nccl_comm_init_ctas(int rank, int nranks, int dev, const void* id, int timeout_ms,
                                int min_ctas, int max_ctas, void** comm_out);
int tp_b200_nccl_comm_destroy(void* comm);                       /* Cncl.cpp:123-135 */
int tp_b200_nccl_comm_abort(void* comm);                         /* Cncl.cpp:137-149 */
int tp_b200_nccl_comm_rank(void* comm, int* rank_out);           /* Cncl.cpp:152-163 */
int tp_b200_nccl_comm_count(void* comm, int* count_out);         /* Cncl.cpp:165-176 */
/* 0 healthy, negative with a message when the communicator reported an
 * asynchronous error.  No reference counterpart. */
int tp_b200_nccl_comm_check(void* comm);
int tp_b200_nccl_all_reduce(const void* send, void* recv, size_t count, int dtype, int op,
                            int dev, void* comm);               /* Cncl.cpp:180-197 */
int tp_b200_nccl_broadcast(const void* send, void* recv, size_t count, int dtype, int root,
                           int dev, void* comm);                /* Cncl.cpp:199-214 */
int tp_b200_nccl_reduce(const void* send, void* recv, size_t count, int dtype, int op,
                        int root, int dev, void* comm);         /* Cncl.cpp:216-234 */
int tp_b200_nccl_all_gather(const void* send, void* recv, size_t count, int dtype, int dev,
                            void* comm);                        /* Cncl.cpp:236-250 */
int tp_b200_nccl_reduce_scatter(const void* send, void* recv, size_t count, int dtype,
                                int op, int dev, void* comm);   /* Cncl.cpp:252-270 */
int tp_b200_nccl_all_to_all(const void* send, void* recv, size_t count, int dtype, int dev,
                            void* comm);                        /* Cncl.cpp:273-287 */
int tp_b200_nccl_send(const void* buf, size_t count, int dtype, int peer, int dev,
                      void* comm);                              /* Cncl.cpp:291-306 */
int tp_b200_nccl_recv(void* buf, size_t count, int dtype, int peer, int dev,
                      void* comm);                              /* Cncl.cpp:308-320 */
int tp_b200_nccl_group_start(void);                              /* Cncl.cpp:324-335 */
int tp_b200_nccl_group_end(void);                                /* Cncl.cpp:337-348 */
int tp_b200_nccl_synchronize(int dev);                           /* Cncl.cpp:351-362 */
int tp_b200_nccl_queue_idle(int dev);   /* 1 idle, 0 busy, <0 error; Cncl.cpp:366-385 */

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* TPB200_H */
