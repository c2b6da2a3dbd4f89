/*
 * libtpcuda: C ABI of the B200 CUDA backend for the torch-pyodide tensor-op
 * hot path.
 *
 * It replaces the bridge python/torch/_runtime.py:15-39 -> runtime.mjs
 * (TorchPyodideRuntime, runtime/src/runtime.ts:17-1212) -> WGSL compute
 * shaders.  Two layers are exported:
 *
 *   tp_*   handle level: one entry per hot runtime.ts method, same argument
 *          order and meaning, tensors named by int64 ids owned by the library
 *          (the reference's TensorRegistry, runtime/src/ops/tensorRegistry.ts).
 *          Each op writes the new tensor's {id, shape, dtype} into a tp_handle
 *          (the reference's TensorHandle, runtime/src/ops/types.ts:10-15).
 *   tpk_*  pointer level: the same kernels on caller-owned device pointers
 *          with plain sizes, asynchronous on the library stream, no allocation
 *          (the step driver captures these in CUDA graphs).
 *
 * Every function returns 0 (TP_OK) or a negative status; tp_last_error()
 * gives the message for the calling thread.  A JS Error in the reference
 * becomes a non-zero status here and a RuntimeError in the Python shim, so the
 * reference's try/except fallbacks keep working (python/torch/optim/
 * __init__.py:193,298,404).
 *
 * Storage: every dtype is stored as float32 (runtime/src/ops/device.ts:
 * 362-364); the dtype code is a tag.  Index outputs of the new max-pool and
 * max-along-dim entries are physically int32.
 *
 * Ordering: all work runs on one CUDA stream per process (tp_get_stream),
 * except what a caller sends to the auxiliary stream between tp_aux_fork and
 * tp_aux_return; the only host synchronisation points are tp_to_host and
 * tp_synchronize, as in the reference where readbacks are the only syncs
 * (runtime.ts:1046-1050).
 * Not re-entrant across threads, like the single-threaded JS event loop.
 */
#ifndef TPCUDA_H
#define TPCUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TP_API __attribute__((visibility("default")))
#define TP_MAX_DIMS 8

/* status codes */
enum {
  TP_OK = 0,
  TP_ERR_ARG = -1,      /* bad shape / id / argument (a JS Error("...") in the reference) */
  TP_ERR_CUDA = -2,     /* CUDA runtime error */
  TP_ERR_OOM = -3,      /* device or host allocation failed */
  TP_ERR_NCCL = -4,     /* collective failed or timed out */
  TP_ERR_TIMEOUT = -5,  /* a bounded device-side wait gave up */
  TP_ERR_INTERNAL = -6
};

/* dtype tags, the SupportedDType list of runtime/src/ops/types.ts:17-29 */
enum {
  TP_FLOAT32 = 0, TP_FLOAT16 = 1, TP_BFLOAT16 = 2, TP_INT8 = 3, TP_INT16 = 4, TP_INT32 = 5,
  TP_INT64 = 6, TP_UINT8 = 7, TP_UINT16 = 8, TP_UINT32 = 9, TP_UINT64 = 10, TP_BOOL = 11
};

/* the reference TensorHandle {id, shape, dtype} (runtime/src/ops/types.ts:10-15) */
typedef struct tp_handle {
  int64_t id;
  int32_t ndim;
  int32_t dtype;
  int64_t shape[TP_MAX_DIMS];
} tp_handle;

/* ---- device, errors, stream --------------------------------------------- */
/* runtime.ts:49-51 init / device.ts:126-188 ensureReady */
TP_API int tp_init(int device);
/* runtime.ts:1056-1058 isAvailable: 1 if a CUDA device is present */
TP_API int tp_is_available(void);
/* runtime.ts:1064-1066 deviceCount */
TP_API int tp_device_count(int* out);
TP_API const char* tp_last_error(void);
TP_API int tp_synchronize(void);
/* the library's CUDA stream (cudaStream_t) for interop and event timing */
TP_API int tp_get_stream(void** out);
/* No counterpart in the reference (one WebGPU queue).  A second stream for
 * work that may overlap: after tp_aux_fork every launch of the calling thread
 * goes to the auxiliary stream, which first waits for all work queued on the
 * library stream; tp_aux_return sends launches back to the library stream
 * (no wait).  tp_aux_record(slot) marks the auxiliary stream's progress in
 * event slot (0..63); tp_main_wait(slot) makes the library stream wait for it;
 * tp_aux_join makes it wait for all auxiliary work.  Each stream has its own
 * scratch space.  tp_synchronize waits for both streams.  Inside a graph
 * capture these become the graph's fork / join edges. */
TP_API int tp_aux_fork(void);
TP_API int tp_aux_return(void);
TP_API int tp_aux_record(int slot);
TP_API int tp_main_wait(int slot);
TP_API int tp_aux_join(void);
/* New: a third stream for work that may run beside the rest of a step.  It is
 * the communicator's stream when one exists (so its work also follows the
 * all-reduces issued so far), else a library stream of its own.
 * tp_side_fork makes it wait for everything queued on the library and
 * auxiliary streams and sends the calling thread's launches there until
 * tp_side_return; tp_side_join (and, with a communicator, tp_comm_wait) makes
 * the library stream wait for it.  Used to run each gradient bucket's
 * optimizer step as soon as its gradients are final. */
TP_API int tp_side_fork(void);
TP_API int tp_side_return(void);
TP_API int tp_side_join(void);
/* runtime.ts:1084-1090 memoryAllocated / memoryReserved */
TP_API int tp_memory_allocated(int64_t* out);
TP_API int tp_memory_reserved(int64_t* out);
/* runtime.ts:1076-1082 getDeviceName */
TP_API int tp_device_name(char* buf, int len);
/* number of kernels this library has launched since load (a counter kept on
 * the host at every launch site) */
TP_API int tp_kernel_launches(int64_t* out);

/* ---- registry ------------------------------------------------------------- */
/* creationOps.ts:25-37 tensorFromData (values already coerced to f32) */
TP_API int tp_tensor_from_data(const float* host, const int64_t* shape, int ndim, int dtype, tp_handle* out);
/* runtime.ts:1046-1050 toList: copies numel f32 values (int32 index tensors
 * are converted to f32) into host memory and synchronises */
TP_API int tp_to_host(int64_t id, float* dst, int64_t numel);
/* runtime.ts:1052-1054 destroy */
TP_API int tp_destroy(int64_t id);
TP_API int tp_meta(int64_t id, tp_handle* out);
/* the device pointer behind an id (for pointer-level calls) */
TP_API int tp_device_ptr(int64_t id, void** out);
/* raw HBM allocations from the library's pool, for pointer-level calls; the
 * memcpy/memset helpers below are ordered on the library stream and
 * tp_memcpy_d2h synchronises */
TP_API int tp_alloc(int64_t bytes, void** out);
TP_API int tp_free(void* ptr);
TP_API int tp_memcpy_h2d(void* dst, const void* src, int64_t bytes);
TP_API int tp_memcpy_d2h(void* dst, const void* src, int64_t bytes);
TP_API int tp_memcpy_d2d(void* dst, const void* src, int64_t bytes);
TP_API int tp_memset(void* dst, int value, int64_t bytes);
/* New, checkpoint I/O (python/torch/_save.py:109-125 packs every tensor through
 * tolist() and struct.pack; _save.py:77-103 unpacks into a Python list for
 * tensorFromData): the tensor's values in one copy.  format 0: little-endian
 * float32 (nbytes = 4 numel); 1: little-endian int64, each value truncated
 * toward zero as toList decodes integer dtypes (nbytes = 8 numel).  Both
 * synchronise, so `dst` / `src` may be pageable and reused on return. */
TP_API int tp_to_bytes(int64_t id, void* dst, int64_t nbytes, int format);
TP_API int tp_from_bytes(const void* src, int64_t nbytes, int format, const int64_t* shape, int ndim, int dtype,
                         tp_handle* out);
/* New, input pipeline (python/torch/tensor_factories_ops.py:18-25 flattens the
 * data to a Python list per tensor): pinned host buffers, and an upload from
 * one that runs on a dedicated copy stream, overlapping the kernels already
 * queued.  defer == 0: work queued on the library streams after the call waits
 * for the copy; defer != 0: nothing waits until tp_ticket_use(ticket), which
 * the caller makes before the tensor's first use (a loader uploads batch i+2
 * while batch i computes and marks each batch used just before handing it
 * out).  *ticket names the copy: tp_ticket_wait(ticket) returns once it has
 * finished and the host buffer may be refilled. */
TP_API int tp_host_alloc(int64_t bytes, void** out);
TP_API int tp_host_free(void* ptr);
TP_API int tp_tensor_from_host_async(const void* pinned_host, const int64_t* shape, int ndim, int dtype, int defer,
                                     tp_handle* out, int64_t* ticket);
TP_API int tp_ticket_use(int64_t ticket);
TP_API int tp_ticket_wait(int64_t ticket);
/* New, batches of a device-resident dataset: out = src[rows] along dim 0 (the
 * reference DataLoader selects each sample of a TensorDataset with one runtime
 * call and stacks them, utils/data/__init__.py:24-37,205-210); rows are
 * checked against dim 0 */
TP_API int tp_gather_rows(int64_t src, const int64_t* rows, int64_t n, tp_handle* out);

/* ---- creation (creationOps.ts, random.wgsl, fill.wgsl) -------------------- */
/* zeros/ones/full/empty: creationOps.ts:39-45,107-145 (fill.wgsl) */
TP_API int tp_full(const int64_t* shape, int ndim, int dtype, float value, tp_handle* out);
/* fullLike/zerosLike/onesLike/emptyLike: creationOps.ts:111-145; dtype -1 = same */
TP_API int tp_full_like(int64_t id, int dtype, float value, tp_handle* out);
/* unaryOps.ts:171-179 fill: a new tensor of the same shape and dtype */
TP_API int tp_fill(int64_t id, float value, tp_handle* out);
/* creationOps.ts:21-23 setSeed (the counter starts at 42) */
TP_API int tp_set_seed(uint32_t seed);
/* creationOps.ts:47-101 rand/randn/normal/sampleOp: kind 0 rand, 1 randn, 2 normal(p0,p1),
 * 3 bernoulli(p0), 4 exponential(p0); consumes one seed (random.wgsl:23-91) */
TP_API int tp_random(const int64_t* shape, int ndim, int dtype, int kind, float p0, float p1, tp_handle* out);

/* ---- element-wise (arithmeticOps.ts, broadcastOps.ts, compareOps.ts, unaryOps.ts) */
/* binary op codes (elementwise.wgsl entry points; compare.wgsl) */
enum {
  TP_ADD = 0, TP_SUB = 1, TP_MUL = 2, TP_DIV = 3, TP_POW = 4, TP_MAXIMUM = 5, TP_MINIMUM = 6,
  TP_EQ = 10, TP_NE = 11, TP_LT = 12, TP_LE = 13, TP_GT = 14, TP_GE = 15
};
/* unary op codes (unary.wgsl entry points) */
enum {
  TP_NEG = 0, TP_ABS = 1, TP_SQRT = 2, TP_EXP = 3, TP_LOG = 4, TP_RELU = 5, TP_RSQRT = 6,
  TP_RECIPROCAL = 7, TP_SQUARE = 8, TP_SIGMOID = 9, TP_TANH = 10
};
/* add/sub/mul/div/pow/maximum/minimum/eq/ne/lt/le/gt/ge with right-aligned
 * broadcasting (arithmeticOps.ts:342-355, broadcastOps.ts:21-82); the
 * broadcast operand is read in place, never materialised */
TP_API int tp_binary(int op, int64_t a, int64_t b, tp_handle* out);
TP_API int tp_add(int64_t a, int64_t b, tp_handle* out);
TP_API int tp_sub(int64_t a, int64_t b, tp_handle* out);
TP_API int tp_mul(int64_t a, int64_t b, tp_handle* out);
TP_API int tp_div(int64_t a, int64_t b, tp_handle* out);
TP_API int tp_pow(int64_t a, int64_t b, tp_handle* out);
TP_API int tp_gt(int64_t a, int64_t b, tp_handle* out);
/* arithmeticOps.ts:206-219 mulScalar */
TP_API int tp_mul_scalar(int64_t a, float value, tp_handle* out);
/* unaryOps.ts:156-169 unary dispatch (relu, rsqrt, neg, ...) */
TP_API int tp_unary(int op, int64_t a, tp_handle* out);
TP_API int tp_relu(int64_t a, tp_handle* out);
TP_API int tp_rsqrt(int64_t a, tp_handle* out);
TP_API int tp_neg(int64_t a, tp_handle* out);

/* ---- shape (shapeOps.ts) ------------------------------------------------- */
/* shapeOps.ts:72-81 reshape (flatten/squeeze/unsqueeze reduce to it) */
TP_API int tp_reshape(int64_t id, const int64_t* shape, int ndim, tp_handle* out);
/* shapeOps.ts:715-725 transpose2d */
TP_API int tp_transpose2d(int64_t id, tp_handle* out);
/* shapeOps.ts:125-154 permute */
TP_API int tp_permute(int64_t id, const int32_t* dims, int ndim, tp_handle* out);
/* shapeOps.ts:305-329 expand */
TP_API int tp_expand(int64_t id, const int64_t* shape, int ndim, tp_handle* out);

/* ---- reductions (reductionOps.ts) ----------------------------------------- */
/* reductionOps.ts:161-213 reduceAll: mode 0 sum, 1 mean, 2 max; the scalar
 * stays in HBM (no host readback, unlike the reference) */
TP_API int tp_reduce_all(int64_t id, int mode, tp_handle* out);
TP_API int tp_sum(int64_t id, tp_handle* out);
TP_API int tp_mean(int64_t id, tp_handle* out);
TP_API int tp_max(int64_t id, tp_handle* out);
/* reductionOps.ts:215-251 reduceDim: mode 0 sum, 1 mean */
TP_API int tp_reduce_dim(int64_t id, int dim, int keepdim, int mode, tp_handle* out);
TP_API int tp_sum_dim(int64_t id, int dim, int keepdim, tp_handle* out);
TP_API int tp_mean_dim(int64_t id, int dim, int keepdim, tp_handle* out);
/* max along a dim with first-index ties (the reference sorts instead,
 * python/torch/tensor_ops.py:1531-1537); writes values and int32 indices */
TP_API int tp_max_dim(int64_t id, int dim, int keepdim, tp_handle* values, tp_handle* indices);
/* reductionOps.ts:119-138 argmax over the last dim (argmax.wgsl) */
TP_API int tp_argmax(int64_t id, tp_handle* out);
/* reductionOps.ts:300-328 softmax (softmax.wgsl) */
TP_API int tp_softmax(int64_t id, int dim, tp_handle* out);
/* reductionOps.ts:357-388 logSoftmax (log_softmax.wgsl) */
TP_API int tp_log_softmax(int64_t id, int dim, tp_handle* out);
/* reductionOps.ts:416-443 softmaxBackward (softmax_backward.wgsl) */
TP_API int tp_softmax_backward(int64_t grad_out, int64_t softmax, int64_t batch, int64_t classes, tp_handle* out);
/* reductionOps.ts:390-414 logSoftmaxBackward (log_softmax_backward.wgsl) */
TP_API int tp_log_softmax_backward(int64_t grad_out, int64_t softmax, int64_t batch, int64_t classes,
                                   tp_handle* out);
/* reductionOps.ts:471-489 crossEntropy: per-row loss [B] (cross_entropy.wgsl) */
TP_API int tp_cross_entropy(int64_t input, int64_t targets, tp_handle* out);
/* reductionOps.ts:491-531 crossEntropyBackward: reduction 0 none, 1 sum, 2 mean */
TP_API int tp_cross_entropy_backward(int64_t grad_out, int64_t input, int64_t targets, int reduction,
                                     tp_handle* out);

/* ---- dense contractions (arithmeticOps.ts:260-340, convOps.ts) ---------------- */
/* arithmeticOps.ts:260-308 matmul / mm / bmm / mv shape rules (matmul.wgsl:52-85) */
TP_API int tp_matmul(int64_t a, int64_t b, tp_handle* out);
/* New: y = x . W^T + b (nn.Linear, python/torch/nn/functional.py:95-101 issues a
 * transpose, a matmul, a reshape and a broadcast add); bias id 0 = none */
TP_API int tp_linear(int64_t x, int64_t weight, int64_t bias, tp_handle* out);
/* convOps.ts:17-62 conv2d (conv.wgsl:25-60): bias is a host list of Cout values
 * or NULL; dilation is accepted and ignored, as in the reference */
TP_API int tp_conv2d(int64_t input, int64_t weight, const float* bias, int nbias, const int64_t* stride, int ns,
                     const int64_t* padding, int np, const int64_t* dilation, int nd, int groups, tp_handle* out);
/* New: conv2d with the bias as a tensor id (0 = none) instead of a host list,
 * so a convolution needs no readback of its bias (tensor_nn_ops.py:27 reads
 * it back on every call); same values as tp_conv2d */
TP_API int tp_conv2d_dev_bias(int64_t input, int64_t weight, int64_t bias, const int64_t* stride, int ns,
                              const int64_t* padding, int np, const int64_t* dilation, int nd, int groups,
                              tp_handle* out);
/* convOps.ts:64-108 conv2dInputBackward (conv_backward.wgsl:24-61) */
TP_API int tp_conv2d_input_backward(int64_t grad_out, int64_t weight, const int64_t* input_shape,
                                    const int64_t* grad_out_shape, const int64_t* stride, int ns,
                                    const int64_t* padding, int np, tp_handle* out);
/* convOps.ts:110-155 conv2dWeightBackward (conv_backward.wgsl:66-101) */
TP_API int tp_conv2d_weight_backward(int64_t grad_out, int64_t input, const int64_t* weight_shape,
                                     const int64_t* grad_out_shape, const int64_t* input_shape, const int64_t* stride,
                                     int ns, const int64_t* padding, int np, tp_handle* out);
/* convOps.ts:157-198 conv2dBiasBackward (conv_backward.wgsl:103-119) */
TP_API int tp_conv2d_bias_backward(int64_t grad_out, int64_t out_ch, const int64_t* grad_out_shape, tp_handle* out);

/* contraction engine: 0 = tcgen05 tensor cores with the 3xTF32 split (default
 * where M >= 64), operand tiles brought in by TMA where the operands allow it,
 * on CTA pairs (cta_group::2, 256 x 256 tiles) for large products with N >= 256;
 * 1 = the CUDA-core fp32 kernel everywhere (cross-check); 2 = tensor cores
 * with gathered operand tiles only (no TMA; cross-check of the TMA path);
 * 3 = as 0 with single-CTA TMA tiles only; 4 = as 0 with CTA pairs wherever
 * they fit (N > 32, two row tiles; cross-checks of the pair kernel) */
TP_API int tp_set_gemm_path(int path);
/* 1 (default; environment TP_PDL=0 turns it off at load) = every kernel is
 * launched as a programmatic dependent of the kernel before it on its stream:
 * its CTAs may be scheduled while that kernel's last CTAs drain and wait on the
 * device for its completion before touching memory, which hides launch latency
 * between the many short kernels of a training step.  0 = plain stream order.
 * Results are identical either way.  Applies to launches made (or captured)
 * after the call. */
TP_API int tp_set_pdl(int on);
/* synchronises, then reports the tensor-core kernel's status word: 0 = ok,
 * else the code of a bounded wait that expired; reset != 0 clears it.
 * tp_synchronize and tp_comm_sync read (and clear) the same word and return
 * TP_ERR_TIMEOUT when it is set, so an expired wait reaches every caller that
 * synchronises. */
TP_API int tp_gemm_status(int* out, int reset);
/* Accuracy switch of the tensor-core GEMMs: for K above 4 x kblocks x 32, no
 * split-K split accumulates more than `kblocks` k-blocks of 32 in tensor memory
 * (default 64; 0 = no cap); such reductions are cut into more splits (at most
 * 2048) whose partials are added in fp32 on CUDA cores. */
TP_API int tp_set_gemm_kmax(int kblocks);
/* Tuning switch of the single-CTA TMA GEMM's 128-column tiles: 0 = 4-stage
 * operand ring, one CTA per SM; 1 (default) = a 2-stage ring with two CTAs per
 * SM (one's prologue and epilogue under the other's main loop) when the GEMM
 * has more CTAs (tiles x split-K splits) than SMs; 2 = always two CTAs per SM.
 * Same bits either way. */
TP_API int tp_set_gemm_twocta(int mode);
/* New, for testing the path above: one CTA waits on an mbarrier nothing
 * arrives on, with the tensor-core kernels' own bounded-wait function and a
 * limit of limit_ns (1e3 .. 2e9); the wait runs out, records code 99 in the
 * status word and the kernel returns.  No copy or tensor memory is involved.
 * The next tp_synchronize then returns TP_ERR_TIMEOUT. */
TP_API int tp_wait_probe(int64_t limit_ns);

/* ---- pooling (poolingOps.ts:18-48, max_pool2d.wgsl:22-49) ------------------------ */
TP_API int tp_max_pool2d(int64_t input, const int64_t* kernel, int nk, const int64_t* stride, int ns,
                         const int64_t* padding, int np, const int64_t* dilation, int nd, tp_handle* out);
/* New: also writes the flat ih*W+iw of each window's first maximum (int32) */
TP_API int tp_max_pool2d_with_indices(int64_t input, const int64_t* kernel, int nk, const int64_t* stride, int ns,
                                      const int64_t* padding, int np, const int64_t* dilation, int nd,
                                      tp_handle* out, tp_handle* indices);
/* New: the reference has no max-pool backward (tensor_nn_ops.py:57-72) */
TP_API int tp_max_pool2d_backward(int64_t grad_out, int64_t indices, const int64_t* input_shape,
                                  const int64_t* kernel, int nk, const int64_t* stride, int ns,
                                  const int64_t* padding, int np, const int64_t* dilation, int nd, tp_handle* out);

/* ---- normalisation (normalizationOps.ts, tensor_nn_ops.py) ------------------------ */
/* normalizationOps.ts:20-126 batchNorm (inference, batchnorm.wgsl:20-36); ids of
 * 0 mean "null" (weight 1, bias 0, mean 0, var 1) */
TP_API int tp_batch_norm(int64_t input, int64_t weight, int64_t bias, int64_t running_mean, int64_t running_var,
                         float eps, tp_handle* out);
/* New: training-mode forward of tensor_nn_ops.py:92-254 (three launches, or
 * one for large tensors, tp_set_bn_flow); updates running stats in place,
 * returns y and the saved mean / inv_std; fuse_relu applies ReLU to y */
TP_API int tp_batch_norm_train(int64_t input, int64_t weight, int64_t bias, int64_t running_mean,
                               int64_t running_var, float eps, float momentum, int fuse_relu, tp_handle* out,
                               tp_handle* save_mean, tp_handle* save_invstd);
/* New: backward with PyTorch's rule (the reference's autograd_rules.py:
 * 1049-1130 throws for W != C and scales dweight/dbias by weight); relu_out id
 * != 0 masks grad_out by relu_out > 0 first */
TP_API int tp_batch_norm_backward(int64_t grad_out, int64_t input, int64_t weight, int64_t save_mean,
                                  int64_t save_invstd, int64_t relu_out, tp_handle* dx, tp_handle* dweight,
                                  tp_handle* dbias);
/* New, a tuning switch of the NCHW BatchNorm training kernels (tp_batch_norm_train,
 * tp_batch_norm_backward, tpk_bn_train, tpk_bn_backward): mode 0 = two passes
 * (per-channel sums, then the element-wise pass; a tensor larger than L2 is
 * read twice from HBM); 1 (default) = for tensors of 32 MB or more with
 * H*W % 4 == 0, one launch whose CTAs claim work items in a fixed order --
 * the sums of a channel, then, `lag` channels later, its element-wise pass,
 * which re-reads the channel from L2; 2 = that launch whenever H*W % 4 == 0.
 * lag 0 = automatic; ctas_per_sm 0 = 4; item_values 0 = 16384 values of one
 * channel per work item (rounded down to whole images).  Same formulas either
 * way; the f64 sums are grouped differently, so mean and inv_std may differ in
 * the last bit.  A wait of that launch that expires (2 s) is reported like the
 * tensor-core kernels' (tp_gemm_status, tp_synchronize). */
TP_API int tp_set_bn_flow(int mode, int lag, int ctas_per_sm, int item_values);
/* normalizationOps.ts:128-171 layerNorm (layernorm.wgsl:14-42) over the last
 * normalized_size values; save_mean / save_rstd may be NULL */
TP_API int tp_layer_norm(int64_t input, int64_t normalized_size, int64_t gamma, int64_t beta, float eps,
                         tp_handle* out, tp_handle* save_mean, tp_handle* save_rstd);
/* New: LN backward, PyTorch's rule (autograd_rules.py:1133-1209 scales
 * dgamma/dbeta by gamma) */
TP_API int tp_layer_norm_backward(int64_t grad_out, int64_t input, int64_t normalized_size, int64_t gamma,
                                  int64_t save_mean, int64_t save_rstd, tp_handle* dx, tp_handle* dgamma,
                                  tp_handle* dbeta);

/* ---- optimizer steps (reductionOps.ts:533-653), in place ------------------- */
/* adamw_step.wgsl */
TP_API int tp_adamw_step(int64_t param, int64_t grad, int64_t exp_avg, int64_t exp_avg_sq, float lr, float beta1,
                         float beta2, float eps, float weight_decay, float step_size, float inv_sqrt_bc2);
/* adam_step.wgsl */
TP_API int tp_adam_step(int64_t param, int64_t grad, int64_t exp_avg, int64_t exp_avg_sq, float lr, float beta1,
                        float beta2, float eps, float weight_decay, float step_size, float inv_sqrt_bc2);
/* sgd_step.wgsl */
TP_API int tp_sgd_step(int64_t param, int64_t grad, int64_t momentum_buf, float lr, float momentum,
                       float weight_decay, float dampening, int nesterov);
/* New: one fused launch for a whole parameter group (the per-parameter loops
 * of optim/__init__.py:158-205,238-312,345-418 become one kernel). */
TP_API int tp_adamw_step_multi(const int64_t* params, const int64_t* grads, const int64_t* exp_avgs,
                               const int64_t* exp_avg_sqs, int n, float lr, float beta1, float beta2, float eps,
                               float weight_decay, float step_size, float inv_sqrt_bc2);
TP_API int tp_adam_step_multi(const int64_t* params, const int64_t* grads, const int64_t* exp_avgs,
                              const int64_t* exp_avg_sqs, int n, float lr, float beta1, float beta2, float eps,
                              float weight_decay, float step_size, float inv_sqrt_bc2);
TP_API int tp_sgd_step_multi(const int64_t* params, const int64_t* grads, const int64_t* momentum_bufs, int n,
                             float lr, float momentum, float weight_decay, float dampening, int nesterov);
/* runtime.ts:683-705 rmspropStep (rmsprop_step.wgsl); momentum != 0 uses
 * momentum_buf, as the shader's use_momentum flag (reductionOps.ts:655-688) */
TP_API int tp_rmsprop_step(int64_t param, int64_t grad, int64_t square_avg, int64_t momentum_buf, float lr,
                           float alpha, float eps, float weight_decay, float momentum);
/* runtime.ts:707-716 adagradStep (extended_step.wgsl adagrad_step) */
TP_API int tp_adagrad_step(int64_t param, int64_t grad, int64_t sum_squares, float lr, float eps,
                           float weight_decay);
/* runtime.ts:718-744 adamaxStep (extended_step.wgsl adamax_step) */
TP_API int tp_adamax_step(int64_t param, int64_t grad, int64_t exp_avg, int64_t exp_inf, float lr, float beta1,
                          float beta2, float eps, float weight_decay, float step_size, float bias_correction1);
/* runtime.ts:746-772 nadamStep (extended_step.wgsl nadam_step) */
TP_API int tp_nadam_step(int64_t param, int64_t grad, int64_t exp_avg, int64_t exp_avg_sq, float lr, float beta1,
                         float beta2, float eps, float weight_decay, float step_size, float mu);
/* runtime.ts:774-801 radamStep (extended_step.wgsl radam_step); `step` is the
 * integer step count the shader reads from dims.y (the reference's Python
 * passes it, optim/__init__.py:825-839, but runtime.ts drops it, so the shader
 * sees 0 and uses 1; here the count is used as intended) */
TP_API int tp_radam_step(int64_t param, int64_t grad, int64_t exp_avg, int64_t exp_avg_sq, float lr, float beta1,
                         float beta2, float eps, float weight_decay, float step_size, float beta1_pow_t,
                         float beta2_pow_t, int64_t step);
/* New: the same five as one fused launch per parameter group */
TP_API int tp_rmsprop_step_multi(const int64_t* params, const int64_t* grads, const int64_t* square_avgs,
                                 const int64_t* momentum_bufs, int n, float lr, float alpha, float eps,
                                 float weight_decay, float momentum);
TP_API int tp_adagrad_step_multi(const int64_t* params, const int64_t* grads, const int64_t* sum_squares, int n,
                                 float lr, float eps, float weight_decay);
TP_API int tp_adamax_step_multi(const int64_t* params, const int64_t* grads, const int64_t* exp_avgs,
                                const int64_t* exp_infs, int n, float lr, float beta1, float beta2, float eps,
                                float weight_decay, float step_size, float bias_correction1);
TP_API int tp_nadam_step_multi(const int64_t* params, const int64_t* grads, const int64_t* exp_avgs,
                               const int64_t* exp_avg_sqs, int n, float lr, float beta1, float beta2, float eps,
                               float weight_decay, float step_size, float mu);
TP_API int tp_radam_step_multi(const int64_t* params, const int64_t* grads, const int64_t* exp_avgs,
                               const int64_t* exp_avg_sqs, int n, float lr, float beta1, float beta2, float eps,
                               float weight_decay, float step_size, float beta1_pow_t, float beta2_pow_t,
                               int64_t step);

/* ---- pointer-level optimizer kernels ---------------------------------------- */
/* A tensor group is a device-side table of n (param, grad, state0, state1,
 * numel) rows built once; steps then take only hyper-parameters. */
TP_API int tpk_group_create(int n, float* const* params, float* const* grads, float* const* state0,
                            float* const* state1, const int64_t* numels, int64_t* out_group);
/* The same with lo (NULL, or n pointers, each NULL or 16-byte aligned): the
 * SGD step then writes lo[i] = the tf32 low parts of the updated params[i]
 * (as tpk_tf32_lo), which the conv entries read as w_lo.  No reference
 * counterpart (the reference has no tensor-core split). */
TP_API int tpk_group_create_lo(int n, float* const* params, float* const* grads, float* const* state0,
                               float* const* state1, float* const* lo, const int64_t* numels, int64_t* out_group);
TP_API int tpk_group_destroy(int64_t group);
/* kind 0 AdamW, 1 Adam */
TP_API int tpk_adam_group(int64_t group, int kind, float lr, float beta1, float beta2, float eps,
                          float weight_decay, float step_size, float inv_sqrt_bc2);
/* grad_scale multiplies each gradient on read (1/world for averaged DP grads);
 * rows created with a lo pointer (tpk_group_create_lo) also get the tf32 low
 * parts of their updated parameter there */
TP_API int tpk_sgd_group(int64_t group, float lr, float momentum, float weight_decay, float dampening,
                         int nesterov, float grad_scale);

/* ---- pointer-level kernels for a step driver (no allocation) ----------------- */
/* conv2d forward / data-gradient / weight-gradient on NCHW device buffers
 * (the kernels behind tp_conv2d, tp_conv2d_input_backward and
 * tp_conv2d_weight_backward; groups = 1) */
TP_API int tpk_conv2d_fwd(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t Cin,
                          int64_t H, int64_t W, int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW);
TP_API int tpk_conv2d_dgrad(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H, int64_t W,
                            int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW);
TP_API int tpk_conv2d_wgrad(const float* dy, const float* x, float* dw, int64_t N, int64_t Cin, int64_t H, int64_t W,
                            int64_t Cout, int KH, int KW, int SH, int SW, int PH, int PW);
/* The same three on channels-last buffers: x [N][H][W][Cin], y / dy
 * [N][OH][OW][Cout], stride 1, dilation 1, groups 1, OH = H + 2PH - KH + 1.
 * filter_layout 0: w and dw in the reference layout [Cout][Cin][KH][KW];
 * 1: [Cout][KH][KW][Cin], which the forward uses as it is, the data gradient
 * reads in place and the weight gradient writes with contiguous stores.  No
 * reference counterpart: the reference's shaders are NCHW only (conv.wgsl:25-60,
 * conv_backward.wgsl:24-101); these serve a training step that keeps its
 * activations channels-last (tpcuda.vgg). */
TP_API int tpk_conv2d_fwd_nhwc(const float* x, const float* w, const float* bias, float* y, int64_t N, int64_t Cin,
                               int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH, int PW, int filter_layout);
TP_API int tpk_conv2d_dgrad_nhwc(const float* dy, const float* w, float* dx, int64_t N, int64_t Cin, int64_t H,
                                 int64_t W, int64_t Cout, int KH, int KW, int PH, int PW, int filter_layout);
TP_API int tpk_conv2d_wgrad_nhwc(const float* dy, const float* x, float* dw, int64_t N, int64_t Cin, int64_t H,
                                 int64_t W, int64_t Cout, int KH, int KW, int PH, int PW, int filter_layout);
/* The same forward and data gradient with the filters' tf32 low parts w_lo
 * (tpk_tf32_lo of w; NULL: computed per call) kept by the caller beside w --
 * a step driver whose optimizer writes them (tpk_group_create_lo) saves
 * the per-call split.  Used with filter_layout 1 (filters read in place). */
TP_API int tpk_conv2d_fwd_nhwc_lo(const float* x, const float* w, const float* w_lo, const float* bias, float* y,
                                  int64_t N, int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH,
                                  int PW, int filter_layout);
TP_API int tpk_conv2d_dgrad_nhwc_lo(const float* dy, const float* w, const float* w_lo, float* dx, int64_t N,
                                    int64_t Cin, int64_t H, int64_t W, int64_t Cout, int KH, int KW, int PH, int PW,
                                    int filter_layout);
/* lo[i] = x[i] - (x[i] with its 13 low mantissa bits cleared): the low part
 * of the 3xTF32 split (x and lo 16-byte aligned) */
TP_API int tpk_tf32_lo(const float* x, float* lo, int64_t n);
/* Channels-last ([P][C], P = pixels) companions of tpk_bn_train,
 * tpk_bn_backward, tpk_channel_sum and tpk_maxpool_fwd / _bwd (2x2, stride
 * 2), for the same step; C % 4 == 0 and 16-byte aligned buffers.  Pool
 * indices are plane offsets h*W + w as in the NCHW kernels.  No reference
 * counterpart (NCHW only: batchnorm / max_pool2d shaders,
 * tensor_nn_ops.py:57-254). */
TP_API int tpk_bn_train_nhwc(const float* x, const float* w, const float* b, float* running_mean,
                             float* running_var, float* y, float* save_mean, float* save_invstd, int64_t P, int64_t C,
                             float eps, float momentum, int relu);
/* dx_sum (optional): the per-channel sum of dx, which is the gradient of a
 * bias added just before the BatchNorm (the conv bias), from the same pass */
TP_API int tpk_bn_backward_nhwc(const float* dy, const float* x, const float* relu_src, const float* w,
                                const float* mean, const float* invstd, float* dx, float* dw, float* db,
                                float* dx_sum, int64_t P, int64_t C);
/* BatchNorm train forward (+ReLU when relu) fused with the 2x2 / stride-2
 * max-pool after it: x [N][H][W][C] -> pooled y [N][H/2][W/2][C] and idx (plane
 * offsets h*W + w of each window's maximum, as tpk_maxpool2x2_nhwc_fwd); the
 * full-size activation a is written only when a is not NULL.  Same values as
 * tpk_bn_train_nhwc followed by tpk_maxpool2x2_nhwc_fwd. */
TP_API int tpk_bn_train_pool_nhwc(const float* x, const float* w, const float* b, float* running_mean,
                                  float* running_var, float* y, int32_t* idx, float* a, float* save_mean,
                                  float* save_invstd, int64_t N, int64_t H, int64_t W, int64_t C, float eps,
                                  float momentum, int relu);
/* BatchNorm backward whose ReLU mask (relu != 0) is recomputed from x with
 * the forward's formula (gamma w, beta b), so no activation is read.  idx NULL:
 * g is the gradient at the BN(+ReLU) output, [N][H][W][C].  idx given: g is the
 * gradient of the 2x2 / stride-2 max-pool that followed, [N][H/2][W/2][C], with
 * that pool's idx, and is routed to each window's argmax in place (the same
 * values as tpk_maxpool2x2_nhwc_bwd, then tpk_bn_backward_nhwc). */
TP_API int tpk_bn_backward_fused_nhwc(const float* g, const int32_t* idx, const float* x, const float* w,
                                      const float* b, const float* mean, const float* invstd, float* dx, float* dw,
                                      float* db, float* dx_sum, int64_t N, int64_t H, int64_t W, int64_t C,
                                      int relu);
TP_API int tpk_channel_sum_nhwc(const float* x, int64_t P, int64_t C, float* out);
TP_API int tpk_maxpool2x2_nhwc_fwd(const float* x, float* y, int32_t* idx, int64_t N, int64_t H, int64_t W,
                                   int64_t C);
TP_API int tpk_maxpool2x2_nhwc_bwd(const float* dy, const int32_t* idx, float* dx, int64_t N, int64_t H, int64_t W,
                                   int64_t C);
/* NCHW [N][C][H][W] -> channels-last [N][H][W][Cpad], channels >= C zero */
TP_API int tpk_nchw_to_nhwc(const float* x, float* y, int64_t N, int64_t C, int64_t H, int64_t W, int64_t Cpad);
/* per-channel sum over N and the spatial dims (the conv bias gradient) */
TP_API int tpk_channel_sum(const float* x, int64_t N, int64_t C, int64_t P, float* out);
/* the kernels behind tp_batch_norm_train / tp_batch_norm_backward */
TP_API int tpk_bn_train(const float* x, const float* w, const float* b, float* running_mean, float* running_var,
                        float* y, float* save_mean, float* save_invstd, int64_t N, int64_t C, int64_t S, float eps,
                        float momentum, int relu);
TP_API int tpk_bn_backward(const float* dy, const float* x, const float* relu_src, const float* w, const float* mean,
                           const float* invstd, float* dx, float* dw, float* db, int64_t N, int64_t C, int64_t S);
/* square-window max-pool with int32 indices, and its backward */
TP_API int tpk_maxpool_fwd(const float* x, float* y, int32_t* idx, int64_t N, int64_t C, int64_t H, int64_t W, int k,
                           int s, int p);
TP_API int tpk_maxpool_bwd(const float* dy, const int32_t* idx, float* dx, int64_t N, int64_t C, int64_t H, int64_t W,
                           int k, int s, int p);
/* C[M,N] = op(A) op(B) (+ bias[N]); a_t: A stored [K,M]; b_t: B stored [N,K] */
TP_API int tpk_gemm(const float* A, int a_t, const float* B, int b_t, float* C, int64_t M, int64_t N, int64_t K,
                    const float* bias);
/* cross-entropy per row and its mean, both left in HBM (the reference reads
 * the mean back to the host, reductionOps.ts:203-212) */
TP_API int tpk_cross_entropy_mean(const float* logits, const float* targets, float* loss_rows, float* loss_mean,
                                  int64_t B, int64_t C);
/* No counterpart in the reference.  The same mean cross-entropy as
 * tpk_cross_entropy_mean for callers that cannot allocate device memory (a
 * process whose HBM budget is fixed at start-up, a latency-critical loop): the
 * caller passes only inputs and the one-float output; the per-row losses and
 * reduction partials live in a fixed device array reserved when the library
 * loads (about 1 MB per GPU, kept until exit), so B <= 262144 rows, larger B is
 * rejected with TP_ERR_ARG; B = 0 writes 0, as tpk_cross_entropy_mean does.
 * The first call on a device looks up that array's address (guarded, so
 * concurrent first calls are safe); make it before any stream capture.  Calls
 * share the array: calls that overlap on the GPU race. */
TP_API int tpk_cross_entropy_mean_noalloc(const float* logits, const float* targets, float* loss_mean, int64_t B,
                                          int64_t C);
/* New: a classifier head's forward and backward in one launch.  x [B][F],
 * w [K][F], b [K] (NULL: none), targets [B] (class indices as floats, clamped
 * as cross_entropy.wgsl does); writes logits [B][K] = x w^T + b, loss_rows [B],
 * loss_mean [1], and with g = (softmax(logits) - onehot(target)) * scale
 * (scale 1/B for the mean loss): dx [B][F] = g w, dw [K][F] = g^T x,
 * db [K] = sum_rows g.  Any output may be NULL.  Replaces tpk_gemm +
 * tpk_cross_entropy_mean + tpk_cross_entropy_backward + two tpk_gemm +
 * tpk_channel_sum of the per-op path (the linear layer of
 * python/torch/nn/modules.py with the loss of reductionOps.ts:471-531).
 * K <= 32, F <= 1024; every sum runs in a fixed order (deterministic).  Uses
 * one device-wide ticket word: calls must not overlap on the GPU. */
TP_API int tpk_linear_cross_entropy_step(const float* x, const float* w, const float* b, const float* targets,
                                         float* logits, float* loss_rows, float* loss_mean, float* dx, float* dw,
                                         float* db, int64_t B, int64_t F, int64_t K, float scale);
/* grad = (softmax(logits) - onehot(target)) * scale (cross_entropy_backward.wgsl) */
TP_API int tpk_cross_entropy_backward(const float* logits, const float* targets, float* grad, int64_t B, int64_t C,
                                      float scale);
TP_API int tpk_fill(float* x, int64_t n, float value);

/* ---- data-parallel gradient exchange (new: the reference has no parallelism) ---- */
/* NCCL unique id of rank 0 (128 bytes) to hand to every rank */
TP_API int tp_comm_unique_id(char* out, int len);
/* New: before tp_comm_init, 1 (the default) creates the communicator's stream
 * at the device's highest stream priority (its all-reduces then start ahead of
 * pending compute CTAs); 0 at the normal priority. */
TP_API int tp_set_comm_priority(int high);
TP_API int tp_comm_init(int rank, int world, const char* unique_id, int len);
/* in-place sum over ranks, queued after the work already on the library stream,
 * run on the communication stream */
TP_API int tp_comm_allreduce_async(float* ptr, int64_t count);
/* the library stream waits for every all-reduce issued so far */
TP_API int tp_comm_wait(void);
/* host wait for the library stream with a communicator watchdog: on an NCCL
 * error or after timeout_ms the communicator is aborted and an error returned */
TP_API int tp_comm_sync(int timeout_ms);
TP_API int tp_comm_destroy(void);
TP_API int tp_comm_info(int* rank, int* world);

/* ---- CUDA graphs of the library stream ------------------------------------------ */
/* capture every launch made between begin and end into one graph; call the
 * same sequence once before capturing so scratch buffers have their size */
TP_API int tp_graph_begin(void);
TP_API int tp_graph_end(int64_t* out_graph);
TP_API int tp_graph_launch(int64_t graph);
TP_API int tp_graph_destroy(int64_t graph);

#ifdef __cplusplus
}
#endif
#endif /* TPCUDA_H */
