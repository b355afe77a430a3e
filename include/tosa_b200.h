/*
 * tosa_b200 -- B200 (sm_100a) execution backend for the dense-contraction path
 * of the tosa-interp TOSA interpreter: CONV2D, DEPTHWISE_CONV2D and MATMUL
 * (and MATMUL_T, TRANSPOSE_CONV2D, CONV3D) with their zero points, bias and
 * acc_type, fused with the RESCALE (and
 * CLAMP) that follows them, plus AVG_POOL2D / MAX_POOL2D and the glue ops the
 * quantized graphs need (standalone RESCALE, CLAMP, ADD).
 *
 * C ABI: plain pointers and sizes, no C++ types, no exceptions across the
 * boundary. Every entry point returns a tb_status; on failure the thread's
 * last error message (tb_last_error) says why.
 *
 * Memory: tensor data passed to the operator entry points are DEVICE pointers
 * on the context's device (allocate with tb_malloc or any CUDA allocator on
 * the same device). Small attribute arrays (RESCALE multiplier/shift) are HOST
 * pointers, as they are CONST tensors of the graph. `stream` is a
 * cudaStream_t (NULL = the legacy default stream); launches are asynchronous
 * and data-dependent errors (the reference's RESCALE/apply_scale range
 * errors) are reported by the next tb_synchronize on that context.
 *
 * Reference interfaces replaced (tosa-interp, path:line):
 *   operator dispatch          src/ops/mod.rs:22-150 (dispatch)
 *   CONV2D                     src/ops/conv.rs:502-508 (eval_conv2d), :398-500
 *   CONV3D                     src/ops/conv.rs:510-516 (eval_conv3d), :107-181
 *   DEPTHWISE_CONV2D           src/ops/conv.rs:518-524
 *   TRANSPOSE_CONV2D           src/ops/conv.rs:526-532 (eval_transpose_conv2d), :286-371
 *   MATMUL                     src/ops/matmul.rs:176-178 (eval_matmul), :98-174
 *   MATMUL_T                   src/ops/matmul.rs:180-182 (eval_matmul_t), :98-174
 *   RESCALE                    src/ops/type_conv.rs:111-191 (eval_rescale)
 *   CLAMP                      src/ops/elementwise.rs:319-343 (eval_clamp)
 *   ADD                        src/ops/elementwise.rs:395-397 (eval_add)
 *   AVG_POOL2D / MAX_POOL2D    src/ops/pool.rs:146-151, :233-238
 *   run_graph*                 src/lib.rs:20-43; Interpreter::run src/interpreter.rs:122-147
 *   InterpreterHook / HookSet  src/stats.rs:11-75
 *   Error                      src/error.rs:4-31
 */
#ifndef TOSA_B200_H
#define TOSA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TB_API __attribute__((visibility("default")))
#else
#define TB_API
#endif

/* Status codes. 1..9 map one-to-one onto the reference's Error variants
 * (src/error.rs:4-31); 64.. are backend conditions. */
typedef enum tb_status {
    TB_OK = 0,
    TB_ERR_DESERIALIZE = 1,      /* Error::Deserialize */
    TB_ERR_UNSUPPORTED_OP = 2,   /* Error::UnsupportedOp */
    TB_ERR_TENSOR_NOT_FOUND = 3, /* Error::TensorNotFound */
    TB_ERR_DTYPE_MISMATCH = 4,   /* Error::DTypeMismatch */
    TB_ERR_SHAPE_MISMATCH = 5,   /* Error::ShapeMismatch */
    TB_ERR_BROADCAST = 6,        /* Error::Broadcast */
    TB_ERR_GRAPH = 7,            /* Error::GraphError (ERROR_IF, apply_scale range) */
    TB_ERR_CONTROL_FLOW = 8,     /* Error::ControlFlow */
    TB_ERR_IO = 9,               /* Error::Io */
    TB_ERR_CUDA = 64,            /* a CUDA call failed */
    TB_ERR_TIMEOUT = 65,         /* a bounded device wait gave up */
    TB_ERR_INVALID_ARGUMENT = 66,/* null pointer, bad handle */
    TB_ERR_NOT_ACCELERATED = 67  /* valid TOSA this backend does not run (caller keeps its own path) */
} tb_status;

/* DType codes: the serialized TOSA DType enum (schema/tosa.fbs:26-46). */
enum {
    TB_DT_BOOL = 1, TB_DT_INT4 = 2, TB_DT_INT8 = 3, TB_DT_INT16 = 4, TB_DT_INT32 = 5,
    TB_DT_INT48 = 6, TB_DT_FP32 = 7, TB_DT_FP16 = 8, TB_DT_BF16 = 9, TB_DT_SHAPE = 10,
    TB_DT_FP8E4M3 = 11, TB_DT_FP8E5M2 = 12, TB_DT_INT64 = 17
};
/* RescaleAttribute.rounding_mode (schema/tosa.fbs:60-65). */
enum { TB_ROUND_SINGLE = 1, TB_ROUND_INEXACT = 2, TB_ROUND_DOUBLE = 3 };
/* NanPropagationMode (schema/tosa.fbs:54-58). */
enum { TB_NAN_PROPAGATE = 1, TB_NAN_IGNORE = 2 };

typedef struct tb_context tb_context;

/* ---- context, memory, errors ------------------------------------------- */

/* One context per CUDA device; not shared between threads. */
TB_API tb_status tb_context_create(int device, tb_context **out);
TB_API void tb_context_destroy(tb_context *ctx);
/* Message of the last failure on the calling thread ("" if none). */
TB_API const char *tb_last_error(void);
/* Wait for `stream`, then read and clear the context's device error word;
 * returns TB_ERR_GRAPH if a kernel hit a RESCALE/apply_scale range error
 * (src/ops/quant.rs:18-25, src/ops/type_conv.rs:183-186), TB_ERR_TIMEOUT if a
 * bounded wait gave up. */
TB_API tb_status tb_synchronize(tb_context *ctx, void *stream);
TB_API tb_status tb_malloc(tb_context *ctx, size_t bytes, void **dptr);
TB_API tb_status tb_free(tb_context *ctx, void *dptr);
TB_API tb_status tb_memcpy_h2d(tb_context *ctx, void *dst, const void *src, size_t bytes, void *stream);
TB_API tb_status tb_memcpy_d2h(tb_context *ctx, void *dst, const void *src, size_t bytes, void *stream);
/* Bound on every in-kernel wait of later launches on this context, in
 * milliseconds (default 2000, or TB_WAIT_TIMEOUT_MS at context creation). A
 * wait that gives up makes its kernel unwind (its own copies and MMAs drain
 * under a separate bound of about a second, tensor memory is released) and
 * the next tb_synchronize return TB_ERR_TIMEOUT; the context stays usable. */
TB_API tb_status tb_context_set_wait_timeout_ms(tb_context *ctx, double ms);
/* Number of kernels this context launched so far (for launch accounting). */
TB_API uint64_t tb_launch_count(tb_context *ctx);
/* Diagnostics: in a library built with -DTB_GEMM_TRACE=1 and with TB_TRACE=1
 * in the environment at context creation, the tensor-core kernels record
 * clock64 stamps of CTA 0 (producer stage issues, MMA stage starts, row-sum
 * stage ends, epilogue tile start/end); copies the 512-entry buffer to
 * host512. Regular builds carry no stamp code and return
 * TB_ERR_INVALID_ARGUMENT. */
TB_API tb_status tb_debug_trace(tb_context *ctx, long long *host512);

/* ---- fused RESCALE epilogue ---------------------------------------------- */

/* The RESCALE that follows a contraction (src/ops/type_conv.rs:111-191), and
 * optionally the CLAMP after it (src/ops/elementwise.rs:319-343). The RESCALE
 * input is the contraction's int32 result, so input_zp must be 0 and
 * input_unsigned false, as the reference requires for INT32 input. */
typedef struct tb_rescale_attr {
    int32_t scale32;          /* RescaleAttribute.scale32 */
    int32_t rounding_mode;    /* TB_ROUND_* */
    int32_t per_channel;      /* multiplier/shift have `channels` entries */
    int32_t input_unsigned;
    int32_t output_unsigned;
    int32_t input_zp;         /* raw value of the input_zp operand */
    int32_t output_zp;        /* raw value of the output_zp operand */
    int32_t out_dtype;        /* TB_DT_INT8 / INT16 / INT32 */
    int32_t channels;         /* 1, or the last dimension when per_channel */
    const int32_t *multiplier;/* HOST, `channels` values (int16 values widened when !scale32) */
    const int8_t *shift;      /* HOST, `channels` values */
    int32_t clamp_enabled;    /* fuse a following CLAMP of the RESCALE output */
    int32_t clamp_min, clamp_max;
} tb_rescale_attr;

/* ---- MATMUL (src/ops/matmul.rs:98-174) -------------------------------------
 * a [n,h,c], b [n,c,w] -> out [n,h,w]. Integer: INT8 x INT8 -> INT32 with
 * zero points; float: BF16 x BF16 -> FP32 and FP16 x FP16 -> FP32 (fp32
 * accumulation, results within the stated tolerance of the reference). With a
 * rescale attribute the INT32 result is rescaled in the same kernel and `out`
 * has rescale->out_dtype. */
typedef struct tb_matmul_desc {
    int32_t n, h, c, w;
    int32_t a_dtype, b_dtype, out_dtype;
    int32_t a_zp, b_zp;
} tb_matmul_desc;

typedef struct tb_matmul_plan tb_matmul_plan;
TB_API tb_status tb_matmul_plan_create(tb_context *ctx, const tb_matmul_desc *desc, const tb_rescale_attr *rescale,
                                       tb_matmul_plan **out);
TB_API tb_status tb_matmul_plan_run(tb_matmul_plan *plan, const void *a, const void *b, void *out, void *stream);
/* Declares `b` (device) constant for this plan, as a MATMUL whose B operand is a
 * CONST tensor of the graph: its column sums (the a_zp term) and, when its rows
 * need it, its 16-byte-padded copy are computed now, once; later runs with this
 * same pointer reuse them (a run with another B discards them). The data must
 * not change while the plan is used with it. Returns after the work on `stream`
 * finished. No-op for plans that keep nothing per B (float, direct and
 * zero-a_zp unpadded paths). */
TB_API tb_status tb_matmul_plan_set_constant_b(tb_matmul_plan *plan, const void *b, void *stream);
TB_API void tb_matmul_plan_destroy(tb_matmul_plan *plan);
TB_API tb_status tb_matmul(tb_context *ctx, const tb_matmul_desc *desc, const tb_rescale_attr *rescale,
                           const void *a, const void *b, void *out, void *stream);

/* ---- MATMUL_T (src/ops/matmul.rs:180-182 eval_matmul_t, :98-174) ----------
 * a [n,h,c], b [b_batch,w,c] with b_batch == n or 1 (one B for every batch of
 * a) -> out [n,h,w]; desc fields mean what they mean for MATMUL. Types are
 * matmul_t_types (matmul.rs:42-51): INT8 x INT8 -> INT32 (zero points, and an
 * optional fused rescale, as MATMUL), INT16 x INT16 -> INT48, FP16 x FP16 ->
 * FP16, and any pair of FP8/FP16/BF16/FP32 into FP32, or into BF16 without
 * FP32 operands and not FP16 x FP16. INT8 with c % 16 == 0 and BF16 x BF16 /
 * FP16 x FP16 -> FP32 with c % 8 == 0 run on the tensor cores (B K-major);
 * the rest on the direct kernels in the reference's order. The plan runs,
 * declares a constant B and is destroyed with the tb_matmul_plan_* calls. */
TB_API tb_status tb_matmul_t_plan_create(tb_context *ctx, const tb_matmul_desc *desc, int32_t b_batch,
                                         const tb_rescale_attr *rescale, tb_matmul_plan **out);
TB_API tb_status tb_matmul_t(tb_context *ctx, const tb_matmul_desc *desc, int32_t b_batch,
                             const tb_rescale_attr *rescale, const void *a, const void *b, void *out, void *stream);

/* INT8 x INT8 -> INT32 MATMUL (+ optional fused RESCALE) that allocates no
 * device memory. This entry point has no counterpart in the reference; it is
 * for callers that cannot call cudaMalloc (their device memory belongs to
 * another allocator, or allocation is not allowed where they run). The
 * caller passes device inputs and outputs; the kernel's scratch lives in a
 * fixed 2 MiB file-scope device array that every GPU using the library holds
 * until exit, which limits n*w to 131072 when a_zp != 0 and the rescale to
 * 16384 channels (larger shapes are rejected with TB_ERR_INVALID_ARGUMENT).
 * B rows that are not 16-byte multiples (w % 16 != 0, e.g. 1000 classes) and
 * operands that are not 16-byte aligned run the direct CUDA-core kernel, which
 * needs no scratch (the tensor-core path would pad B into a buffer of its own).
 * Runs on the calling thread's current device; its first call on a device
 * resolves the array's device address (cudaGetSymbolAddress) and keeps it, so
 * make that first call before any stream capture, and do not reset the
 * device's primary context (cudaDeviceReset) while the process still calls
 * this entry point. Every call clears the scratch it
 * needs, then waits for `stream` and returns data-dependent errors itself.
 * Calls that overlap on the GPU share the array and race: serialise them. */
TB_API tb_status tb_matmul_i8_noalloc(const tb_matmul_desc *desc, const tb_rescale_attr *rescale, const void *a,
                                      const void *b, void *out, void *stream);

/* ---- CONV2D / DEPTHWISE_CONV2D (src/ops/conv.rs:398-524) -------------------
 * input NHWC [n,ih,iw,ic]; CONV2D weight OHWI [oc,kh,kw,ic]; DEPTHWISE weight
 * [kh,kw,ic,m] with oc = ic*m; bias [bias_len] (1 or oc) of out_dtype;
 * pad = [top, bottom, left, right]. Integer: INT8 x INT8|INT4 (INT4 held one
 * value per byte) -> INT32 with zero points; float: BF16 x BF16 and
 * FP16 x FP16 with acc_type FP32 -> out_dtype (BF16/FP16/FP32 per the
 * reference's type tables). The weight and bias pointers are read when the
 * plan is created (per-channel sums; TRANSPOSE_CONV2D's tap-reversed copy) and
 * again at every run. Plan creation reads them on the legacy default stream
 * and waits for that work, so weights written on another stream (in
 * particular a non-blocking one) must be complete before the plan is created. */
typedef struct tb_conv2d_desc {
    int32_t n, ih, iw, ic;
    int32_t oc, kh, kw;       /* CONV2D; for DEPTHWISE oc = ic * m */
    int32_t m;                /* DEPTHWISE channel multiplier (ignored by CONV2D) */
    int32_t pad[4], stride[2], dilation[2];
    int32_t in_dtype, w_dtype, acc_dtype, out_dtype;
    int32_t input_zp, weight_zp;
    int32_t bias_len;
} tb_conv2d_desc;

typedef struct tb_conv2d_plan tb_conv2d_plan;
TB_API tb_status tb_conv2d_plan_create(tb_context *ctx, const tb_conv2d_desc *desc, const void *weight,
                                       const void *bias, const tb_rescale_attr *rescale, tb_conv2d_plan **out);
TB_API tb_status tb_depthwise_conv2d_plan_create(tb_context *ctx, const tb_conv2d_desc *desc, const void *weight,
                                                 const void *bias, const tb_rescale_attr *rescale,
                                                 tb_conv2d_plan **out);
TB_API tb_status tb_conv2d_plan_run(tb_conv2d_plan *plan, const void *input, void *out, void *stream);
TB_API void tb_conv2d_plan_destroy(tb_conv2d_plan *plan);
TB_API tb_status tb_conv2d(tb_context *ctx, const tb_conv2d_desc *desc, const tb_rescale_attr *rescale,
                           const void *input, const void *weight, const void *bias, void *out, void *stream);
TB_API tb_status tb_depthwise_conv2d(tb_context *ctx, const tb_conv2d_desc *desc, const tb_rescale_attr *rescale,
                                     const void *input, const void *weight, const void *bias, void *out,
                                     void *stream);

/* ---- CONV3D (src/ops/conv.rs:510-516, ConvNd :107-181 with three dims) ------
 * input NDHWC [n,id,ih,iw,ic]; weight [oc,kd,kh,kw,ic]; bias [bias_len] (1 or
 * oc) of out_dtype; pad = [front, back, top, bottom, left, right]; stride and
 * dilation [d, h, w]. Types: standard_types (conv.rs:388-396), zero points as
 * CONV2D, optional fused rescale for INT8. INT8 with kd == 1, no depth
 * padding and depth stride 1 runs as one CONV2D over n*id images (tensor
 * cores where its layout allows); the rest runs the direct kernel in the
 * reference's order (taps kd, kh, kw row-major, ic innermost). The plan shares
 * tb_conv2d_plan_run / tb_conv2d_plan_destroy with the 2-D convolutions. */
typedef struct tb_conv3d_desc {
    int32_t n, id, ih, iw, ic;
    int32_t oc, kd, kh, kw;
    int32_t pad[6], stride[3], dilation[3];
    int32_t in_dtype, w_dtype, acc_dtype, out_dtype;
    int32_t input_zp, weight_zp;
    int32_t bias_len;
} tb_conv3d_desc;
TB_API tb_status tb_conv3d_plan_create(tb_context *ctx, const tb_conv3d_desc *desc, const void *weight,
                                       const void *bias, const tb_rescale_attr *rescale, tb_conv2d_plan **out);
TB_API tb_status tb_conv3d(tb_context *ctx, const tb_conv3d_desc *desc, const tb_rescale_attr *rescale,
                           const void *input, const void *weight, const void *bias, void *out, void *stream);

/* ---- TRANSPOSE_CONV2D (src/ops/conv.rs:526-532, Transpose :286-371) --------
 * The tb_conv2d_desc fields keep their CONV2D meaning (weight OHWI [oc,kh,kw,ic],
 * the types of standard_types conv.rs:388-396) except that pad = out_pad
 * [top, bottom, left, right], each > -kernel size (may be negative), and
 * dilation is ignored; output [n, (ih-1)*stride_y + pad[0] + pad[1] + kh,
 * (iw-1)*stride_x + pad[2] + pad[3] + kw, oc]. INT8 with stride 1 runs as the
 * CONV2D with reversed taps on the tensor cores (exact: integer sums); every
 * other case runs the direct gather kernel in the reference's order. Runs and
 * is destroyed with tb_conv2d_plan_run / tb_conv2d_plan_destroy. */
TB_API tb_status tb_transpose_conv2d_plan_create(tb_context *ctx, const tb_conv2d_desc *desc, const void *weight,
                                                 const void *bias, const tb_rescale_attr *rescale,
                                                 tb_conv2d_plan **out);
TB_API tb_status tb_transpose_conv2d(tb_context *ctx, const tb_conv2d_desc *desc, const tb_rescale_attr *rescale,
                                     const void *input, const void *weight, const void *bias, void *out,
                                     void *stream);

/* ---- standalone elementwise ops ----------------------------------------- */

/* RESCALE of `count` elements of in_dtype (INT8/INT16/INT32), channel of
 * element i = i % channels when per_channel (src/ops/type_conv.rs:111-191). */
TB_API tb_status tb_rescale(tb_context *ctx, const tb_rescale_attr *attr, int32_t in_dtype, const void *input,
                            int64_t count, void *out, void *stream);
/* CLAMP (src/ops/elementwise.rs:319-343): INT8/INT16 with integer bounds, or
 * FP16/BF16/FP32 with float bounds and a NaN mode. */
TB_API tb_status tb_clamp(tb_context *ctx, int32_t dtype, const void *input, int64_t count, int64_t min_i,
                          int64_t max_i, float min_f, float max_f, int32_t nan_mode, void *out, void *stream);
/* ADD of two equal-shape tensors (INT32 wraps; FP32 rounds), src/ops/elementwise.rs:395-397. */
TB_API tb_status tb_add(tb_context *ctx, int32_t dtype, const void *a, const void *b, int64_t count, void *out,
                        void *stream);

/* ---- pooling (src/ops/pool.rs:146-286) ----------------------------------- */
typedef struct tb_pool2d_desc {
    int32_t n, ih, iw, c;
    int32_t kernel[2], stride[2], pad[4];
    int32_t dtype;            /* INT8 / INT16 / FP16 / BF16 / FP32 */
    int32_t acc_dtype;        /* AVG_POOL2D: INT32 for integers, FP32 for floats */
    int32_t input_zp, output_zp; /* AVG_POOL2D, INT8 only */
    int32_t nan_mode;         /* MAX_POOL2D */
} tb_pool2d_desc;
TB_API tb_status tb_avg_pool2d(tb_context *ctx, const tb_pool2d_desc *desc, const void *input, void *out,
                               void *stream);
TB_API tb_status tb_max_pool2d(tb_context *ctx, const tb_pool2d_desc *desc, const void *input, void *out,
                               void *stream);

/* ---- graph runner ----------------------------------------------------------
 * Runs a serialized TOSA graph (.tosa flatbuffer) on the device: the
 * counterpart of Interpreter::from_flatbuffer + Interpreter::run
 * (src/interpreter.rs:108-147, :154-253) and run_graph / run_graph_with_hooks
 * (src/lib.rs:20-43). Operators execute in the reference's ready-queue order
 * and every operator emits the reference's hook events (pre_op, then
 * on_tensor_alloc for each output, then post_op; src/interpreter.rs:199-216),
 * fused or not. The runner accepts CONST, CONST_SHAPE, IDENTITY, RESHAPE,
 * TRANSPOSE, CONV2D, DEPTHWISE_CONV2D, MATMUL, RESCALE, CLAMP, ADD,
 * AVG_POOL2D and MAX_POOL2D; a graph with any other operator is rejected
 * with TB_ERR_UNSUPPORTED_OP at tb_graph_load (those graphs stay on the
 * reference path).
 *
 * Fusion (off with TB_GRAPH_NO_FUSION): a contraction whose only consumer is
 * a RESCALE (and that RESCALE's only consumer a CLAMP) runs as one kernel, and
 * the residual chain RESCALE, RESCALE -> ADD -> RESCALE [-> CLAMP] runs as one
 * elementwise pass. Intermediate tensors of a fused group are not
 * materialised: their tb_tensor_info.data is NULL in hook callbacks.
 *
 * Tensor data in host and device buffers use one element per slot: INT8/BOOL
 * 1 byte, INT4 1 byte per element (sign-extended, as the contraction entry
 * points take INT4 weights), INT16/FP16/BF16 2, INT32/FP32 4, INT48/INT64/SHAPE
 * 8 bytes, little-endian. TB_GRAPH_CUDA_GRAPH needs a non-default stream. */
typedef struct tb_graph tb_graph;

typedef struct tb_tensor_info {   /* a tensor as hooks see it (src/tensor.rs:228-249) */
    const char *name;
    int32_t dtype;                /* TB_DT_* (SHAPE values report TB_DT_INT64, like the reference) */
    int32_t rank;
    const int64_t *shape;
    uint64_t bytes;               /* element_count (>= 1) * element size */
    const void *data;             /* device pointer, NULL when fused away */
} tb_tensor_info;

typedef struct tb_op_info {       /* OpInfo (src/stats.rs:6-9) */
    int32_t op;                   /* serialized Op code (schema/tosa.fbs:88-201) */
    int32_t op_index;             /* index in the block's operator list */
} tb_op_info;

/* InterpreterHook (src/stats.rs:11-16); NULL members do nothing. Called on the
 * thread that runs the graph. */
typedef struct tb_hooks {
    void *user;
    void (*pre_op)(void *user, const tb_op_info *op, const tb_tensor_info *inputs, int32_t n_inputs);
    void (*post_op)(void *user, const tb_op_info *op, const tb_tensor_info *inputs, int32_t n_inputs,
                    const tb_tensor_info *outputs, int32_t n_outputs);
    void (*on_tensor_alloc)(void *user, const char *name, const int64_t *shape, int32_t rank, int32_t dtype,
                            uint64_t bytes);
    void (*on_tensor_free)(void *user, const char *name, uint64_t bytes);
} tb_hooks;

enum {
    TB_GRAPH_NO_FUSION = 1,   /* run every operator as its own kernel (every tensor materialised) */
    TB_GRAPH_SYNC_EACH_OP = 2,/* synchronize the stream before each post_op (wall-clock timing hooks) */
    TB_GRAPH_CUDA_GRAPH = 4,  /* capture the launches into a CUDA graph on the first run, replay it after */
    TB_GRAPH_TIME_OPS = 8     /* CUDA-event device time of each operator's kernels (eager runs only) */
};

/* Parse `data` (Graph::from_flatbuffer, src/ir.rs:592-614) and check that
 * every operator is one the runner executes. Plans, constants and device
 * buffers are prepared on the first tb_graph_run for the bound input shapes.
 * Fault injection (tests): with TB_FAULT_ALLOC_FAIL=k in the environment at
 * load, the k-th device buffer allocation of the graph fails as if the device
 * were out of memory: the run that needed it returns TB_ERR_CUDA, the buffers
 * made so far stay with the graph, and a later run allocates the rest. */
TB_API tb_status tb_graph_load(tb_context *ctx, const void *data, size_t len, uint32_t flags, tb_graph **out);
TB_API void tb_graph_destroy(tb_graph *graph);
/* The main block's declared inputs / outputs (name, dtype, declared shape). */
TB_API int32_t tb_graph_num_inputs(const tb_graph *graph);
TB_API int32_t tb_graph_num_outputs(const tb_graph *graph);
TB_API tb_status tb_graph_input_info(const tb_graph *graph, int32_t i, tb_tensor_info *info);
TB_API tb_status tb_graph_output_info(const tb_graph *graph, int32_t i, tb_tensor_info *info);
/* Bind one input tensor (an entry of the reference's `inputs` map). `data` is
 * a host buffer (copied to the device before this returns) or, with
 * on_device != 0, a device pointer used in place until the next bind. */
TB_API tb_status tb_graph_set_input(tb_graph *graph, const char *name, int32_t dtype, const int64_t *shape,
                                    int32_t rank, const void *data, uint64_t bytes, int32_t on_device, void *stream);
/* Interpreter::run: execute the main block on `stream` with `hooks` (may be
 * NULL), then wait for the stream and report data-dependent errors. */
TB_API tb_status tb_graph_run(tb_graph *graph, const tb_hooks *hooks, void *stream);
/* After a run: any tensor of the block by name (typically an output): its
 * shape, dtype and device data (the runner's buffer, valid until the next
 * run or bind; NULL when fused away). */
TB_API tb_status tb_graph_get_output(tb_graph *graph, const char *name, tb_tensor_info *info);
/* Copy that tensor's data to the host buffer `dst` (`bytes` >= its size). */
TB_API tb_status tb_graph_read_output(tb_graph *graph, const char *name, void *dst, uint64_t bytes, void *stream);
/* Kernels the last tb_graph_run launched (CUDA-graph replays count their nodes). */
TB_API uint64_t tb_graph_last_launches(const tb_graph *graph);
/* With TB_GRAPH_TIME_OPS: device milliseconds of the operator's kernels in the
 * last run (a fused group's time is reported on its first operator); -1 when
 * the operator launched nothing. */
TB_API float tb_graph_op_time_ms(const tb_graph *graph, int32_t op_index);

#ifdef __cplusplus
}
#endif
#endif /* TOSA_B200_H */
