/*
 * matrixman_b200.h -- C ABI of libmatrixman_b200.so, the B200 (sm_100a) execution
 * runtime behind the `matrixman` PrivateUse1 tensor-op backend.
 *
 * This boundary replaces MatrixMan's legacy-CUDA execution runtime
 * (drivers/matrixman/backends/cuda/gpumatrix.py, class CudaExecutionBackend,
 * gpumatrix.py:4549-5900), which the Python backend façade
 * (drivers/matrixman/backends/cuda/backend.py) drives through ctypes with raw
 * CUdeviceptr values and u32 sizes.  Here every call takes plain pointers,
 * int64 sizes/strides and an opaque stream handle; no torch type crosses it.
 *
 * Conventions
 *  - Every function returns an int status: MM_OK (0) or an mm_status error code.
 *    The message of the last failure on the calling thread is returned by
 *    mm_last_error(); the Python layer maps codes to RuntimeError /
 *    NotImplementedError / ValueError / MemoryError, mirroring the reference's
 *    convention of "RuntimeError(<action>: <CUDA_ERROR_NAME> (<message>))"
 *    (gpumatrix.py:4508-4518).
 *  - `stream` is a cudaStream_t passed as void*; NULL means the device's runtime
 *    stream created by mm_init().
 *  - Tensor descriptors carry the element pointer of logical index [0,...,0]
 *    (storage offset already applied), rank <= MM_MAX_DIMS, sizes and strides in
 *    elements.  Strides may be 0 (broadcast/expand) but never negative.
 *  - All kernels are asynchronous on `stream`.  Waits are bounded polls that
 *    return MM_ERR_TIMEOUT instead of blocking forever.
 */
#ifndef MATRIXMAN_B200_H
#define MATRIXMAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MM_MAX_DIMS 6
#define MM_ABI_VERSION 1

typedef enum mm_status {
  MM_OK = 0,
  MM_ERR_INVALID = 1,      /* bad argument (maps to ValueError) */
  MM_ERR_UNSUPPORTED = 2,  /* unsupported op/dtype/shape (NotImplementedError) */
  MM_ERR_OOM = 3,          /* device memory exhausted after drain + retry (MemoryError) */
  MM_ERR_CUDA = 4,         /* CUDA runtime error (RuntimeError) */
  MM_ERR_TIMEOUT = 5,      /* a bounded wait gave up (TimeoutError) */
  MM_ERR_STATE = 6         /* runtime not initialised / wrong device (RuntimeError) */
} mm_status_t;

typedef enum mm_dtype { MM_F32 = 0, MM_I64 = 1 } mm_dtype_t;

typedef enum mm_pool_kind {
  MM_POOL_ACTIVATION = 0,  /* op outputs: matrixman.config.activation_pool */
  MM_POOL_SCRATCH = 1,     /* intra-op temporaries: matrixman.config.scratch_pool */
  MM_POOL_PARAMETER = 2    /* uploaded/prepacked weights: never pooled */
} mm_pool_kind_t;

typedef enum mm_act {
  MM_ACT_NONE = 0,
  MM_ACT_RELU = 1,
  MM_ACT_SILU = 2,
  MM_ACT_SIGMOID = 3
} mm_act_t;

typedef enum mm_unary_op {
  MM_UNARY_COPY = 0,
  MM_UNARY_SILU = 1,
  MM_UNARY_RELU = 2,
  MM_UNARY_SIGMOID = 3,
  MM_UNARY_ADD_SCALAR = 4,   /* y = x + a */
  MM_UNARY_MUL_SCALAR = 5,   /* y = x * a */
  MM_UNARY_DIV_SCALAR = 6,   /* y = x / a (IEEE division) */
  MM_UNARY_NEG = 7,
  MM_UNARY_CLAMP = 8         /* y = min(max(x, a), b) */
} mm_unary_op_t;

typedef enum mm_binary_op {
  MM_BINARY_ADD = 0,  /* y = a + alpha*b */
  MM_BINARY_SUB = 1,  /* y = a - alpha*b */
  MM_BINARY_MUL = 2,  /* y = a * b */
  MM_BINARY_DIV = 3   /* y = a / b */
} mm_binary_op_t;

typedef struct mm_tensor {
  void* data;
  int32_t dtype;  /* mm_dtype_t */
  int32_t ndim;
  int64_t size[MM_MAX_DIMS];
  int64_t stride[MM_MAX_DIMS];
} mm_tensor_t;

typedef struct mm_device_info {
  char name[256];
  int32_t cc_major;
  int32_t cc_minor;
  int32_t sm_count;
  int32_t reserved;
  int64_t total_bytes;
  int64_t free_bytes;
} mm_device_info_t;

typedef struct mm_pool_stats {
  int64_t live_bytes[3];      /* indexed by mm_pool_kind_t */
  int64_t cached_bytes[3];
  int64_t pending_bytes[3];
  int64_t peak_live_bytes[3];
  int64_t alloc_calls[3];
  int64_t pool_hits[3];
  int64_t device_mallocs;
  int64_t device_frees;
  int64_t oom_recoveries;
  int64_t capture_pools;
} mm_pool_stats_t;

/* Convolution geometry.  Replaces the positional u32 argument list of
 * CudaExecutionBackend.convolution (gpumatrix.py:5414-5788). */
typedef struct mm_conv_params {
  int32_t stride_h, stride_w;
  int32_t pad_h, pad_w;
  int32_t dil_h, dil_w;
  int32_t groups;
  int32_t act;                 /* mm_act_t applied in the epilogue */
  int32_t residual_before_act; /* 1: act(conv+bias+res); 0: act(conv+bias)+res */
  int32_t algo;                /* 0 = auto, 1 = SIMT fp32, 2 = tcgen05 3xTF32,
                                  3 = implicit-GEMM SIMT only (no direct small-C kernel) */
} mm_conv_params_t;

/* ------------------------------------------------------------------------ */
/* Runtime: errors, devices, streams, events                                 */
/* ------------------------------------------------------------------------ */

/* ABI version of the loaded library (MM_ABI_VERSION). */
int mm_abi_version(void);

/* Copy the calling thread's last error message into buf (NUL-terminated).
 * Replaces gpumatrix.py:4508-4518 (check/CudaError formatting). */
int mm_last_error(char* buf, size_t n);

/* Number of visible CUDA devices.  Replaces detect_device (gpumatrix.py:4521-4546),
 * which only ever looked at device 0. */
int mm_device_count(int* out);

/* Name, compute capability, SM count and memory of a device. */
int mm_device_info(int device, mm_device_info_t* out);

/* Create the per-device runtime: context, runtime stream, arena.  Idempotent.
 * Replaces CudaExecutionBackend.__init__ (gpumatrix.py:4552-4764). */
int mm_init(int device);

/* Synchronise, release every cached block and destroy the runtime stream.
 * Replaces CudaExecutionBackend.close (gpumatrix.py:4765-4784). */
int mm_shutdown(int device);

/* Make `device` current for the calling thread. */
int mm_set_device(int device);

/* The device's runtime stream (created by mm_init). */
int mm_runtime_stream(int device, void** stream_out);

int mm_stream_create(int device, void** stream_out);
int mm_stream_destroy(void* stream);

/* Bounded wait for all work on `stream`; MM_ERR_TIMEOUT after timeout_ms
 * (timeout_ms < 0 waits without limit).  Replaces cuCtxSynchronize at the
 * readback boundary (gpumatrix.py:4896-4911). */
int mm_stream_sync(void* stream, int64_t timeout_ms);

/* 1 in *done if every operation on the stream has completed. */
int mm_stream_query(void* stream, int* done);

int mm_event_create(void** event_out, int timing);
int mm_event_destroy(void* event);
int mm_event_record(void* event, void* stream);
int mm_event_sync(void* event, int64_t timeout_ms);
int mm_stream_wait_event(void* stream, void* event);
/* Milliseconds between two recorded events.  Replaces the CUDA-event GPU
 * timing of gpumatrix.py:4785-4816. */
int mm_event_elapsed_ms(void* start, void* stop, float* ms);

/* ------------------------------------------------------------------------ */
/* Caching arena (activation_pool / scratch_pool)                            */
/* ------------------------------------------------------------------------ */

/* Pool policy.  sync_safe=1: a reused block is ordered after its last use by a
 * stream-event wait ("safe"); 0: stream-ordered reuse only ("relaxed").
 * deferred_*=1: released blocks stay pending until their release event has
 * completed ("deferred"); 0: immediately reusable ("safe").  Maps
 * matrixman.config sync_policy/activation_pool/scratch_pool (config.py:19-42)
 * onto the exact-size pool with deferred release of gpumatrix.py:4846-5012. */
int mm_pool_configure(int device, int sync_safe, int deferred_activation, int deferred_scratch,
                      int disable_pool);

/* Allocate `bytes` of device memory from pool `kind`.  On exhaustion the arena
 * synchronises, drains pending/cached blocks and retries once before failing
 * with MM_ERR_OOM.  Replaces CudaExecutionBackend.allocate / _allocate_driver
 * (gpumatrix.py:4926-4962, 4913-4923). */
int mm_alloc(int device, size_t bytes, int kind, void* stream, void** out);

/* Release a block; reuse is ordered after all work queued on `stream`.
 * Replaces CudaExecutionBackend.free (gpumatrix.py:4965-5001). */
int mm_free(void* ptr, void* stream);

/* Move completed pending blocks to the cache and cudaFree every cached block.
 * Replaces _drain_pool (gpumatrix.py:5002-5012). */
int mm_pool_trim(int device);

int mm_pool_stats(int device, mm_pool_stats_t* out);

/* Test hook: after `n` more successful device allocations, report device OOM
 * (n < 0 disables).  Environment: MATRIXMAN_TEST_FAIL_ALLOC_AFTER. */
int mm_debug_fail_alloc_after(int device, int64_t n);

/* Host-backed arena instance with the same policy code, for CPU-only tests of the
 * pool state machine (no GPU needed).  Events are simulated: a release recorded
 * at generation g completes once mm_host_arena_complete(g' >= g) is called. */
int mm_host_arena_create(int64_t capacity_bytes, int deferred, void** arena_out);
int mm_host_arena_destroy(void* arena);
int mm_host_arena_alloc(void* arena, size_t bytes, int kind, void** out);
int mm_host_arena_free(void* arena, void* ptr);
int mm_host_arena_complete(void* arena, int64_t generation);
int mm_host_arena_generation(void* arena, int64_t* out);
int mm_host_arena_fail_after(void* arena, int64_t n);
int mm_host_arena_stats(void* arena, mm_pool_stats_t* out);

/* ------------------------------------------------------------------------ */
/* Copies                                                                    */
/* ------------------------------------------------------------------------ */

/* Host<->device copies.  `sync` = 1 waits (bounded) for completion.  Replace
 * to_device / from_device (gpumatrix.py:5021-5049). */
int mm_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream, int sync);
int mm_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream, int sync);
int mm_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
/* Copy-engine copy between two devices (NVLink when peer access is enabled). */
int mm_memcpy_peer(void* dst, int dst_device, const void* src, int src_device, size_t bytes,
                   void* stream);
int mm_enable_peer_access(int device, int peer);
/* Device memory shared between processes, one process per GPU (no counterpart
 * in the reference, which drives device 0 only).  mm_ipc_alloc allocates
 * `bytes` on `device` and writes its CUDA IPC handle (64 bytes) to handle_out;
 * another process passes the handle to mm_ipc_open (on its own device) and
 * gets a pointer it may copy into with mm_memcpy_d2d (copy engines over
 * NVLink); mm_ipc_close unmaps it; the owner frees with mm_ipc_free after
 * every opener has closed it. */
#define MM_IPC_HANDLE_BYTES 64
int mm_ipc_alloc(int device, size_t bytes, void** ptr_out, void* handle_out);
int mm_ipc_free(int device, void* ptr);
int mm_ipc_open(int device, const void* handle, void** ptr_out);
int mm_ipc_close(int device, void* ptr);
/* Page-locked host buffers for asynchronous transfers. */
int mm_host_alloc_pinned(size_t bytes, void** out);
int mm_host_free_pinned(void* ptr);
/* 1 in *out when ptr lies in page-locked host memory (torch's
 * Tensor.is_pinned() on the matrixman backend). */
int mm_host_is_pinned(const void* ptr, int* out);

/* ------------------------------------------------------------------------ */
/* CUDA graphs (prepared-model execution)                                    */
/* ------------------------------------------------------------------------ */

/* Begin capturing work queued on `stream`.  Arena allocations made on this
 * device until mm_graph_capture_end come from a private pool owned by the
 * graph, so replay never races with eager allocations. */
int mm_graph_capture_begin(int device, void* stream);
int mm_graph_capture_end(int device, void* stream, void** graph_out);
int mm_graph_launch(void* graph, void* stream);
/* Synchronise and free the graph and its private pool. */
int mm_graph_destroy(void* graph);

/* ------------------------------------------------------------------------ */
/* Operators                                                                 */
/* ------------------------------------------------------------------------ */

/* y = op(x) elementwise, any strides, x and y of equal logical shape (y may
 * alias x for in-place).  Replaces matrix_sigmoid / silu / matrix_add_scalar /
 * matrix_div_scalar kernels (gpumatrix.py:581, 4012, 478, 510) and
 * CudaBackend.{sigmoid,silu,div} (cuda/backend.py:733-796, 1031-1070). */
int mm_unary(int op, const mm_tensor_t* x, const mm_tensor_t* y, double a, double b, void* stream);

/* y = op(a, b) with broadcasting expressed by 0-strides.  Replaces matrix_add /
 * matrix_sub / matrix_mul_elementwise (gpumatrix.py:171, 351, 265) and
 * CudaBackend.{add,sub,mul} (cuda/backend.py:888-1122). */
int mm_binary(int op, const mm_tensor_t* a, const mm_tensor_t* b, const mm_tensor_t* y,
              double alpha, void* stream);

/* y[...] = value.  Replaces matrix_fill (gpumatrix.py:728). */
int mm_fill(const mm_tensor_t* y, double value, void* stream);

/* y[i] = start + i*step over a 1-D tensor.  Replaces matrix_arange (gpumatrix.py:445). */
int mm_arange(const mm_tensor_t* y, double start, double step, void* stream);

/* y = x for arbitrary strides (materialising copy).  Replaces split_copy /
 * stack_copy (gpumatrix.py:4049, 652). */
int mm_copy(const mm_tensor_t* x, const mm_tensor_t* y, void* stream);

/* Concatenate `n` tensors along `dim` into y (one launch per input, each
 * writing only its own slot).  Replaces cat_copy (gpumatrix.py:4135), which
 * launched numel(out) threads per input. */
int mm_cat(const mm_tensor_t* const* inputs, int n, int dim, const mm_tensor_t* y, void* stream);

/* Eval-mode BatchNorm over channel dim 1: y = (x-mean)*rsqrt(var+eps)*w + b.
 * Replaces batch_norm_inference (gpumatrix.py:3945-4010). */
int mm_batch_norm(const mm_tensor_t* x, const float* mean, const float* var, const float* weight,
                  const float* bias, double eps, const mm_tensor_t* y, void* stream);

/* Softmax (log=0) or log-softmax (log=1) along `dim`.  Replaces matrix_softmax
 * (gpumatrix.py:784-931) and CudaBackend.softmax (cuda/backend.py:1290-1349). */
int mm_softmax(const mm_tensor_t* x, int dim, int log, const mm_tensor_t* y, void* stream);

/* Training-path ops (backward passes and Adam's update).  The reference has
 * them on its OpenGL backend only: backends/opengl/dispatch.py:171-179
 * (lerp_), :264-290 (addcmul_, addcdiv_), :299 (sqrt), :377-382
 * (threshold_backward), :463-479 (log-softmax backward, NLL forward and
 * backward). */
enum {
  MM_PW3_THRESHOLD_BACKWARD = 0, /* y = a <= s ? 0 : x   (x = grad, a = self) */
  MM_PW3_ADDCMUL = 1,            /* y = fma(s * a, b, x) */
  MM_PW3_ADDCDIV = 2,            /* y = x + (s * a) / b */
  MM_PW3_LERP = 3,               /* y = lerp(x, a, weight s); b unused */
  MM_PW3_SQRT = 4                /* y = sqrt(x); a, b unused */
};

/* Element-wise op over x, a, b (same shape as y, any strides; y may be x). */
int mm_pointwise3(int op, const mm_tensor_t* x, const mm_tensor_t* a, const mm_tensor_t* b,
                  const mm_tensor_t* y, double s, void* stream);

/* _log_softmax_backward_data: y = grad - exp(output) * sum(grad along dim);
 * contiguous operands. */
int mm_log_softmax_backward(const mm_tensor_t* grad, const mm_tensor_t* output, int dim,
                            const mm_tensor_t* y, void* stream);

/* nll_loss_forward: input [N, C] f32 (log-probabilities), target [N] int64,
 * weight [C] or NULL; reduction 0 none (out [N]), 1 mean, 2 sum (out and
 * total_weight hold one value).  Rows whose target is ignore_index are
 * skipped; targets must otherwise lie in [0, C) (the caller checks). */
int mm_nll_loss(const mm_tensor_t* input, const mm_tensor_t* target, const mm_tensor_t* weight,
                int reduction, int64_t ignore_index, const mm_tensor_t* out,
                const mm_tensor_t* total_weight, void* stream);

/* nll_loss_backward into a contiguous grad_input [N, C] (zeroed here). */
int mm_nll_loss_backward(const mm_tensor_t* grad_output, const mm_tensor_t* input,
                         const mm_tensor_t* target, const mm_tensor_t* weight, int reduction,
                         int64_t ignore_index, const mm_tensor_t* total_weight,
                         const mm_tensor_t* grad_input, void* stream);

/* Generic 2-D max pooling over dims (2,3) of a rank-4 tensor, -inf padding,
 * NaN-propagating like torch.  Replaces max_pool2d_5x5_s1_p2 (gpumatrix.py:74)
 * and CudaBackend.max_pool2d (cuda/backend.py:1351-1393), which only accepted
 * 5x5/s1/p2. */
int mm_max_pool2d(const mm_tensor_t* x, int kh, int kw, int sh, int sw, int ph, int pw, int dh,
                  int dw, const mm_tensor_t* y, void* stream);

/* SPPF pooling chain: y1 = pool5(x), y2 = pool5(y1), y3 = pool5(y2) with 5x5/s1/p2
 * max pooling, computed in one pass (nested 5/9/13 windows).  y1..y3 are
 * typically channel slices of the SPPF concat buffer.  Fuses the three
 * max_pool2d_5x5_s1_p2 launches of the reference SPPF path. */
int mm_sppf_pool(const mm_tensor_t* x, const mm_tensor_t* y1, const mm_tensor_t* y2,
                 const mm_tensor_t* y3, void* stream);

/* avg_pool2d with torch semantics (count_include_pad, divisor_override <= 0 =
 * none, ceil_mode handled by the caller through the output size).  Semantics of
 * the OpenGL-only reference pooling (backends/opengl/ops/pooling.py). */
int mm_avg_pool2d(const mm_tensor_t* x, int kh, int kw, int sh, int sw, int ph, int pw,
                  int count_include_pad, int divisor_override, const mm_tensor_t* y, void* stream);

/* Adaptive average pooling over dims (2,3). */
int mm_adaptive_avg_pool2d(const mm_tensor_t* x, const mm_tensor_t* y, void* stream);

/* Mean (or sum when mean=0) over the dims whose bit is set in dim_mask; y has
 * the reduced dims with size 1.  Semantics of backends/opengl/ops/reduction.py:136-221. */
int mm_reduce(const mm_tensor_t* x, uint32_t dim_mask, int mean, const mm_tensor_t* y, void* stream);

/* Nearest-neighbour 2-D upsampling with torch's index rule; scale_h/scale_w > 0
 * are the user scale factors (source index = floor(dst * (1/scale))), else
 * input/output size ratios.  Replaces upsample_nearest2d (gpumatrix.py:4244-4299). */
int mm_upsample_nearest2d(const mm_tensor_t* x, double scale_h, double scale_w,
                          const mm_tensor_t* y, void* stream);

/* 2-D convolution, fp32, any strides for x/y/residual, weight given as a rank-4
 * tensor [K, C/groups, R, S] with arbitrary strides (KCRS from torch, or the
 * KRSC prepack of matrixman.prepare).  Epilogue: bias, activation, residual.
 * Replaces conv2d_nchw and all specialised conv .entry kernels
 * (gpumatrix.py:989-3943) and CudaBackend.convolution (cuda/backend.py:296-607). */
int mm_conv2d(const mm_tensor_t* x, const mm_tensor_t* w, const float* bias,
              const mm_tensor_t* residual, const mm_conv_params_t* p, const mm_tensor_t* y,
              void* stream);

/* One region of a convolution's output: output rows [row0, row0 + H) and
 * columns [col0, col0 + W), where H x W is y's spatial size (y, and the
 * residual if given, are views of that region; p describes the whole
 * convolution).  The region reads the input rows and columns the whole
 * convolution would read for it (padding applies only at the image borders)
 * and each output value is computed in the same order, so tiling an output
 * into regions gives the same result bit for bit.  The CUDA mapping of the
 * reference's tileLimit (config.py:305-314; consumed by the OpenGL convolution,
 * backends/opengl/convolution.py:1299), which bounds the extent of one
 * convolution pass. */
int mm_conv2d_region(const mm_tensor_t* x, const mm_tensor_t* w, const float* bias,
                     const mm_tensor_t* residual, const mm_conv_params_t* p, int64_t row0, int64_t col0,
                     const mm_tensor_t* y, void* stream);

/* 3xTF32 tensor-core convolution on a prepacked weight: w_hi/w_lo are
 * [K_pad][R*S][C_pad] (C_pad % 32 == 0, K_pad % 16 == 0) with the tf32 high part
 * and the fp32 remainder of each weight.  x/y/residual must be NHWC views
 * (channel stride 1, C % 4 == 0).  Returns MM_ERR_UNSUPPORTED for geometries the
 * tcgen05 path does not cover (the caller then uses mm_conv2d). */
int mm_conv2d_tc(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out, int c_in,
                 int r, int s, int c_pad, int k_pad, const float* bias,
                 const mm_tensor_t* residual, const mm_conv_params_t* p, const mm_tensor_t* y,
                 void* stream);

/* mm_conv2d_tc for one region of the output (rows [row0, row0 + H), columns
 * [col0, col0 + W) of y's H x W), with the same bit-for-bit guarantee as
 * mm_conv2d_region; the tensor-core counterpart of the same tileLimit mapping. */
int mm_conv2d_tc_region(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out, int c_in,
                        int r, int s, int c_pad, int k_pad, const float* bias,
                        const mm_tensor_t* residual, const mm_conv_params_t* p, int64_t row0,
                        int64_t col0, const mm_tensor_t* y, void* stream);

/* Error code recorded by a device-side bounded wait that gave up (0 = none);
 * clear != 0 resets it.  Kernels never trap: a stuck pipeline records the code,
 * frees its tensor memory and returns, and the host reads the code here. */
int mm_kernel_error(int device, int* code_out, int clear);

/* Test hook for the bounded-wait error path of mm_conv2d_tc (no counterpart in
 * the reference): for later launches on `device`, the budget of every
 * device-side wait (wait_ns <= 0 restores the default 200 ms) and, when
 * drop_first_load != 0, CTA 0 leaves its first k-block's loads unissued so that
 * the waits for that stage run out: the kernel records an error code (read
 * with mm_kernel_error), finishes its own in-flight copies and MMAs, frees its
 * tensor memory and returns.  Not for production use. */
int mm_debug_tc_fault(int device, int64_t wait_ns, int drop_first_load);

/* Split prepacked weights into the tf32 high part and the fp32 remainder
 * (w_hi = w with its 13 low mantissa bits cleared, w_lo = w - w_hi), in place on
 * the device: n elements of src -> hi, lo. */
int mm_tf32_split(const float* src, float* hi, float* lo, int64_t n, void* stream);

/* y[M,N] = act(alpha * x[M,K] @ w + beta * bias) with w given as a rank-2 tensor
 * [K, N] of arbitrary strides (pass w^T of a Linear weight).  bias may be NULL
 * or a rank-1/rank-2 broadcastable tensor.  Replaces matrix_mul (gpumatrix.py:933)
 * and adds the OpenGL-only addmm semantics (backends/opengl/ops/matmul.py:262-281). */
int mm_gemm(const mm_tensor_t* x, const mm_tensor_t* w, const mm_tensor_t* bias, double alpha,
            double beta, int act, const mm_tensor_t* y, void* stream);

/* YOLOv8 detect-head decode over `nlevels` feature levels.  feats[i] is an NHWC
 * [B, H_i, W_i, 4*reg_max + nc] tensor (box logits then class logits); out is
 * [B, 4 + nc, A] with A = sum(H_i*W_i).  Per anchor: DFL (softmax over reg_max
 * bins, expectation with weights 0..reg_max-1), dist2bbox against the anchor
 * centre (x+0.5, y+0.5) to xywh, times the level stride; class scores through
 * sigmoid.  Fuses PreparedCudaDFL (preparation.py:197-268) with the decode that
 * the reference leaves to generic ops. */
int mm_yolo_decode(const mm_tensor_t* const* feats, const float* strides, int nlevels, int reg_max,
                   int nc, const mm_tensor_t* out, void* stream);

/* Detection reduction: pred [B, 4+classes, anchors] -> out [B, 6, anchors] =
 * (cx, cy, w, h, best score, best class index as float); the best score starts
 * at -1 and a class replaces it only when strictly greater.  Replaces
 * reduce_detection_output (backends/opengl/ops/postprocessing.py:87-119, the
 * shader at :35-52), exposed as gpu_postprocess_detection (backend.py:263-266);
 * the reference accepts B = 1 only. */
int mm_detect_reduce(const mm_tensor_t* pred, const mm_tensor_t* out, void* stream);

/* Candidates (anchors at or above the confidence threshold) per image that
 * mm_detect_nms sorts and suppresses in shared memory; an image with more takes
 * a slower global-memory pass with the same result. */
#define MM_DETECT_MAX_CANDIDATES 12288

/* Confidence filter, box conversion and per-class greedy NMS on the device, per
 * image: the reference's CPU detections() (demo/yolo_helpers.py:91-137, NMS at
 * :59-89).  Candidates: best class (first maximum) with score >= conf_thr;
 * boxes (cx - w/2, cy - h/2, cx + w/2, cy + h/2) clamped to [0, width-1] x
 * [0, height-1]; NMS keeps a candidate only if IoU <= iou_thr against every
 * earlier kept candidate of its class, in descending score order (equal scores
 * by anchor index).  dets [B, max_det, 6] receives the first max_det kept
 * (x1, y1, x2, y2, score, class) in descending score order and counts (device
 * int32[B]) their number.  The number of candidates per image is not limited
 * (beyond MM_DETECT_MAX_CANDIDATES an image runs a global-memory pass; the
 * reference's detections() has no cap either).  workspace: device
 * memory, 256-byte aligned, of at least mm_detect_nms_workspace_size bytes for
 * this batch and anchor count (it holds the candidates between the two
 * kernels); calls that run at the same time need separate workspaces. */
int mm_detect_nms(const mm_tensor_t* pred, float conf_thr, float iou_thr, float width, float height,
                  int max_det, const mm_tensor_t* dets, int32_t* counts, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Workspace bytes mm_detect_nms needs for a [batch, 4+classes, anchors]
 * prediction (24 bytes per anchor plus 16 per possible candidate, per image).
 * No counterpart in the reference, whose NMS runs on the CPU. */
int mm_detect_nms_workspace_size(int64_t batch, int64_t anchors, size_t* bytes);

/* Scratch size behind mm_detect_nms_static, fixed per GPU: 4 MiB, enough for
 * 10 images of 640 x 640 (8400 anchors) in one call. */
#define MM_DETECT_STATIC_WORK_BYTES (4u << 20)

/* mm_detect_nms for callers that cannot allocate device memory: a plugin
 * inside an application that owns all GPU memory and forbids cudaMalloc after
 * start-up, or a real-time loop whose memory is fixed before it runs.  It
 * takes no workspace and allocates nothing; its scratch is a static device
 * array of MM_DETECT_STATIC_WORK_BYTES that every GPU loading the library
 * holds until the process exits.  Same arguments and results as mm_detect_nms
 * otherwise.  A call whose batch needs more scratch (see
 * mm_detect_nms_workspace_size) fails with MM_ERR_UNSUPPORTED.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  All calls on a device share the
 * array: calls that overlap on the GPU (other streams, other host threads)
 * race, so serialise them.  No counterpart in the reference. */
int mm_detect_nms_static(const mm_tensor_t* pred, float conf_thr, float iou_thr, float width,
                         float height, int max_det, const mm_tensor_t* dets, int32_t* counts,
                         void* stream);

/* Frame preprocessing: frames (device, contiguous uint8 [n, h, w, 3] BGR) ->
 * out [n, 3, out_h, out_w] float32 RGB / 255, resized with OpenCV's 8-bit
 * INTER_LINEAR fixed-point bilinear algorithm.  Replaces the reference's CPU
 * preprocess_frame (demo/yolo_helpers.py:53-56: cv2.resize, cvtColor
 * BGR2RGB, permute, / 255), so uploads carry uint8 frames. */
int mm_preprocess_bgr8(const uint8_t* frames, int64_t n, int64_t h, int64_t w, const mm_tensor_t* out,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MATRIXMAN_B200_H */
