/*
 * liblaya_cuda — C ABI of the B200 (sm_100a) backend for the laya-js
 * tensor-backend contract.
 *
 * Every entry point replaces one member of the reference's `Backend<T>`
 * interface (packages/tensor-backend/src/index.ts:139-317; cited per entry
 * as index.ts:LINE) or one of its optional-op helpers
 * (packages/tensor-backend/src/compose.ts). The calling convention follows
 * how the reference's native backend binds mlx-c over FFI
 * (packages/backend-mlx/src/ffi.ts:31-114):
 *
 *  - handles are opaque 64-bit integers (JS numbers below 2^53);
 *  - every call returns int: 0 = ok, nonzero = error, with the message in
 *    lc_last_error() (thread-local; replaces mlx-c's error-handler callback,
 *    packages/backend-mlx/src/ffi.ts:15-16,190-201);
 *  - results come back through out-parameters (caller scratch), shapes are
 *    int64 arrays plus a count, optional tensors are 0;
 *  - ops are asynchronous on the library's stream (lc_set_stream); only
 *    lc_read synchronises. The library never calls exit().
 *
 * dtype codes (packages/tensor-backend/src/index.ts:39):
 *   0 f32, 1 f16, 2 bf16, 3 i32, 4 bool, 5 u8, 6 i8, 7 u16, 8 i16, 9 u32,
 *   10 u64, 11 i64, 12 f64.
 */
#ifndef LAYA_CUDA_H
#define LAYA_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t lc_tensor;

/* ---- library lifetime (createMlxBackend / destroy: index.ts:164-166) ---- */
/* Binds the calling thread's library state to CUDA device `device`. */
int lc_init(int device);
/* index.ts:165-166 destroy: frees every live tensor and cached table. */
int lc_destroy(void);
const char* lc_last_error(void);
/* Makes `stream` (a cudaStream_t, 0 = the library's own stream) current. */
int lc_set_stream(uint64_t stream);
int lc_get_stream(uint64_t* stream);
/* index.ts:142-143 supports(dtype): 1 or 0 in *out. */
int lc_supports(int dtype, int* out);
/* Counters for tracing: live tensors, live bytes, kernel launches issued. */
int lc_stats(int64_t* live_tensors, int64_t* live_bytes, int64_t* launches);

/* ---- transfer / lifetime (index.ts:145-166) ---- */
/* index.ts:146-154 fromHost: copies `nbytes` of row-major host data before returning. */
int lc_from_host(lc_tensor* out, int dtype, const int64_t* shape, int ndim, const void* data, size_t nbytes);
/* Wraps device memory the caller owns as a dense tensor (never freed by the library). */
int lc_from_device(lc_tensor* out, int dtype, const int64_t* shape, int ndim, void* dptr);
/* index.ts:155-156 read: synchronises and copies the row-major values to `dst`. */
int lc_read(lc_tensor t, void* dst, size_t nbytes);
/* index.ts:157-158 dispose (idempotent at the TS layer; the C call rejects a dead handle). */
int lc_tensor_free(lc_tensor t);
/* Shape and dtype of a handle (Tensor.shape / Tensor.dtype, index.ts:75-78). */
int lc_tensor_info(lc_tensor t, int* dtype, int* ndim, int64_t* shape /* [8] */);
/* Device pointer of a dense tensor (0 when it is a strided view). Read-only:
   the library treats tensors as immutable (only lc_copy_into writes one). */
int lc_tensor_data(lc_tensor t, uint64_t* dptr);
/* index.ts:163-164 flush: waits for queued work. */
int lc_flush(void);

/* ---- shape (index.ts:168-177) ---- */
int lc_reshape(lc_tensor* out, lc_tensor x, const int64_t* shape, int ndim);
int lc_transpose(lc_tensor* out, lc_tensor x, const int32_t* perm, int ndim);
int lc_slice(lc_tensor* out, lc_tensor x, const int64_t* begin, const int64_t* end, int n);
int lc_split(lc_tensor* outs, lc_tensor x, int parts, int axis);
int lc_concat(lc_tensor* out, const lc_tensor* xs, int n, int axis);
int lc_cast(lc_tensor* out, lc_tensor x, int dtype);

/* ---- elementwise, numpy broadcasting (index.ts:179-198) ---- */
int lc_add(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_sub(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_mul(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_div(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_maximum(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_where(lc_tensor* out, lc_tensor cond, lc_tensor a, lc_tensor b);
int lc_scale(lc_tensor* out, lc_tensor x, double s);
int lc_exp(lc_tensor* out, lc_tensor x);
int lc_log(lc_tensor* out, lc_tensor x);
int lc_relu(lc_tensor* out, lc_tensor x);
int lc_gelu(lc_tensor* out, lc_tensor x);

/* ---- reductions (index.ts:200-206) ---- */
int lc_sum(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_max(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_softmax(lc_tensor* out, lc_tensor x, int axis);
int lc_sort(lc_tensor* out, lc_tensor x, int axis);

/* ---- linear algebra & NN (index.ts:208-237) ---- */
int lc_matmul(lc_tensor* out, lc_tensor a, lc_tensor b);
/* index.ts:211-215 linear: y = x·wᵀ (+ b), f32 accumulation; bias 0 = none. */
int lc_linear(lc_tensor* out, lc_tensor x, lc_tensor w, lc_tensor bias);
/* index.ts:216-217 layerNorm; weight/bias 0 = none. */
int lc_layer_norm(lc_tensor* out, lc_tensor x, lc_tensor weight, lc_tensor bias, double eps);
int lc_embedding(lc_tensor* out, lc_tensor table, lc_tensor ids);
int lc_gather_rows(lc_tensor* out, lc_tensor x, lc_tensor idx);
int lc_rope(lc_tensor* out, lc_tensor x, double base);
/* index.ts:230-237 sdpa; mask 0 = none. */
int lc_sdpa(lc_tensor* out, lc_tensor q, lc_tensor k, lc_tensor v, lc_tensor mask, double scale);

/* ---- optional fused ops (index.ts:239-245; compose.ts:87-105) ---- */
int lc_geglu(lc_tensor* out, lc_tensor x);
int lc_mean_pool(lc_tensor* out, lc_tensor x, lc_tensor mask);

/* ---- optional quantized trio (index.ts:247-263) ---- */
/*
 * index.ts:250-255 fromHostQuantized. `data` is HostQuantized.data
 * (N·K·bits/8 bytes, index.ts:98-108); scales/biases are [N, ceil(K/g)]
 * host arrays of `sb_dtype` (0 f32, 1 f16, 2 bf16); biases NULL for
 * symmetric. The values dequantize to `dtype`. Out: packed weight, scales,
 * biases (0 when symmetric) in the library's native layout.
 * mode: 0 = symmetric, 1 = affine.
 */
int lc_from_host_quantized(lc_tensor* w, lc_tensor* scales, lc_tensor* biases,
                           int64_t n, int64_t k, int bits, int group_size, int mode,
                           const uint8_t* data, int sb_dtype, const void* scales_host,
                           const void* biases_host, int dtype);
/* index.ts:256-259 quantizedLinear; biases/bias 0 = none. */
int lc_quantized_linear(lc_tensor* out, lc_tensor x, lc_tensor w, lc_tensor scales, lc_tensor biases,
                        int bits, int group_size, int mode, lc_tensor bias);
/* index.ts:260-262 quantizedEmbedding. */
int lc_quantized_embedding(lc_tensor* out, lc_tensor w, lc_tensor scales, lc_tensor biases,
                           int bits, int group_size, int mode, lc_tensor ids);
/* Dequantized matrix [N, K] in the scales' dtype (each value fl(q·s + b) rounded once). */
int lc_dequantize(lc_tensor* out, lc_tensor w, lc_tensor scales, lc_tensor biases,
                  int bits, int group_size, int mode);
/*
 * No counterpart in the reference. quantizedLinear for callers that cannot
 * allocate device memory (a host whose device memory belongs to another
 * framework's allocator, or a hot path that must not call cudaMalloc/cudaFree,
 * which can synchronise the device): y[m, n] = x[m, k] · dequant(w)ᵀ (+ bias)
 * on raw device pointers, with the dequantised weight in a fixed 8 MiB scratch
 * array that every GPU loading the library reserves (n·k <= 4,194,304).
 * x/y f16 or bf16 (dtype 1/2), k >= 64 and k % 8 == 0, 16-byte aligned
 * pointers; w/scales/biases as lc_from_host_quantized stores them (sb_dtype);
 * bias optional ([n], bias_dtype). Allocates nothing. The first call on each
 * device resolves the scratch address; make it before any stream capture.
 * Calls share the scratch: calls that overlap on the GPU race. As for the
 * rest of this library, make calls from one host thread at a time.
 */
int lc_quantized_linear_noalloc(void* y, const void* x, int64_t m, int64_t k, int dtype, const uint8_t* w, const void* scales,
                                const void* biases, int64_t n, int bits, int group_size, int mode, int sb_dtype,
                                const void* bias, int bias_dtype, uint64_t stream);

/* ---- optional compile (index.ts:244-245) as CUDA-graph capture ----
 * The ops issued on the library stream between _begin and _end are recorded
 * (relaxed stream capture) into a graph that _launch replays; allocations
 * made while capturing belong to the graph and must be released before _end
 * (copy results out with lc_copy_into first). Memory released while
 * capturing that predates the capture is kept until lc_graph_destroy. An op
 * that synchronises with the host fails the capture; _abort discards it. */
int lc_graph_capture_begin(void);
int lc_graph_capture_end(uint64_t* graph);
int lc_graph_capture_abort(void);
int lc_graph_launch(uint64_t graph);
int lc_graph_destroy(uint64_t graph);
/* dst (dense) <- src, same dtype and shape, on the library stream (capturable). */
int lc_copy_into(lc_tensor dst, lc_tensor src);

/* ---- failure-path test hooks (no counterpart in the reference) ----
 * Every mbarrier wait in the pipelined kernels gives up after a limit (2 s),
 * records the timeout in a device error word and returns; lc_flush / lc_read
 * report it. lc_debug_set_wait_limit(ns) shortens that limit (0 restores 2 s)
 * and lc_debug_stuck_wait launches one kernel whose wait nothing satisfies,
 * so a test can check the error path without faulting or hanging the GPU.
 * lc_debug_set_alloc_cap(bytes) makes tensor allocations fail with the
 * out-of-memory error once the live tensor bytes would pass `bytes` (0 = no
 * cap), so the out-of-memory path can be exercised on any GPU. */
int lc_debug_set_wait_limit(uint64_t ns);
int lc_debug_stuck_wait(void);
int lc_debug_set_alloc_cap(int64_t bytes);

/* ---- optional general numerics (index.ts:265-316) ---- */
int lc_equal(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_not_equal(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_less(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_less_equal(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_greater(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_greater_equal(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_logical_and(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_logical_or(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_logical_not(lc_tensor* out, lc_tensor x);
int lc_sqrt(lc_tensor* out, lc_tensor x);
int lc_rsqrt(lc_tensor* out, lc_tensor x);
int lc_pow(lc_tensor* out, lc_tensor a, lc_tensor b);
int lc_neg(lc_tensor* out, lc_tensor x);
int lc_abs(lc_tensor* out, lc_tensor x);
int lc_tanh(lc_tensor* out, lc_tensor x);
int lc_sigmoid(lc_tensor* out, lc_tensor x);
int lc_erf(lc_tensor* out, lc_tensor x);
int lc_argmax(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_argmin(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_mean(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_min(lc_tensor* out, lc_tensor x, int axis, int keep_dims);
int lc_cumsum(lc_tensor* out, lc_tensor x, int axis);

#ifdef __cplusplus
}
#endif
#endif /* LAYA_CUDA_H */
