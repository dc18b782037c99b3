/*
 * b2m.h — C ABI of libb200mm.so, the B200 (sm_100a) backend for the
 * MatMul-family operators of onnx_runtime_dart.
 *
 * The reference runtime executes these operators in pure Dart; its operator
 * dispatch (OnnxGraphExecutor._dispatch, lib/src/onnx_graph.dart:1549) calls
 *   MatMul        -> ops.opMatMul             lib/src/onnx_ops.dart:1710
 *   Gemm          -> ops.opGemm (+ transB prepack)  onnx_ops.dart:2152, onnx_graph.dart:2156-2173
 *   MatMulInteger -> ql.opMatMulInteger       lib/src/onnx_qlinear_ops.dart:32
 *   QLinearMatMul -> ql.opQLinearMatMul       onnx_qlinear_ops.dart:85 (dispatch onnx_graph.dart:2902-2917)
 *   MatMulNBits   -> ql.opMatMulNBits         onnx_qlinear_ops.dart:115 (dispatch onnx_graph.dart:2918-2934)
 * Each b2m_* op below replaces one of those calls for device-resident
 * operands; a dart:ffi binding (pattern: lib/src/ort/ort_backend.dart) calls
 * them from the same dispatch cases.
 *
 * Conventions (mirroring the reference's native binding):
 *   - Every entry point returns a b2m_status; 0 is success. On failure
 *     b2m_last_error() returns a message for the calling thread (the ORT
 *     binding reads GetErrorMessage the same way, ort_backend.dart:774-782).
 *     Status codes map onto the reference's exceptions: INVALID_ARGUMENT ->
 *     ArgumentError, UNSUPPORTED -> UnsupportedError, OUT_OF_MEMORY ->
 *     OnnxMemoryLimitException, CANCELLED -> OnnxCancelledException.
 *   - Nothing aborts the process; no entry point throws across the ABI.
 *   - Tensors are row-major device buffers. Element types use ONNX
 *     TensorProto.DataType codes (B2M_FLOAT = 1, ...), the codes the reference
 *     already keys on (onnx_graph.dart:2903: elem type 3 = INT8).
 *   - Op outputs: `y` is in/out. If *y is NULL the library allocates the
 *     output tensor (the reference allocates fresh outputs, onnx_ops.dart:1741);
 *     otherwise *y must already have the output's dtype and element count
 *     and is written in place (no allocation on the hot path).
 *   - Calls are enqueued on the context's current stream and return without
 *     synchronising, except the b2m_*_host helpers and downloads, which
 *     return after the result is in host memory.
 *   - One b2m_ctx per thread / isolate and device; a context is not safe for
 *     concurrent use from several threads (sessions are not shared across
 *     isolates in the reference either, docs/native_backend.md:99-110).
 */
#ifndef B2M_H_
#define B2M_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B2M_API __attribute__((visibility("default")))
#else
#define B2M_API
#endif

#define B2M_ABI_VERSION 1

typedef int32_t b2m_status;
#define B2M_OK 0
#define B2M_ERR_INVALID_ARGUMENT 1 /* Dart ArgumentError (onnx_qlinear_ops.dart:135,152,162,165) */
#define B2M_ERR_UNSUPPORTED 2      /* Dart UnsupportedError (onnx_qlinear_ops.dart:38,89,127) */
#define B2M_ERR_OUT_OF_MEMORY 3    /* device allocation failed or byte budget exceeded */
#define B2M_ERR_CUDA 4             /* a CUDA runtime/driver call failed */
#define B2M_ERR_TIMEOUT 5          /* a bounded device-side wait gave up */
#define B2M_ERR_CANCELLED 6        /* the context's cancel flag was set before launch */
#define B2M_ERR_NO_DEVICE 7        /* no CUDA device / unsupported device */

/* Element types: ONNX TensorProto.DataType codes. */
#define B2M_FLOAT 1
#define B2M_UINT8 2
#define B2M_INT8 3
#define B2M_INT32 6
#define B2M_INT64 7
#define B2M_FLOAT16 10

/* Arithmetic modes for the floating-point ops. */
#define B2M_MODE_EXACT 0 /* bitwise identical to the reference Dart kernels */
#define B2M_MODE_FAST 1  /* tensor cores; max|d|/max|ref| <= 1e-3, cosine >= 0.99999 */
/* MatMulNBits only: tensor cores on weights dequantized exactly as the
 * reference's weight() and split, with the activations, into two bf16 terms
 * (three products, ~1e-5 relative per op), or the decode GEMV (exact integer
 * weights, fp32 scales, f16 hi + lo activations) where it serves the row
 * count. For chains of many layers whose end result must stay within the
 * FAST tolerance of the reference: single-f16 weights and activations
 * compound to several 1e-3 over 28 layers. */
#define B2M_MODE_PRECISE 2

#define B2M_MAX_RANK 8

typedef struct b2m_ctx b2m_ctx;
typedef struct b2m_tensor b2m_tensor;
typedef struct b2m_weight b2m_weight;

/* ---- library / context ------------------------------------------------ */

/* ABI version of the loaded library (B2M_ABI_VERSION it was built with). */
B2M_API int32_t b2m_abi_version(void);

/* Message for the last failing call on this thread ("" if none). Replaces
 * the ORT status-message read (ort_backend.dart:774-782). */
B2M_API const char *b2m_last_error(void);

/* Number of visible CUDA devices. */
B2M_API b2m_status b2m_device_count(int32_t *count);

/* Opens a context on `device` (a CUDA ordinal). The context owns a
 * non-blocking stream, a stream-ordered memory pool and scratch space.
 * Replaces the session-level resource setup of OrtRuntime.load /
 * OrtNativeSession._create (ort_backend.dart:83-111, 171-448). */
B2M_API b2m_status b2m_init(int32_t device, b2m_ctx **out_ctx);

/* Waits for outstanding work and frees the context. Tensors and weights made
 * on the context must be freed first. */
B2M_API b2m_status b2m_shutdown(b2m_ctx *ctx);

/* Enqueue subsequent work on `stream` (a cudaStream_t of the context's
 * device); NULL selects the context's own stream again. */
B2M_API b2m_status b2m_set_stream(b2m_ctx *ctx, void *stream);

/* Blocks until all work enqueued on the current stream has finished. */
B2M_API b2m_status b2m_synchronize(b2m_ctx *ctx);

/* Execution control, mirroring OnnxExecutionControl
 * (lib/src/execution_control.dart:29-77): a host flag polled before every
 * launch (non-zero -> B2M_ERR_CANCELLED, like checkpoint()), and a byte
 * budget for library-allocated outputs (like checkAdditionalBytes;
 * <= 0 disables). */
B2M_API b2m_status b2m_set_cancel_flag(b2m_ctx *ctx, const volatile int32_t *flag);
B2M_API b2m_status b2m_set_byte_budget(b2m_ctx *ctx, int64_t bytes);

/* Numerics of the attention entry points (b2m_gqa_dev, b2m_mha_dev) on this
 * context. FAST (default): tcgen05 kernels with bf16-split products where the
 * shape allows, and key splits for decode steps of few sequences. EXACT:
 * fp32 CUDA-core kernels and no key splits, so a sequence's result does not
 * depend on the other sequences of the batch — the property the reference's
 * pool guarantees for its partitioned MatMuls (parallel_pool.dart:7-8). */
B2M_API b2m_status b2m_set_attention_mode(b2m_ctx *ctx, int32_t mode);

/* Device time of the last op, from CUDA events around its launches, when
 * timing is on (default off; enabling costs one event pair per op). Replaces
 * the per-node Stopwatch of ExecutionProfile (onnx_graph.dart:1246-1248). */
B2M_API b2m_status b2m_enable_timing(b2m_ctx *ctx, int32_t on);
B2M_API b2m_status b2m_last_kernel_ms(b2m_ctx *ctx, float *ms);

/* ---- tensors (device-resident values; replace Tensor's typed lists,
 *      lib/src/tensor.dart:16-30, for GPU operands) ----------------------- */

B2M_API b2m_status b2m_tensor_alloc(b2m_ctx *ctx, int32_t dtype, const int64_t *shape, int32_t rank,
                                    b2m_tensor **out);
/* Borrows caller-owned device memory (not freed by b2m_tensor_free). */
B2M_API b2m_status b2m_tensor_wrap(b2m_ctx *ctx, void *device_ptr, int32_t dtype, const int64_t *shape,
                                   int32_t rank, b2m_tensor **out);
/* Host <-> device copies of the whole tensor; `bytes` must equal its size.
 * Both return after the copy has completed. */
B2M_API b2m_status b2m_tensor_upload(b2m_ctx *ctx, b2m_tensor *t, const void *host, int64_t bytes);
B2M_API b2m_status b2m_tensor_download(b2m_ctx *ctx, const b2m_tensor *t, void *host, int64_t bytes);
B2M_API b2m_status b2m_tensor_free(b2m_tensor *t);

/* Page-locked host buffers (no counterpart in the reference, whose FFI buffers
 * come from package:ffi's malloc). Staging a host-buffer call's A and Y here
 * lets b2m_matmul_nbits_host's decode GEMV store Y straight into host memory
 * (no device-to-host copy) and makes the copy of A a direct DMA. bytes >= 0;
 * free with b2m_host_free. */
B2M_API b2m_status b2m_host_alloc(b2m_ctx *ctx, int64_t bytes, void **out);
B2M_API b2m_status b2m_host_free(b2m_ctx *ctx, void *p);
/* dtype, rank, shape (B2M_MAX_RANK entries) and device pointer of `t`. */
B2M_API b2m_status b2m_tensor_info(const b2m_tensor *t, int32_t *dtype, int32_t *rank, int64_t *shape,
                                   void **device_ptr);

/* ---- weight prepack (session load) ------------------------------------- */

/* fp32 MatMul / Gemm initializer B. `rows x cols` host row-major; with
 * trans != 0 the stored matrix is B^T (Gemm transB=1) and is transposed once
 * here, as the reference caches opTranspose(B) per initializer
 * (onnx_graph.dart:102-105, 2159-2161). The packed weight is logically
 * [K, N]. */
B2M_API b2m_status b2m_weight_prepack_f32(b2m_ctx *ctx, const float *host_b, int64_t rows, int64_t cols,
                                          int32_t trans, b2m_weight **out);

/* int8 / uint8 MatMulInteger / QLinearMatMul initializer B[K, N]
 * (dtype B2M_INT8 or B2M_UINT8), stored K-major with per-column sums for the
 * zero-point correction. */
B2M_API b2m_status b2m_weight_prepack_i8(b2m_ctx *ctx, const void *host_b, int32_t dtype, int64_t k,
                                         int64_t n, b2m_weight **out);

/* MatMulNBits initializers: b_q uint8[N, ceil(K/block)/1, block/2] (low
 * nibble first), scales float[N * nblocks], zero points either packed uint4
 * uint8[N * ceil(nblocks/2)] (zp_dtype B2M_UINT8), float[N * nblocks]
 * (B2M_FLOAT) or absent (zero_points NULL, zp_dtype 0; zero point 8).
 * Validation mirrors opMatMulNBits (onnx_qlinear_ops.dart:126-166):
 * bits != 4 -> UNSUPPORTED; K, N <= 0 or block not a power of two >= 16
 * -> INVALID_ARGUMENT. */
B2M_API b2m_status b2m_weight_prepack_nbits(b2m_ctx *ctx, const uint8_t *b_q, const float *scales,
                                            const void *zero_points, int32_t zp_dtype, int64_t k,
                                            int64_t n, int32_t bits, int32_t block_size,
                                            b2m_weight **out);
B2M_API b2m_status b2m_weight_free(b2m_weight *w);

/* Declares `next` (a MatMulNBits weight of the same context, or NULL to
 * clear) as the weight of the call that follows each MatMulNBits call of `w`
 * in the caller's op order — the next projection of a decoder layer, the
 * first of the next layer. Kernels running `w` then prefetch the part of
 * `next` its call will read into L2, so that call's weight prologue (which
 * runs under programmatic dependent launch while `w`'s call finishes) reads
 * L2 instead of HBM. A hint: results do not change. Freeing either weight
 * drops the link; a CUDA graph captured with the link keeps prefetching
 * `next`, so free `next` only after such graphs. No counterpart in the
 * reference, whose kernels run on the host. */
B2M_API b2m_status b2m_weight_set_next(b2m_weight *w, const b2m_weight *next);

/* ---- operators --------------------------------------------------------- */

/* MatMul (opMatMul, onnx_ops.dart:1710-1766): numpy-broadcast batched
 * A[..., M, K] . B[..., K, N]. Exactly one of `b` (device tensor) and
 * `b_packed` (from b2m_weight_prepack_f32) is non-NULL. mode EXACT is
 * bitwise identical to the reference's matmulKernel. */
B2M_API b2m_status b2m_matmul_f32(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                  const b2m_weight *b_packed, int32_t mode, b2m_tensor **y);

/* Gemm (opGemm, onnx_ops.dart:2152-2173): alpha * A' . B' + beta * C with
 * 2-D A, B; C (optional) broadcasts onto [M, N]. With `b_packed` the
 * transpose was applied at prepack and trans_b must be 0. */
B2M_API b2m_status b2m_gemm_f32(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                const b2m_weight *b_packed, const b2m_tensor *c, float alpha, float beta,
                                int32_t trans_a, int32_t trans_b, int32_t mode, b2m_tensor **y);

/* MatMulInteger (opMatMulInteger, onnx_qlinear_ops.dart:32-81):
 * Y int32 = (A - a_zp)(B - b_zp), A uint8/int8 [..., M, K], B uint8/int8
 * [..., K, N] or prepacked. Zero points: NULL, scalar, per-row [M] (A) or
 * per-column [N] (B), same dtype as their operand. Batches must match or be
 * 1. Exact (the reference accumulates in int64; values outside int32 need
 * K > 33025 and are rejected as UNSUPPORTED). */
B2M_API b2m_status b2m_matmul_integer(b2m_ctx *ctx, const b2m_tensor *a, const b2m_tensor *b,
                                      const b2m_weight *b_packed, const b2m_tensor *a_zp,
                                      const b2m_tensor *b_zp, b2m_tensor **y);

/* QLinearMatMul (opQLinearMatMul, onnx_qlinear_ops.dart:85-108):
 * per-tensor scales (host floats), zero-point tensors as above, y_zp scalar
 * (NULL = 0); output dtype of y is uint8 if lo == 0, int8 if lo == -128
 * (the reference picks lo/hi from y_zp's dtype, onnx_graph.dart:2903). */
B2M_API b2m_status b2m_qlinear_matmul(b2m_ctx *ctx, const b2m_tensor *a, float a_scale,
                                      const b2m_tensor *a_zp, const b2m_tensor *b,
                                      const b2m_weight *b_packed, float b_scale, const b2m_tensor *b_zp,
                                      float y_scale, int32_t y_zp, int32_t lo, int32_t hi,
                                      b2m_tensor **y);

/* MatMulNBits (opMatMulNBits, onnx_qlinear_ops.dart:115-228):
 * Y[..., N] = A[..., K] . dequant(W)^T + bias, A float32, W from
 * b2m_weight_prepack_nbits, bias float[N] or NULL. mode EXACT reproduces the
 * reference bit for bit (double accumulation for one row, float32 tiles
 * otherwise); FAST uses f16 tensor-core MMA with fp32 accumulation. */
B2M_API b2m_status b2m_matmul_nbits(b2m_ctx *ctx, const b2m_tensor *a, const b2m_weight *w,
                                    const b2m_tensor *bias, int32_t mode, b2m_tensor **y);

/* Host-buffer convenience for callers without device tensors: copies A
 * (m rows of K floats) and bias (N floats or NULL) to the device, runs
 * b2m_matmul_nbits, copies Y (m x N floats) back, and returns when Y is in
 * host memory. */
B2M_API b2m_status b2m_matmul_nbits_host(b2m_ctx *ctx, const float *a_host, int64_t m,
                                         const b2m_weight *w, const float *bias_host, int32_t mode,
                                         float *y_host);

/* Raw device-pointer form of b2m_matmul_nbits for callers that manage their
 * own device memory (a: m x K floats, bias: N floats or NULL, y: m x N
 * floats), enqueued on the current stream. */
B2M_API b2m_status b2m_matmul_nbits_dev(b2m_ctx *ctx, const float *a, int64_t m, const b2m_weight *w,
                                        const float *bias, int32_t mode, float *y);

/* Which kernels b2m_matmul_nbits_dev runs for an m-row call of `w` in
 * `mode`: B2M_ROUTE_GEMV (the decode GEMV, fp32 activations read as they
 * are), B2M_ROUTE_TC_F16 (the tensor-core GEMM, which first rounds the
 * activations to f16; b2m_matmul_nbits_f16_dev takes them already rounded)
 * or B2M_ROUTE_OTHER. No counterpart in the reference: a chain driver uses it
 * to have each projection's producer write the f16 operand. */
#define B2M_ROUTE_GEMV 0
#define B2M_ROUTE_TC_F16 1
#define B2M_ROUTE_OTHER 2
B2M_API b2m_status b2m_matmul_nbits_route(b2m_ctx *ctx, const b2m_weight *w, int64_t m, int32_t mode,
                                          int32_t *route);

/* FAST MatMulNBits on activations already rounded to f16 by their producer:
 * a16 holds m rows of K f16 values (K % 8 == 0), round to nearest of the fp32
 * activations, as b2m_rmsnorm_f16_dev and b2m_silu_mul_f16_dev write them. The
 * result is bit for bit that of b2m_matmul_nbits_dev in FAST mode on the fp32
 * rows; the call is accepted only where that call's route is
 * B2M_ROUTE_TC_F16 (otherwise B2M_ERR_UNSUPPORTED). Saves the conversion
 * launch in front of the GEMM. */
B2M_API b2m_status b2m_matmul_nbits_f16_dev(b2m_ctx *ctx, const uint16_t *a16, int64_t m, const b2m_weight *w,
                                            const float *bias, float *y);

/* The SwiGLU front half of an MLP in one call: the gate and up MatMulNBits
 * of a layer (one weight of N = 2I output rows) followed by silu(gate) * up,
 * the Sigmoid / Mul / Mul nodes between them and the down MatMulNBits
 * (lib/src/onnx_qlinear_ops.dart:115-228 for each MatMulNBits, then the
 * elementwise nodes). The weight's rows are TILE-INTERLEAVED: for t in
 * [0, I/64) its rows 128t .. 128t+63 are the gate rows 64t .. 64t+63 and rows
 * 128t+64 .. 128t+127 the matching up rows (N % 128 == 0). act: [m][I] fp32
 * and / or act16: the same rounded to f16 (the operand of
 * b2m_matmul_nbits_f16_dev for the down projection); either may be NULL,
 * both 16-byte aligned. a: the fp32 activations [m][K]; a16: NULL or their
 * f16 copy (as b2m_rmsnorm_f16_dev writes it), used where the call's route
 * is B2M_ROUTE_TC_F16, where the tensor-core GEMM forms the products in its
 * epilogue (no fp32 gate / up rows in memory). On other routes a is required
 * and the result is b2m_matmul_nbits_dev followed by the elementwise pass.
 * Results are bit for bit those of b2m_matmul_nbits_dev on the same weight
 * (mode as given) followed by b2m_silu_mul_dev / b2m_silu_mul_f16_dev on the
 * gate and up columns. */
B2M_API b2m_status b2m_matmul_nbits_swiglu_dev(b2m_ctx *ctx, const float *a, const uint16_t *a16, int64_t m,
                                               const b2m_weight *w, int32_t mode, float *act, uint16_t *act16);

/* Allocation-free MatMulNBits. No counterpart in the reference: this entry
 * point exists for callers that must not allocate device memory while they
 * run an operator — a host application that has handed all device memory to
 * its own pool, or an inference loop that must not risk an out-of-memory
 * failure or the device-wide synchronisation cudaMalloc/cudaFree can cause.
 * It runs the same tensor-core kernels as b2m_matmul_nbits (FAST numerics)
 * on caller-owned device buffers (a: m x K floats, bias: N floats or NULL,
 * y: m x N floats) and the prepacked weight `w`, on `stream` (a cudaStream_t
 * of w's device; NULL = legacy default stream), and returns after Y is
 * complete. Its only working memory is a fixed file-scope device array of
 * B2M_NOALLOC_SCRATCH_BYTES (+256) bytes that every device loading the library
 * holds until the process exits; calls needing more (m * roundup(K, 8) * 2
 * bytes) fail with B2M_ERR_INVALID_ARGUMENT. The array is shared by all calls
 * on a device and keeps the last call's contents, so calls that overlap on
 * the GPU race; serialise them (one stream, or host-side ordering). The first
 * call on a device resolves the array's device address
 * (cudaGetSymbolAddress), so make that first call before any stream capture.
 * That address is kept for the life of the process: a cudaDeviceReset after
 * the first call is not supported. Every call copies the kernels' error word
 * back and synchronises `stream`, so it blocks the host until the stream has
 * drained (two calls cannot be queued back to back). */
#define B2M_NOALLOC_SCRATCH_BYTES (8u << 20)
B2M_API b2m_status b2m_matmul_nbits_noalloc(const b2m_weight *w, const float *a, int64_t m, const float *bias,
                                            float *y, void *stream);

/* ------------------------------------------------------------------------
 * Device-resident glue for the transformer chains (configs 4 and 5), so that
 * a chain of MatMuls never round-trips through host memory. All pointers are
 * device memory of the context's device; the ops are enqueued on the current
 * stream and return at once. Rows are contiguous (row length = d).
 * ---------------------------------------------------------------------- */

/* RMSNorm over the last axis: s = x (+ skip when non-NULL; s is stored to
 * sum_out when non-NULL), y = s * gamma / sqrt(mean(s^2) + eps), statistics in
 * double. Replaces opRMSNorm (lib/src/onnx_ops.dart:1771) and the fused
 * SkipSimplifiedLayerNormalization (lib/src/onnx_graph.dart:1793). */
B2M_API b2m_status b2m_rmsnorm_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma, float *y,
                                   float *sum_out, int64_t rows, int64_t d, double eps);

/* b2m_rmsnorm_dev that also writes y as f16 (round to nearest) into y16
 * (rows x d, d % 8 == 0): the operand of b2m_matmul_nbits_f16_dev. y may be
 * NULL when only the f16 rows are consumed (16-byte aligned operands; other
 * layouts need y). */
B2M_API b2m_status b2m_rmsnorm_f16_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma, float *y,
                                       float *sum_out, uint16_t *y16, int64_t rows, int64_t d, double eps);

/* RMSNorm of every head vector of [tokens][heads x head_dim] rows placed
 * token_stride floats apart (per-head q / k norms read from a packed
 * projection output; y may alias x, with the same layout). */
B2M_API b2m_status b2m_rmsnorm_heads_dev(b2m_ctx *ctx, const float *x, const float *gamma, float *y, int64_t tokens,
                                         int64_t heads, int64_t head_dim, int64_t token_stride, double eps);

/* b2m_rmsnorm_heads_dev with a gain row per head: head h of every token uses
 * gamma_rows[h * head_dim ...]. Lets the per-head q and k norms of one packed
 * q|k|v projection (different gains) run as one launch. */
B2M_API b2m_status b2m_rmsnorm_head_rows_dev(b2m_ctx *ctx, const float *x, const float *gamma_rows, float *y,
                                             int64_t tokens, int64_t heads, int64_t head_dim, int64_t token_stride,
                                             double eps);

/* LayerNormalization over the last axis (mean / variance in double), with an
 * optional residual as above; beta may be NULL. Replaces
 * opLayerNormalization (lib/src/onnx_ops.dart:1666). */
B2M_API b2m_status b2m_layernorm_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma,
                                     const float *beta, float *y, float *sum_out, int64_t rows, int64_t d,
                                     double eps);

/* b2m_layernorm_dev that also writes y as the bf16 hi / lo planes of the
 * FAST fp32 Gemm's A operand into y_planes (rows x d hi values, then rows x d
 * lo values; d % 64 == 0): the operand of b2m_gemm_f32_split_dev. */
B2M_API b2m_status b2m_layernorm_split_dev(b2m_ctx *ctx, const float *x, const float *skip, const float *gamma,
                                           const float *beta, float *y, float *sum_out, uint16_t *y_planes,
                                           int64_t rows, int64_t d, double eps);

/* y[r][c] = silu(gate[r*gate_rs + c]) * up[r*up_rs + c] for c < d (the
 * Sigmoid/Mul pair of a SwiGLU MLP; gate and up may be the two halves of one
 * packed projection). */
B2M_API b2m_status b2m_silu_mul_dev(b2m_ctx *ctx, const float *gate, const float *up, int64_t gate_rs,
                                    int64_t up_rs, float *y, int64_t rows, int64_t d);

/* b2m_silu_mul_dev that also writes y as f16 (round to nearest) into y16
 * (rows x d, d % 8 == 0). */
B2M_API b2m_status b2m_silu_mul_f16_dev(b2m_ctx *ctx, const float *gate, const float *up, int64_t gate_rs,
                                        int64_t up_rs, float *y, uint16_t *y16, int64_t rows, int64_t d);

/* erf GELU, y = 0.5 x (1 + erf(x / sqrt 2)) (opGelu, lib/src/onnx_ops.dart:706). */
B2M_API b2m_status b2m_gelu_dev(b2m_ctx *ctx, const float *x, float *y, int64_t n);

/* erf GELU of rows x d values (d % 64 == 0) written as the bf16 hi / lo planes
 * of a FAST Gemm's A operand (layout as b2m_layernorm_split_dev), and to y
 * when y is not NULL; 16-byte aligned pointers. */
B2M_API b2m_status b2m_gelu_split_dev(b2m_ctx *ctx, const float *x, float *y, uint16_t *y_planes, int64_t rows,
                                      int64_t d);

/* FAST Gemm y = A . B + bias (B prepacked by b2m_weight_prepack_f32, bias N
 * floats or NULL) with A given as its bf16 hi / lo planes, as the _split_dev
 * producers write them (m x roundup(K, 64) hi values, then as many lo values):
 * bit for bit b2m_gemm_f32 in FAST mode (alpha = beta = 1, C = bias) on the
 * fp32 rows, without the split pass in front of the GEMM. No counterpart in
 * the reference (its Gemm reads fp32 rows, onnx_ops.dart:2152). */
B2M_API b2m_status b2m_gemm_f32_split_dev(b2m_ctx *ctx, const uint16_t *a_planes, int64_t m, const b2m_weight *w,
                                          const float *bias, float *y);

/* y = a + b over rows x d; with b_broadcast, b is one row of d added to every
 * row (bias). */
B2M_API b2m_status b2m_add_dev(b2m_ctx *ctx, const float *a, const float *b, float *y, int64_t rows, int64_t d,
                               int32_t b_broadcast);

/* y[r][:] = table[ids[r]][:] (Gather of embedding rows; ids int64 in [0, v)). */
B2M_API b2m_status b2m_gather_rows_dev(b2m_ctx *ctx, const float *table, const int64_t *ids, float *y,
                                       int64_t rows, int64_t v, int64_t d);

/* out[r] = argmax over the v entries of row r (first maximum wins; int64),
 * as opArgMinMax with keepdims over the last axis. */
B2M_API b2m_status b2m_argmax_dev(b2m_ctx *ctx, const float *x, int64_t *out, int64_t rows, int64_t v);

/* GroupQueryAttention (lib/src/onnx_ops.dart:1844) over a caller-owned KV
 * cache. q: [b][s] rows of h*head_dim floats (row stride q_rs), k / v: [b][s]
 * rows of kvh*head_dim (row stride kv_rs). k_cache / v_cache:
 * [b][kvh][cap][head_dim]. past[b] (int32, device memory) is the number of
 * positions already cached for sequence b: this call writes its keys/values
 * at past[b] .. past[b]+s-1 (rotary applied to K) and attends causally over
 * [0, past[b] + i] for query i. cos / sin: [max_pos][rotary_half] caches or
 * NULL (no rotary); rotary_dim <= head_dim, interleaved as the attribute.
 * Scale <= 0 means 1/sqrt(head_dim). out: [b][s] rows of h*head_dim.
 * head_dim <= 256, h a multiple of kvh. Reading `past` from device memory
 * lets a decode step replay as a CUDA graph. */
B2M_API b2m_status b2m_gqa_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                               int64_t kv_rs, float *k_cache, float *v_cache, const int32_t *past,
                               const float *cos_cache, const float *sin_cache, int32_t rotary_half,
                               int32_t rotary_dim, int32_t interleaved, float *out, int32_t b, int32_t s, int32_t h,
                               int32_t kvh, int32_t head_dim, int32_t cap, float scale);

/* b2m_gqa_dev that also writes the attention output as f16 (round to
 * nearest) into out16 ([b*s][h*head_dim], h*head_dim % 8 == 0): the operand of
 * b2m_matmul_nbits_f16_dev for the output projection. out may be NULL when
 * only the f16 copy is consumed: the decode and flash prefill kernels then
 * skip the fp32 rows, other kernels write them to scratch. */
B2M_API b2m_status b2m_gqa_f16_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                                   int64_t kv_rs, float *k_cache, float *v_cache, const int32_t *past,
                                   const float *cos_cache, const float *sin_cache, int32_t rotary_half,
                                   int32_t rotary_dim, int32_t interleaved, float *out, uint16_t *out16, int32_t b,
                                   int32_t s, int32_t h, int32_t kvh, int32_t head_dim, int32_t cap, float scale);

/* b2m_gqa_dev preceded by the per-head RMSNorm of q and k (the q_norm /
 * k_norm SimplifiedLayerNormalization nodes of a Qwen3 layer, each head of
 * head_dim values normalised with its gain row): qk_gain is [h + kvh][head_dim],
 * the gain rows of the h query heads, then those of the kvh key heads; eps the
 * norm's epsilon. out16: NULL, or the f16 copy of out as b2m_gqa_f16_dev
 * writes it (with out16 given, out may be NULL as there). Results equal b2m_rmsnorm_head_rows_dev on q and k followed by
 * b2m_gqa_dev / b2m_gqa_f16_dev. A single-token call (s == 1) normalises
 * inside the decode attention kernel, which also appends the token's key and
 * value (one launch); other calls normalise q and k IN PLACE first, so both
 * buffers may hold their normalised values afterwards. */
B2M_API b2m_status b2m_gqa_qknorm_dev(b2m_ctx *ctx, float *q, float *k, const float *v, int64_t q_rs, int64_t kv_rs,
                                      const float *qk_gain, double eps, float *k_cache, float *v_cache,
                                      const int32_t *past, const float *cos_cache, const float *sin_cache,
                                      int32_t rotary_half, int32_t rotary_dim, int32_t interleaved, float *out,
                                      uint16_t *out16, int32_t b, int32_t s, int32_t h, int32_t kvh, int32_t head_dim,
                                      int32_t cap, float scale);

/* MultiHeadAttention over projected rows (opMultiHeadAttention,
 * lib/src/onnx_ops.dart:2019; the scale + mask + softmax between the two
 * batched MatMuls of opFusedSDPA, :2106-2148). q: [b][s] rows of h*head_dim
 * (row stride q_rs); k / v: [b][t] rows of kvh*head_dim (row stride kv_rs),
 * h a multiple of kvh (query head i reads kv head i / (h / kvh)).
 * mask: NULL or an additive bias on the scaled scores, the element for
 * (batch r, query head i, query row p, key j) at
 * mask[r*mask_bs + i*mask_hs + p*mask_qs + j]; zero strides broadcast. A
 * BERT-style key-padding mask [b][t] is (t, 0, 0); the reference's
 * attention_bias [b][bias_heads][s][t] is (bias_heads*s*t, bias_heads == 1 ?
 * 0 : s*t, t). causal != 0 additionally hides keys j > p. Scale <= 0 means
 * 1/sqrt(head_dim). out: [b][s] rows of h*head_dim. head_dim <= 256. */
B2M_API b2m_status b2m_mha_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                               int64_t kv_rs, const float *mask, int64_t mask_bs, int64_t mask_hs, int64_t mask_qs,
                               float *out, int32_t b, int32_t s, int32_t t, int32_t h, int32_t kvh, int32_t head_dim,
                               float scale, int32_t causal);

/* b2m_mha_dev that also writes the attention output as the bf16 hi / lo
 * planes of a FAST Gemm's A operand into out_planes ([b*s][h*head_dim] hi
 * values, then as many lo values; h*head_dim % 64 == 0): the operand of
 * b2m_gemm_f32_split_dev for the output projection. */
B2M_API b2m_status b2m_mha_split_dev(b2m_ctx *ctx, const float *q, const float *k, const float *v, int64_t q_rs,
                                     int64_t kv_rs, const float *mask, int64_t mask_bs, int64_t mask_hs,
                                     int64_t mask_qs, float *out, uint16_t *out_planes, int32_t b, int32_t s,
                                     int32_t t, int32_t h, int32_t kvh, int32_t head_dim, float scale,
                                     int32_t causal);

/* DynamicQuantizeLinear (opDynamicQuantizeLinear, lib/src/onnx_ops.dart:3556):
 * uint8 y[n] from float x[n] with the range's scale (float, written to
 * *scale) and zero point (uint8, *zero_point), all device memory, bit-exact
 * with the reference (scale and zero point in double then float32, round
 * half to even). y / scale / zero_point feed b2m_matmul_integer directly. */
B2M_API b2m_status b2m_dynamic_quantize_linear_dev(b2m_ctx *ctx, const float *x, int64_t n, uint8_t *y,
                                                   float *scale, uint8_t *zero_point);

/* RotaryEmbedding (opRotaryEmbedding, lib/src/onnx_ops.dart:2659-2717) over
 * [b][s] rows of heads*head_dim floats (row strides x_rs / y_rs; y may be x).
 * positions: int64 ids [b][s], or [s] shared by the batch when
 * pos_per_batch is 0; cos_cache / sin_cache: [max_pos][half]. The first
 * rotary_dim (even, <= 2*half) values of each head rotate, GPT-NeoX
 * rotate-half or, with interleaved, GPT-J pairs; the rest pass through.
 * head_dim <= 256. A position outside [0, max_pos) is a device error. */
B2M_API b2m_status b2m_rotary_dev(b2m_ctx *ctx, const float *x, int64_t x_rs, const int64_t *positions,
                                  int32_t pos_per_batch, const float *cos_cache, const float *sin_cache,
                                  int32_t half, int32_t max_pos, float *y, int64_t y_rs, int32_t b, int32_t s,
                                  int32_t heads, int32_t head_dim, int32_t rotary_dim, int32_t interleaved);

/* past[i] += delta for i < n (int32 device counters of a decode loop). */
B2M_API b2m_status b2m_advance_positions_dev(b2m_ctx *ctx, int32_t *past, int32_t n, int32_t delta);

/* ---- convolutions through the GEMM cores --------------------------------
 * The reference's other matmulKernel callers: opConv
 * (lib/src/onnx_nn_ops.dart:179-545; dispatch lib/src/onnx_graph.dart:2436-2490)
 * and the integer convolutions opConvInteger / opQLinearConv
 * (lib/src/onnx_qlinear_ops.dart:230-382; dispatch onnx_graph.dart:2889-2901,
 * 2935-2956). Each runs as an im2col panel on the device feeding the fp32 or
 * int8 GEMM kernels above; outputs are NC[D]HW. */

/* auto_pad attribute values (the attribute's strings, _resolvePads
 * onnx_nn_ops.dart:38-88). */
#define B2M_AUTO_PAD_NOTSET 0
#define B2M_AUTO_PAD_SAME_UPPER 1
#define B2M_AUTO_PAD_SAME_LOWER 2
#define B2M_AUTO_PAD_VALID 3

/* Conv / ConvInteger / QLinearConv weight [m][C/group][kernel...] (host,
 * row-major, viewed as m rows of k = C/group * kernel volume) packed as the
 * GEMM operand: dtype B2M_FLOAT -> an fp32 weight holding W^T [k][m] (the
 * layout b2m_weight_prepack_f32 makes with trans = 1); B2M_UINT8 / B2M_INT8
 * -> an int8 weight holding W^T with k zero-padded to a multiple of 16 (so
 * the tensor-core path takes it). Replaces the per-call weight reads of the
 * reference's convolutions. */
B2M_API b2m_status b2m_weight_prepack_conv(b2m_ctx *ctx, const void *host_w, int32_t dtype, int64_t m, int64_t k,
                                           b2m_weight **out);

/* Conv (opConv): x float [n][C][spatial...] with 1-3 spatial dims, w from
 * b2m_weight_prepack_conv (B2M_FLOAT), kernel_shape[nd] (the weight's spatial
 * dims), strides[nd] / dilations[nd] or NULL (all 1), pads[2 nd]
 * (begin..., end...) or NULL (all 0; ignored unless auto_pad is NOTSET),
 * group >= 1, bias float[m] or NULL. y: [n][m][out spatial...].
 * mode EXACT reproduces the reference's arithmetic: the im2col panel times
 * matmulKernel's per-element k order (double tails for fewer than four
 * outputs per group), the bias added in float32 afterwards; depthwise 1-D /
 * 2-D and every 3-D conv accumulate in double from the bias. The reference
 * switches to Winograd F(2x2, 3x3) for initializer 3x3 stride-1 group-1
 * convs with >= 1024 output pixels; EXACT follows the im2col arithmetic
 * there, which the Winograd path only matches within rounding.
 * mode FAST runs the im2col panel as bf16 split planes through the tcgen05
 * FAST GEMM (tolerance contract; depthwise and 3-D as in EXACT). */
B2M_API b2m_status b2m_conv_f32(b2m_ctx *ctx, const b2m_tensor *x, const b2m_weight *w, const b2m_tensor *bias,
                                const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads,
                                const int64_t *dilations, int32_t group, int32_t auto_pad, int32_t mode,
                                b2m_tensor **y);

/* ConvInteger (opConvInteger): x uint8 / int8 [n][C][W] or [n][C][H][W]
 * (1-D or 2-D, as the reference), x_zp (first element used) or NULL, w from
 * b2m_weight_prepack_conv (int8 kinds), w_zp NULL, scalar or per output
 * channel [m] (else UNSUPPORTED, :322-326), same dtype as the weight. No
 * auto_pad (the dispatch passes none). y int32 [n][m][out...], exact. */
B2M_API b2m_status b2m_conv_integer(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *x_zp, const b2m_weight *w,
                                    const b2m_tensor *w_zp, const int64_t *kernel_shape, const int64_t *strides,
                                    const int64_t *pads, const int64_t *dilations, int32_t group, b2m_tensor **y);

/* QLinearConv (opQLinearConv), 2-D: ConvInteger's accumulator, then per
 * output channel q = roundEven((acc + bias) * (x_scale * w_scale[c] /
 * y_scale)) + y_zp in double, clamped to [lo, hi] (0..255 -> uint8 y,
 * -128..127 -> int8 y; the reference picks them from y_zp's dtype,
 * onnx_graph.dart:2936). w_scale: float device tensor of 1 or m values;
 * bias int32 [m] or NULL. No host buffer is read after the call returns. */
B2M_API b2m_status b2m_qlinear_conv(b2m_ctx *ctx, const b2m_tensor *x, float x_scale, const b2m_tensor *x_zp,
                                    const b2m_weight *w, const b2m_tensor *w_scale,
                                    const b2m_tensor *w_zp, float y_scale, int32_t y_zp, const b2m_tensor *bias,
                                    const int64_t *kernel_shape, const int64_t *strides, const int64_t *pads,
                                    const int64_t *dilations, int32_t group, int32_t lo, int32_t hi, b2m_tensor **y);

/* ConvTranspose (opConvTranspose, lib/src/onnx_nn_ops.dart:815-1060; dispatch
 * onnx_graph.dart:2491-2515): x float [n][C][spatial...] (1-3 spatial dims),
 * w float [C][M/group][kernel...] (a device tensor, read as is), bias
 * float[M] or NULL; strides / dilations / output_padding [nd] or NULL
 * (1 / 1 / 0), pads [2 nd] or NULL, output_shape [nd] (the spatial dims) or
 * NULL. y: [n][M][out...]. The reference's arithmetic in every call: for one
 * image of 1-D / 2-D without output_shape, the exact GEMM W_g^T . X_g (the
 * matmulKernel rule) and an overlap-add in float32; otherwise its scatter,
 * each non-zero input adding x * w in double onto the float32 output, in
 * the reference's order; then the bias in float32. */
B2M_API b2m_status b2m_conv_transpose_f32(b2m_ctx *ctx, const b2m_tensor *x, const b2m_tensor *w,
                                          const b2m_tensor *bias, const int64_t *strides, const int64_t *pads,
                                          const int64_t *dilations, const int64_t *output_padding,
                                          const int64_t *output_shape, int32_t group, b2m_tensor **y);

/* Serialises a packed weight (its device layouts, as prepacked) into buf, for
 * an on-disk prepack cache: *needed receives the byte size; with buf NULL
 * only the size is returned. The blob is tied to this library's
 * B2M_ABI_VERSION. */
B2M_API b2m_status b2m_weight_export(const b2m_weight *w, void *buf, size_t capacity, size_t *needed);

/* Recreates a packed weight on ctx's device from a b2m_weight_export blob,
 * without redoing the host-side layout work. UNSUPPORTED for a blob of
 * another library version, INVALID_ARGUMENT for a malformed one. */
B2M_API b2m_status b2m_weight_import(b2m_ctx *ctx, const void *buf, size_t size, b2m_weight **out);

/* Shape of a packed weight: K and N (logical B is [K, N]). */
B2M_API b2m_status b2m_weight_info(const b2m_weight *w, int64_t *k, int64_t *n);

#ifdef __cplusplus
}
#endif

#endif /* B2M_H_ */
