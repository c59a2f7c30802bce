/*
 * xe_b200.h — C ABI of the B200 (sm_100a) kernels behind extended_einsum's
 * stable-materialization hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * and a CUDA stream passed as `void*` (a `cudaStream_t`; NULL = legacy default
 * stream).  Nothing here allocates device memory: outputs and scratch buffers
 * are allocated by the caller.  All calls are stream-ordered and asynchronous;
 * a non-OK status means nothing was launched (argument errors) or the launch
 * itself failed.  Device-side waits are bounded: a wait that runs out records
 * a code that xe_device_status() reports.
 *
 * Status codes map onto the exceptions the reference raises on this path:
 *   XE_ERR_INVALID_ARGUMENT -> ValueError          (backend_translation/runtime.py:13-14)
 *   XE_ERR_NOT_SUPPORTED    -> NotImplementedError (backend_translation/translate.py:41, 585, 810)
 *   XE_ERR_CUDA, XE_ERR_DEVICE_TIMEOUT -> RuntimeError
 *
 * Reference paths below are relative to the extended_einsum project root.
 */
#ifndef XE_B200_H
#define XE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  XE_OK = 0,
  XE_ERR_INVALID_ARGUMENT = 1,
  XE_ERR_NOT_SUPPORTED = 2,
  XE_ERR_CUDA = 3,
  XE_ERR_DEVICE_TIMEOUT = 4
} xe_status;

/* Which per-operand shift the log-space lowering uses
 * (translate.py:698: max for logspace_max, min for logspace_min). */
typedef enum { XE_SHIFT_MAX = 0, XE_SHIFT_MIN = 1 } xe_shift_mode;

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int xe_version(void);

/* Human-readable message of the most recent failing call on this host thread. */
const char* xe_last_error_string(void);

/* Reads (and with `clear` != 0 resets) the device-side status word of the
 * current device: 0 when no bounded wait ran out since the last clear,
 * otherwise an XE_ERR_DEVICE_TIMEOUT-class code with the site in the low bits.
 * Synchronises the current device. */
int xe_device_status(int clear);

/* Limit of the kernels' ordinary bounded waits on the current device, in
 * nanoseconds (2 s by default; 0 restores the default).  Waits that guard the
 * release of resources when a CTA winds down keep the 2 s limit.  The value
 * lives in device memory and applies to every later launch on the device.
 * No counterpart in the reference, whose executor has no device waits: this
 * is the knob a caller (and the failure tests) uses to bound a stuck launch.
 * XE_ERR_INVALID_ARGUMENT for a limit below 1 us or above 60 s. */
xe_status xe_set_wait_timeout_ns(uint64_t ns);

/* Test kernel of the bounded waits, stream-ordered: one CTA whose first warp
 * waits on a barrier that expects one arrival.  complete != 0: a second warp
 * arrives after a short bounded delay and the wait ends normally.
 * complete == 0: nothing arrives, the wait runs out after the limit above, and
 * xe_device_status() then reports (XE_ERR_DEVICE_TIMEOUT << 16) | 17.
 * No counterpart in the reference (test infrastructure for the device status). */
xe_status xe_wait_probe(int complete, void* stream);

/* ------------------------------------------------------------------------ */
/* Log-space batched contraction (the GEMM-shaped stable einsum).
 *
 * Replaces the call sequence that _append_logspace_einsum
 * (backend_translation/translate.py:686-750) emits for a binary einsum whose
 * contracted labels appear in both operands:
 *   max/min over the contracted axis, stop_gradient, subtract, exp  (:727-740)
 *   einsum                                                          (:743)
 *   log, shift reduction + reshape + add per operand                (:744-749)
 * as executed by TorchBackendFunctions (backends/torch.py:37-118).
 *
 *   C[b,m,n] = log( sum_k  A'[b,m,k] * B'[b,k,n] ) (+ sA[b,m]) (+ sB[b,n])
 *
 * A log-domain operand X becomes X' = exp(X - sX) with sX its max (or min)
 * over k; a linear operand (a parameter-derived value, translate.py:723-725)
 * is used as is and adds no shift.  If `a2` is not NULL the A operand is the
 * log-domain sum a + a2 (a fused log-space Hadamard product,
 * translate.py:706-718), read with the strides of `a`.
 * Element (b,m,k) of A is a[b*a_sb + m*a_sm + k*a_sk]; B (b,k,n) and C (b,m,n)
 * likewise.  Arithmetic: fp32 in, split-TF32 (3 passes) tensor-core products,
 * fp32 accumulation, fp32 out.
 *
 * `workspace` must hold xe_logspace_gemm_workspace_size(...) bytes of device
 * memory (the shift vectors); it may be NULL when that size is 0.
 */
size_t xe_logspace_gemm_workspace_size(int64_t batch, int64_t m, int64_t n, int64_t k,
                                       int32_t a_linear, int32_t b_linear);

xe_status xe_logspace_gemm(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                           int32_t a_linear,
                           const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear,
                           float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                           int64_t batch, int64_t m, int64_t n, int64_t k, int32_t shift_mode,
                           void* workspace, size_t workspace_bytes, void* stream);

/* xe_logspace_gemm without a caller-provided workspace, for callers that
 * cannot allocate device memory: code running where cudaMalloc is not
 * permitted or not wanted (inside a stream-ordered region that must not
 * synchronise, a host without its own allocator, an embedding runtime that
 * owns all device memory), which still pass their own A, B and C.
 * No counterpart in the reference (which has no allocation-free variant).
 *
 * The shift vectors live in a static device array of this library,
 * XE_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU, held by every GPU that loads the
 * library until the process exits.  A call needs
 * xe_logspace_gemm_workspace_size(batch, m, n, k, a_linear, b_linear) bytes of
 * it (about 4*batch*(m+n) when both operands are log-domain); larger problems
 * return XE_ERR_INVALID_ARGUMENT.
 * The first call on a device resolves that array's device address (with the
 * device current), so make the first call before any stream capture.  Calls
 * share the array: calls that overlap on the GPU (other streams, other host
 * threads) race on it.  Nothing in it needs clearing; every call overwrites
 * what it reads.  Allocates nothing (no cudaMalloc, cudaFree or allocating
 * library call). */
#define XE_NOALLOC_SCRATCH_BYTES (4u << 20)
xe_status xe_logspace_gemm_noalloc(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                   int32_t a_linear,
                                   const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear,
                                   float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                   int64_t batch, int64_t m, int64_t n, int64_t k, int32_t shift_mode,
                                   void* stream);

/* The contraction kernel of xe_logspace_gemm alone, with caller-provided
 * shift vectors: `shift_a` (batch*m floats) for a log-domain A, NULL for a
 * linear A; `shift_b` (batch*n floats) likewise.  xe_logspace_gemm is
 * xe_logspace_shift for each log-domain operand followed by this call. */
xe_status xe_logspace_gemm_shifted(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                   const float* shift_a,
                                   const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, const float* shift_b,
                                   float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                   int64_t batch, int64_t m, int64_t n, int64_t k, void* stream);

/* xe_logspace_gemm_shifted with shift vectors of any element strides: the
 * shift of row m of batch entry t is shift_a[t*sa_sb + m*sa_sm], that of column
 * n shift_b[t*sb_sb + n*sb_sn] (a stride of 0 repeats one value).  Both
 * operands are log-domain.  Any per-row / per-column values are mathematically
 * valid shifts; this is how the scaled modes' log(einsum(exp(A), exp(B))) runs
 * as one contraction: the shift of an operand is its exp rule's fibre maximum
 * (translate.py:410-420) brought to a common value over the contracted axes
 * (:329-340), and log(n * e^s) = log(n) + s (:421-425) is the kernel's epilogue. */
xe_status xe_logspace_gemm_shifted_strided(const float* a, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                           const float* shift_a, int64_t sa_sb, int64_t sa_sm,
                                           const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                           const float* shift_b, int64_t sb_sb, int64_t sb_sn,
                                           float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                           int64_t batch, int64_t m, int64_t n, int64_t k, void* stream);

/* Prepared B operand.  The same B'[b,k,n] = exp(B - sB) (or a linear B as is)
 * that xe_logspace_gemm computes per 128-row tile of A, computed once and
 * stored split into TF32 hi / lo parts in the tiled, swizzled layout of the
 * contraction kernel's shared-memory stages (an opaque buffer: one 32 KB block
 * per batch entry, 128-column tile and 32-k block).  The kernel then loads each
 * stage with one bulk copy and spends no shared-memory bandwidth on B's
 * transform.  Results are bit-identical to xe_logspace_gemm's.  It replaces,
 * like xe_logspace_gemm, the per-operand shift / exp part of
 * _append_logspace_einsum (translate.py:727-740) for the B operand.
 *
 * xe_logspace_gemm does this by itself when its workspace holds
 * xe_logspace_gemm_workspace_size_prepared(...) bytes (B spanning more than
 * 64 columns, A more than 128 rows, k above 96; otherwise that size equals
 * xe_logspace_gemm_workspace_size).  A caller that contracts one B against
 * several A (row blocks of a sharded A) prepares it once with
 * xe_logspace_b_prepare and calls xe_logspace_gemm_prepared per A.
 *
 * xe_logspace_b_prepare: B (b,k,n) at b[b*b_sb + k*b_sk + n*b_sn] with n or k
 * contiguous, 16-byte aligned rows and that axis a multiple of 4
 * (XE_ERR_NOT_SUPPORTED otherwise).  A log-domain B (b_linear == 0) also writes
 * its column shifts sB (batch*n floats, max or min over k) to shift_b.
 * `prepared` holds xe_logspace_b_prepared_size(batch, n, k) bytes, 16-byte
 * aligned. */
size_t xe_logspace_b_prepared_size(int64_t batch, int64_t n, int64_t k);
size_t xe_logspace_gemm_workspace_size_prepared(int64_t batch, int64_t m, int64_t n, int64_t k,
                                                int32_t a_linear, int32_t b_linear);
xe_status xe_logspace_b_prepare(const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn, int32_t b_linear,
                                int64_t batch, int64_t n, int64_t k, int32_t shift_mode,
                                float* prepared, size_t prepared_bytes, float* shift_b, void* stream);

/* The contraction with a prepared B: as xe_logspace_gemm_shifted, with
 * `shift_a` (batch*m floats, from xe_logspace_shift) for a log-domain A or NULL
 * for a linear one, and the prepared B with its shift_b (NULL for a linear B). */
xe_status xe_logspace_gemm_prepared(const float* a, const float* a2, int64_t a_sb, int64_t a_sm, int64_t a_sk,
                                    const float* shift_a, const float* prepared, const float* shift_b,
                                    float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                    int64_t batch, int64_t m, int64_t n, int64_t k, void* stream);

/* Per-row shift of a strided 3-D operand: out[b*R + r] = max_k (or min_k) of
 * x[b*sb + r*sr + k*sk] (+ x2[...] when x2 is not NULL).  This is the
 * `max(x, axis=reduction_axes, keepdims=True)` call of translate.py:733
 * (TorchBackendFunctions.max -> torch.amax, backends/torch.py:37-48). */
xe_status xe_logspace_shift(const float* x, const float* x2, int64_t sb, int64_t sr, int64_t sk,
                            int64_t batch, int64_t rows, int64_t k, int32_t shift_mode,
                            float* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Softmax over the middle axis of a contiguous (outer, axis, inner) view:
 *   y[o,a,i] = exp(x[o,a,i] - max_a x[o,:,i]) / sum_a exp(x[o,:,i] - max)
 * Replaces TorchBackendFunctions.softmax (backends/torch.py:102-113), reached
 * raw-in/raw-out from translate.py:770-773; a trailing block of axes is
 * flattened into one axis by the caller exactly as torch.py:107-110 does.
 * `log_output` != 0 writes log(softmax) instead (used for categorical inputs,
 * whose log is taken next by the log-space lowering, translate.py:639-644). */
xe_status xe_softmax(const float* x, float* y, int64_t outer, int64_t axis_len, int64_t inner,
                     int32_t log_output, void* stream);

/* ------------------------------------------------------------------------ */
/* Log-space reduction of one operand (an einsum with a single operand, e.g.
 * 'ij->' or 'ij->i'), as _append_logspace_einsum lowers it
 * (translate.py:727-749 with one operand: max over the reduced axes, exp,
 * einsum, log, + shift):
 *   y[b*R + r] = log( sum_k exp(x[b,r,k] - s) ) + s,   s = max_k (or min_k)
 * Element (b,r,k) is x[b*sb + r*sr + k*sk]; y is contiguous (batch, rows). */
xe_status xe_logspace_reduce(const float* x, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows,
                             int64_t k, int32_t shift_mode, float* y, void* stream);

/* ------------------------------------------------------------------------ */
/* Log-space product / quotient of up to 6-D broadcast operands:
 * y = a + b (negate_b == 0) or y = a - b (negate_b != 0).
 * The contraction-free einsum of translate.py:706-718 (Hadamard / Kronecker
 * product, lowered by the reference to `add` after _broadcast_einsum_operand),
 * the log-space multiply of translate.py:790-793 and divide of :794-797.
 * Shapes/strides are in elements; a broadcast axis has stride 0.  y is
 * written contiguously in `shape` order. */
xe_status xe_log_add(const float* a, const int64_t* a_strides, const float* b, const int64_t* b_strides,
                     float* y, const int64_t* shape, int32_t ndim, int32_t negate_b, void* stream);

/* Log-space sum / difference with a common scalar shift (translate.py:774-789
 * with _append_shifted, :647-664):
 *   m = max (or min) over all elements of a and b
 *   y = log( exp(a - m) + exp(b - m) ) + m      (subtract == 0)
 *   y = log( exp(a - m) - exp(b - m) ) + m      (subtract != 0)
 * a, b broadcast as in xe_log_add.  `scratch` is device memory for one float
 * (the shift m). */
xe_status xe_log_add_exp(const float* a, const int64_t* a_strides, int64_t a_numel, const float* b,
                         const int64_t* b_strides, int64_t b_numel, float* y, const int64_t* shape, int32_t ndim,
                         int32_t subtract, int32_t shift_mode, float* scratch, void* stream);

/* Elementwise domain conversion of a contiguous array (translate.py:631-644):
 * op 0: y = exp(x) (log space -> raw), op 1: y = log(x) (raw -> log space). */
xe_status xe_unary(const float* x, float* y, int64_t n, int32_t op, void* stream);

/* ------------------------------------------------------------------------ */
/* Categorical input units of the circuit (demo/cirkit.py:525-527 builds
 * softmax(logits, dim=1)[v, x[b,v], :] in torch; the log-space lowering then
 * takes its log, translate.py:639-644):
 *   y[f,b,:] = table[f, pixels[b*pixel_stride + var_of_fold[f]], :]
 * table is (folds, states, units) and already in the log domain (see
 * xe_softmax with log_output).  var_of_fold may be NULL for the identity. */
xe_status xe_categorical_gather(const float* table, const uint8_t* pixels, int64_t pixel_stride,
                                const int32_t* var_of_fold, float* y, int64_t folds, int64_t states,
                                int64_t units, int64_t batch, void* stream);

/* Backward of the categorical gather (and of the gathers fused into the first
 * two circuit layers): table_grad[f + fold_offset, pixels[b, v], :] += grad[f, b, :]
 * with v = var_of_fold[f + fold_offset] (or f + fold_offset when null), for
 * f < folds.  grad is (folds, batch, units) contiguous; table_grad holds at least
 * fold_offset + folds folds of (states, units) and is accumulated into.  The
 * reference differentiates the demo's gather probabilities[pixel_range, batch.T]
 * (demo/cirkit.py:525-527) through torch indexing, whose backward is this
 * scatter-add.  Bad indices are clamped and reported as in xe_categorical_gather. */
xe_status xe_categorical_scatter_add(const float* grad, const uint8_t* pixels, int64_t pixel_stride,
                                     const int32_t* var_of_fold, float* table_grad, int64_t folds, int64_t states,
                                     int64_t units, int64_t batch, int64_t fold_offset, void* stream);

/* The first sum layer of a circuit over categorical input units, with the
 * gather fused into the contraction (replaces xe_categorical_gather followed
 * by xe_logspace_gemm on its output; demo/cirkit.py:525-527 feeding the
 * folded CP layer 'dac,dbc->dab', preprocess.py:1310-1337, lowered by
 * translate.py:686-750):
 *   C[f,b,n] = log( sum_k exp(T[f, x_b, k] - s) B'[f,k,n] ) + s (+ B's shift)
 *   with x_b = pixels[b*pixel_stride + var_of_fold[f]] and s = max (or min)
 *   over k of T[f, x_b, :].
 * T is the (folds, states, k) log table, k contiguous, fold stride t_sf and
 * state stride t_ss in elements.  B and C as in xe_logspace_gemm (batch =
 * folds, M = batch of samples).  var_of_fold may be NULL for the identity;
 * its entries must lie in [0, pixel_stride).  k <= 128.  A pixel value at or
 * above `states` (or a variable out of range) is clamped and recorded:
 * xe_device_status() then reports XE_ERR_INVALID_ARGUMENT << 16. */
xe_status xe_logspace_gemm_gather(const float* table, int64_t t_sf, int64_t t_ss, int64_t states, const uint8_t* pixels,
                                  int64_t pixel_stride, const int32_t* var_of_fold, const float* b, int64_t b_sb,
                                  int64_t b_sk, int64_t b_sn, int32_t b_linear, float* c, int64_t c_sb, int64_t c_sm,
                                  int64_t c_sn, int64_t folds, int64_t batch, int64_t n, int64_t k, int32_t shift_mode,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* The second sum layer of a circuit over categorical input units, with the
 * first layer read from a state table and the Hadamard product of its two
 * halves fused (replaces the first layer's per-sample output and the folded
 * Hadamard product 'cab,cab->cab', translate.py:706-718, that the next CP
 * layer 'dac,dbc->dab', preprocess.py:1310-1337, consumes):
 *   A[f,b,:] = T[f, x_b, :] + T[f + fold_offset, x'_b, :]
 *   with x_b = pixels[b*pixel_stride + var_of_fold[f]] and
 *   x'_b = pixels[b*pixel_stride + var_of_fold[f + fold_offset]];
 *   C[f,b,n] = log( sum_k exp(A[f,b,k] - s) B'[f,k,n] ) + s (+ B's shift).
 * T is then the first layer's output for every state, (folds0, states, k),
 * which one xe_logspace_gemm of the categorical table computes: a row of the
 * first layer depends on the sample only through its pixel value.  Every
 * argument as in xe_logspace_gemm_gather; fold_offset > 0, and the table and
 * var_of_fold hold at least folds + fold_offset folds. */
xe_status xe_logspace_gemm_gather_pair(const float* table, int64_t t_sf, int64_t t_ss, int64_t states,
                                       const uint8_t* pixels, int64_t pixel_stride, const int32_t* var_of_fold,
                                       int64_t fold_offset, const float* b, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                                       int32_t b_linear, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn,
                                       int64_t folds, int64_t batch, int64_t n, int64_t k, int32_t shift_mode,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Backward pass of the folded CP sum layer 'dac,dbc->dab' with K = N = 64
 * (preprocess.py:1310-1337, lowered by translate.py:686-750): the gradients
 * that torch autograd gives for the reference's executor calls, in which the
 * shift is a stop_gradient (translate.py:727-740; backends/torch.py:14-16).
 * Forward:  Y[f,m,o] = log( sum_k exp(X[f,m,k] - s) w[f,o,k] ) + s,
 *           X = A (+ A2), s = max_k (or min_k) X[f,m,:],
 *           w (folds, 64 o, 64 k) the linear weights (the contraction's B
 *           operand is w[f] transposed).
 * With G = dL/dY and V = G exp(s - Y):
 *   dA[f,m,k] = exp(X[f,m,k] - s) sum_o V[f,m,o] w[f,o,k]   (also dA2)
 *   dw[f,o,k] = sum_m V[f,m,o] exp(X[f,m,k] - s).
 * A, A2, Y, dA are (folds, m, 64) and G is (g_folds, m, 64), all contiguous
 * and 16-byte aligned; fold f reads G[f % g_folds] (g_folds = folds / 2 when
 * G is the next layer's dA, the gradient of both halves of its input).  dw
 * is (folds, 64, 64) contiguous and written whole, deterministically.
 * `workspace` must hold xe_cp_layer_backward_workspace_size(folds, m) bytes
 * (per-CTA partial sums of dw). */
size_t xe_cp_layer_backward_workspace_size(int64_t folds, int64_t m);
xe_status xe_cp_layer_backward(const float* a, const float* a2, const float* y, const float* g, int64_t g_folds,
                               const float* w, float* da, float* dw, int64_t folds, int64_t m, int32_t shift_mode,
                               void* workspace, size_t workspace_bytes, void* stream);

/* The same for the second layer over a state table (the backward of
 * xe_logspace_gemm_gather_pair): X[f,m,:] = T[f, x_m, :] + T[f + fold_offset,
 * x'_m, :], with T the (table_folds, states, 64) contiguous table and x_m,
 * x'_m the pixels of variables var_of_fold[f], var_of_fold[f + fold_offset]
 * (NULL: the fold) of sample m: pixels[m * pixel_sample_stride +
 * v * pixel_var_stride] for v < variables (a variable-major copy, strides
 * (1, m), reads one sector per 32 samples).  dA is the gradient of both
 * gathered rows; xe_state_table_pair_grad scatters it into the table. */
xe_status xe_cp_layer_backward_gather_pair(const float* table, int64_t table_folds, int64_t states,
                                           const uint8_t* pixels, int64_t pixel_sample_stride,
                                           int64_t pixel_var_stride, int64_t variables, const int32_t* var_of_fold,
                                           int64_t fold_offset, const float* y, const float* g, int64_t g_folds,
                                           const float* w, float* da, float* dw, int64_t folds, int64_t m,
                                           int32_t shift_mode, void* workspace, size_t workspace_bytes, void* stream);

/* The gradient of the state table from dA (folds, m, 64) contiguous: for each
 * f < folds, table_grad[f, s, :] is the sum of dA[f, m, :] over the samples m
 * whose pixel of variable var_of_fold[f] is s, and table_grad[f + fold_offset,
 * s, :] the same for var_of_fold[f + fold_offset] (the backward of torch
 * indexing in demo/cirkit.py:525-527 composed with the pair gather).  Those
 * 2 * folds table folds are written whole (zero for states no sample takes);
 * table_grad, contiguous (>= folds + fold_offset, states, 64), is not read.
 * The sums run in sample order, so the result is deterministic.  states <= 256.
 * Pixels as in xe_cp_layer_backward_gather_pair.  Bad pixel values are clamped
 * and reported as in xe_categorical_gather. */
xe_status xe_state_table_pair_grad(const float* da, int64_t folds, int64_t m, const uint8_t* pixels,
                                   int64_t pixel_sample_stride, int64_t pixel_var_stride, int64_t variables,
                                   const int32_t* var_of_fold, int64_t fold_offset, int64_t states,
                                   float* table_grad, void* stream);

/* y (cols, rows), contiguous, = the transpose of the uint8 matrix x (rows,
 * cols) with row stride row_stride: the pixels variable-major for the
 * state-table backward above (no counterpart in the reference, whose pixels
 * stay in torch; glue of this path).  rows <= 65535 * 32. */
xe_status xe_u8_transpose(const uint8_t* x, int64_t rows, int64_t cols, int64_t row_stride, uint8_t* y, void* stream);

/* ------------------------------------------------------------------------ */
/* Log-space Tucker layer 'bfi,bfj,foij->bfo' (the ternary einsum that
 * OptimizeContractionPaths fuses for Tucker circuits, preprocess.py:1095-1106,
 * lowered by _append_logspace_einsum, translate.py:686-750):
 *   y[b,f,o] = log( sum_ij exp(l[b,f,i]-sl) exp(r[b,f,j]-sr) w[f,o,i,j] ) + sl[b,f] + sr[b,f]
 * with sl = max_i (or min_i) l[b,f,:], sr likewise, and w linear.
 * l, r are (batch, folds, I) / (batch, folds, J) contiguous, w is
 * (folds, O, I, J) contiguous, y is (batch, folds, O) contiguous. */
xe_status xe_logspace_tucker(const float* l, const float* r, const float* w, float* y, int64_t batch,
                             int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                             void* stream);

/* The same layer over strided rows: l[b, f, :], r[b, f, :] and y[b, f, :] start at
 * b * x_sb + f * x_sf (element strides; for l and r non-negative multiples of 4) with
 * the units contiguous; w is (F, O, I, J) contiguous.  The folded Tucker circuits of the
 * reference (FoldSameShapedOperations + OptimizeContractionPaths,
 * preprocess.py:1095-1106, 1310-1393) carry their folds first:
 * 'acde,abd,abe->abc' over (F, B, I) slices of the previous layer's (F, B, O)
 * output, which these strides address without a copy. */
xe_status xe_logspace_tucker_strided(const float* l, int64_t l_sb, int64_t l_sf, const float* r, int64_t r_sb,
                                     int64_t r_sf, const float* w, float* y, int64_t y_sb, int64_t y_sf, int64_t batch,
                                     int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                                     void* stream);

/* ------------------------------------------------------------------------ */
/* Scaled stability modes (scaled_sum / scaled_max / scaled_min,
 * translate.py:115-585).  A value is a pair (normalized, log_scale) with
 * raw = normalized * exp(log_scale) and one log scale per last-axis fibre
 * (translate.py:119-126, 174-199). */

/* The einsum of normalized (linear) operands (translate.py:372): the batched
 * fp32 product C[b,m,n] = sum_k A[b,m,k] B[b,k,n] on the tensor cores (three
 * TF32 products per multiply-add, fp32 accumulation), raw output.  Strides as
 * in xe_logspace_gemm.  k must be >= 1. */
xe_status xe_scaled_gemm(const float* a, int64_t a_sb, int64_t a_sm, int64_t a_sk, const float* b, int64_t b_sb,
                         int64_t b_sk, int64_t b_sn, float* c, int64_t c_sb, int64_t c_sm, int64_t c_sn, int64_t batch,
                         int64_t m, int64_t n, int64_t k, void* stream);

/* Fibre normalisation of a strided tensor of rank <= 7 over its last axis
 * (translate.py:174-199, 373-382 and the exp rule :436-444):
 *   XE_FIBER_SUM / MAX / MIN: t = sum / max / min of the fibre,
 *                             normalized = x / t, log_scale = log(t)
 *   XE_FIBER_EXP: x is raw, the result is the pair of exp(x):
 *                             log_scale = max x, normalized = exp(x - log_scale)
 *   XE_FIBER_LSE: x is log-domain, the result is the sum-normalised pair of exp(x):
 *                             log_scale = logsumexp x, normalized = exp(x - log_scale)
 * normalized is written contiguous in x's shape, log_scale contiguous with one
 * value per fibre.  A rank-0 x is one fibre of length 1.  max / min reductions
 * propagate NaN (torch.amax / torch.amin).  MAX, MIN and EXP need a non-empty
 * fibre. */
typedef enum { XE_FIBER_SUM = 0, XE_FIBER_MAX = 1, XE_FIBER_MIN = 2, XE_FIBER_EXP = 3, XE_FIBER_LSE = 4 } xe_fiber_kind;
xe_status xe_fiber_normalize(const float* x, const int64_t* shape, const int64_t* strides, int32_t ndim, int32_t kind,
                             float* normalized, float* log_scale, void* stream);

/* Plain reduction y[b*rows + r] = sum / max / min over k of x[b*sb + r*sr + k*sk]
 * (the sum / amax / amin backend calls of the scaled translation, e.g.
 * translate.py:336, 396-400).  kind is XE_FIBER_SUM, XE_FIBER_MAX or
 * XE_FIBER_MIN; max and min need k >= 1. */
xe_status xe_reduce(const float* x, int64_t sb, int64_t sr, int64_t sk, int64_t batch, int64_t rows, int64_t k,
                    int32_t kind, float* y, void* stream);

/* Broadcast elementwise glue of the scaled translation, rank <= 6,
 * y contiguous in `shape`, operand strides in elements (0 = broadcast):
 *   XE_OP_ADD a+b, XE_OP_SUB a-b, XE_OP_MUL a*b, XE_OP_DIV a/b,
 *   XE_OP_MAX / XE_OP_MIN NaN-propagating maximum / minimum (torch.maximum),
 *   XE_OP_MUL_EXP  a*exp(b)    (raw value of a pair, translate.py:168-170)
 *   XE_OP_LOG_ADD  log(a)+b    (log of a pair, translate.py:445-449)
 *   XE_OP_RESCALE  a*exp(b-c)  (a pair at the common scale c, translate.py:253-257, 336-339)
 * c is used by XE_OP_RESCALE only and may be NULL otherwise. */
typedef enum {
  XE_OP_ADD = 0,
  XE_OP_SUB = 1,
  XE_OP_MUL = 2,
  XE_OP_DIV = 3,
  XE_OP_MAX = 4,
  XE_OP_MIN = 5,
  XE_OP_MUL_EXP = 6,
  XE_OP_LOG_ADD = 7,
  XE_OP_RESCALE = 8
} xe_elementwise_op;
xe_status xe_elementwise(int32_t op, const float* a, const int64_t* a_strides, const float* b, const int64_t* b_strides,
                         const float* c, const int64_t* c_strides, float* y, const int64_t* shape, int32_t ndim,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XE_B200_H */
