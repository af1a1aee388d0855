/*
 * firefly_b200.h — C ABI of the FireFly INT8 training hot path on NVIDIA B200 (sm_100a).
 *
 * Plain pointers, sizes and a CUDA stream; no framework types.  Every entry
 * point is asynchronous on `stream` (a cudaStream_t passed as void*; NULL is
 * the legacy default stream), performs no host synchronisation, allocates no
 * device memory, and returns FF_OK or an FF_ERR_* code.  On error,
 * ff_last_error() returns a message for the calling thread.
 *
 * Device pointers must point to memory of the current device.  All matrices
 * are row-major with an explicit leading dimension in ELEMENTS.
 *
 * Kernel-side waits (mbarrier / pipeline waits) are bounded in time; when one
 * gives up, the kernel records FF_DEVICE_TIMEOUT in the per-device status word
 * (ff_device_status) and returns instead of hanging.
 *
 * Reference: fumitoshi0524/FireFly (pure PyTorch).  Each entry point names the
 * reference function it replaces.
 */
#ifndef FIREFLY_B200_H
#define FIREFLY_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define FF_API __attribute__((visibility("default")))
#else
#define FF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FF_OK 0
#define FF_ERR_INVALID_ARG 1  /* null pointer, negative size, bad leading dimension */
#define FF_ERR_UNSUPPORTED 2  /* shape/alignment the kernel does not handle */
#define FF_ERR_CUDA 3         /* a CUDA runtime/driver call failed */

/* bits of the per-device status word */
#define FF_DEVICE_TIMEOUT 0x1u  /* a bounded in-kernel wait expired */
#define FF_DEVICE_BADARG 0x2u   /* a kernel-side argument check failed */

/* element types of floating-point inputs */
#define FF_DTYPE_F32 0
#define FF_DTYPE_BF16 1
#define FF_DTYPE_F16 2

/* GEMM output kinds */
#define FF_OUT_S32 0        /* raw int32 accumulators */
#define FF_OUT_F32 1        /* fp32  ((acc * sa[m]) * sb[n]) + bias[n] */
#define FF_OUT_BF16 2       /* bf16 of the fp32 value above */
#define FF_OUT_BF16_ACCUM 3 /* D = bf16(f32(D) + f32(bf16(value)))  (grad-cache add) */

/* Library version string, e.g. "firefly_b200 0.1.0 sm_100a". */
FF_API const char* ff_version(void);

/* Message of the last error on this host thread ("" if none). */
FF_API const char* ff_last_error(void);

/* Number of SMs of the current device (used for persistent grids). */
FF_API int ff_num_sms(int* out);

/*
 * Per-device status word (FF_DEVICE_* bits) written by kernels.  Reading it
 * synchronises the device.  `clear` != 0 resets it to 0 after reading.
 * No reference counterpart (the reference has no kernels of its own).
 */
FF_API int ff_device_status(uint32_t* out, int clear);

/*
 * Per-row absmax int8 quantiser.
 * Replaces fireflykernels.py:96-104 quantize_fp_to_int8 (and bitLinear.py:15-27):
 *   s[r] = max(max_c |x[r,c]*colmul[c]|, eps) / 127        (fp32, IEEE divide)
 *   q[r,c] = clamp(rint((x[r,c]*colmul[c]) / s[r]), -127, 127)   (round half even)
 * x: rows x cols of `dtype` with leading dim ldx.  colmul: NULL or fp32[cols].
 * q: int8 rows x ldq (ldq >= cols; entries cols..ldq-1 are written as 0).
 * s: fp32[rows].  rows == 0 is a no-op; cols must be >= 1.
 * Used per token on activations (the forward's activation quantiser).
 */
FF_API int ff_quant_rows_i8(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                     const float* colmul, float eps, int8_t* q, int64_t ldq, float* s,
                     void* stream);

/*
 * Row + column quantiser of one matrix in two passes (backward operands).
 * Row part: exactly ff_quant_rows_i8 (with optional colmul) into q_rows/s_rows.
 * Column part: the same quantiser applied to each COLUMN of x (no colmul),
 *   s_cols[c] = max(max_r |x[r,c]|, eps)/127, codes written TRANSPOSED:
 *   q_cols_t[c, r] (int8, leading dim ldqt >= rows; r in rows..ldqt-1 written as 0).
 * q_rows/s_rows may be NULL (column part only); q_cols_t/s_cols may be NULL
 * (row part only).  absmax_ws: fp32 workspace of rows + cols elements
 * (caller-owned device memory; contents on return are the raw absmax values).
 * Replaces the bf16 operand preparation of fireflykernels.py:164-193
 * (x2d.to(bf16) saved for backward, go_bf16, int_weight*weight_scale).
 */
FF_API int ff_quant_dual_i8(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                     const float* row_colmul, float eps,
                     int8_t* q_rows, int64_t ldq, float* s_rows,
                     int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                     float* absmax_ws, void* stream);

/*
 * Test hook for the failure path (no counterpart in the reference, which has no device code):
 * sets the limit, in nanoseconds, of the in-kernel waits of later launches on the current
 * device (0 restores the default of 2 s).  A wait that runs out sets FF_DEVICE_TIMEOUT in
 * the device status word, the kernel drains its in-flight copies and MMAs and returns, and
 * the context stays usable.  Synchronous; for tests only.
 */
FF_API int ff_set_wait_limit_ns(uint64_t ns);

/* Largest rows + cols that ff_quant_dual_i8_noalloc accepts (its scratch: 1 MiB of fp32). */
#define FF_NOALLOC_DUAL_MAX_ELEMS 262144

/*
 * ff_quant_dual_i8 for callers that cannot allocate device memory: same
 * arguments and results, minus absmax_ws.  No counterpart in the reference.
 *
 * Who needs it: a host runtime whose device memory is all handed out by its own
 * pool allocator (cudaMalloc from inside it would take memory the pool has
 * reserved and is not freed back through the pool), and callers on a pipelined
 * step that cannot afford cudaMalloc's implicit device-wide synchronisation.
 * The absmax scratch is a static array inside this library (FF_NOALLOC_DUAL_MAX_ELEMS
 * floats, held on every GPU that loads the library until the process exits);
 * rows + cols above that limit return FF_ERR_UNSUPPORTED.  Each call looks up the
 * array's device address on the current device (cudaGetSymbolAddress: a runtime
 * query, no allocation, correct again after a context reset); the first call on a
 * device may also load this library's kernels there, so make that first call
 * before any stream capture.  All calls share the
 * array: calls whose kernels overlap on the GPU (different streams, no ordering)
 * race on it and must be serialised by the caller.  The call allocates nothing
 * (no cudaMalloc, cudaFree or allocating library routine).
 */
FF_API int ff_quant_dual_i8_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ldx,
                                    const float* row_colmul, float eps,
                                    int8_t* q_rows, int64_t ldq, float* s_rows,
                                    int8_t* q_cols_t, int64_t ldqt, float* s_cols, void* stream);

/*
 * Exhaustive check of the SwiGLU kernels' branch-free arithmetic on the current
 * device: for every bf16 value x, 1/(1+exp(-x)) and x/(1+exp(-x)) as the kernels
 * compute them must equal the IEEE fp32 divides torch uses.  *mismatches = number of
 * inputs where they differ (must be 0 before ff_swiglu_quant_i8 / ff_swiglu_bwd_quant_i8
 * results can be trusted; run it once per device), *ieee_inputs = inputs the kernels
 * route to the IEEE operations instead (x <= -87, non-finite x, and x whose
 * 1 + exp(-x) has an all-ones significand), *first_mismatch = the smallest mismatching
 * bf16 bit pattern (0xFFFFFFFF when none).  Synchronous (it waits for the device), on
 * the legacy default stream.
 */
FF_API int ff_swiglu_selftest(uint32_t* mismatches, uint32_t* ieee_inputs, uint32_t* first_mismatch);

/*
 * SwiGLU activation fused with the dual quantiser: computes
 *   h[r,c] = bf16(bf16(silu(g[r,c])) * u[r,c]),  silu(x) = x / (1 + exp(-x))  (fp32)
 * exactly as torch's bf16 F.silu(g) * u does, writes it to h (bf16, leading dim ldh)
 * while taking its row and column absmax in the same pass, then quantises h exactly
 * as ff_quant_dual_i8 quantises a bf16 matrix (no colmul).  g, u: bf16 rows x cols
 * with the common leading dim ld (the gate and up halves of one [rows, 2*cols]
 * projection output: u = g + cols).  Outputs and absmax_ws (rows + cols floats) as
 * ff_quant_dual_i8.  Two kernels; g and u are read once.  Requires a passing
 * ff_swiglu_selftest on the device.
 * Replaces, on the SwiGLU MLP block built from BitLinear layers, the elementwise
 * silu and mul between the projections plus the down projection's input
 * quantisation (fireflykernels.py:164-167 applied to h).
 */
FF_API int ff_swiglu_quant_i8(const uint16_t* g, const uint16_t* u, int64_t ld, int64_t rows, int64_t cols,
                              float eps, uint16_t* h, int64_t ldh, int8_t* q_rows, int64_t ldq, float* s_rows,
                              int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws, void* stream);

/*
 * The gate/up GEMM of a SwiGLU block with the activation and the first pass of its
 * quantiser in the GEMM epilogue.  B: int8 [2F, K] (leading dim ldb): the F gate rows
 * then the F up rows of one BitLinear d -> 2F; A: int8 activation codes [M, K].
 * Writes gu = [g | u] (bf16 [M, 2F], leading dim ldgu), exactly as ff_gemm_i8 with
 * FF_OUT_BF16 would (scale_a per row, scale_b per column of gu, optional bias), and
 * h = bf16(bf16(silu(g)) * u) (bf16 [M, F], leading dim ldh) as ff_swiglu_quant_i8
 * computes it, then quantises h exactly as ff_swiglu_quant_i8 does (outputs as
 * ff_quant_dual_i8, no colmul; absmax_ws M + F floats).  Two kernels (the GEMM and the
 * quantiser pass) instead of three.  F must be a multiple of 128; gu, h, scale_b and
 * bias 16-byte aligned, ldgu and ldh multiples of 8.  Requires a passing
 * ff_swiglu_selftest on the device.
 */
FF_API int ff_swiglu_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                             const float* scale_b, const float* bias, uint16_t* gu, int64_t ldgu, uint16_t* h,
                             int64_t ldh, int64_t M, int64_t F, int64_t K, float eps, int8_t* q_rows, int64_t ldq,
                             float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws,
                             void* stream);

/*
 * The GEMM dh = dY * W_down of a SwiGLU block's backward with the SwiGLU backward and the
 * first pass of the [dg | du] quantiser in its epilogue.  A: int8 codes of dY * s_w
 * [M, K] (K = the block's output width), B: W_down int8 [K, F] row-major (read as the
 * K x N operand, as ff_gemm_i8_kn does), scale_a: fp32 [M] row scales.  With
 * dh = bf16(acc * scale_a[m]) (what ff_gemm_i8_kn gives with FF_OUT_BF16) and gu = [g | u]
 * (bf16 [M, 2F], leading dim ldgu: the saved gate/up output), writes
 * dgu = [dg | du] (bf16 [M, 2F], leading dim lddgu) exactly as ff_swiglu_bwd_quant_i8
 * forms it and quantises it exactly as ff_swiglu_bwd_quant_i8 does (colmul: NULL or fp32
 * [2F]; outputs as there; absmax_ws M + 2F floats).  dh itself is not written.
 * F must be a multiple of 128; gu, dgu and colmul 16-byte aligned, ldgu and lddgu
 * multiples of 8.  Requires a passing ff_swiglu_selftest on the device.
 */
FF_API int ff_swiglu_bwd_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                                 const uint16_t* gu, int64_t ldgu, const float* colmul, uint16_t* dgu, int64_t lddgu,
                                 int64_t M, int64_t F, int64_t K, float eps, int8_t* q_rows, int64_t ldq,
                                 float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws,
                                 void* stream);

/*
 * LayerNorm of the rows of a bf16 matrix x [rows, cols] (leading dim ldx) with fp32 gamma, beta:
 *   mean = sum(x)/cols, var = sum((x - mean)^2)/cols, rstd = 1/sqrt(var + eps)   (fp32)
 *   y = bf16((x - mean)*rstd*gamma + beta)        (bf16 [rows, cols], leading dim ldy)
 * writing mean and rstd (fp32 [rows]).  Unless q_rows and q_cols_t are both NULL it also
 * quantises y exactly as ff_quant_dual_i8 quantises a bf16 matrix (no colmul; outputs and
 * absmax_ws (rows + cols floats) as there; q_eps its eps), taking the absmax pass inside the
 * LayerNorm kernel.  cols a multiple of 8 up to 4096; x, y, gamma, beta 16-byte aligned,
 * ldx and ldy multiples of 8.  One kernel, or two with the quantiser.
 * No reference counterpart (the reference has no model code): the LayerNorm before a BitLinear
 * of the decoder plus that BitLinear's input quantisation (fireflykernels.py:164-167).
 */
FF_API int ff_layernorm_i8(const uint16_t* x, int64_t ldx, int64_t rows, int64_t cols, const float* gamma,
                           const float* beta, float eps, uint16_t* y, int64_t ldy, float* mean, float* rstd,
                           float q_eps, int8_t* q_rows, int64_t ldq, float* s_rows, int8_t* q_cols_t, int64_t ldqt,
                           float* s_cols, float* absmax_ws, void* stream);

/* fp32 workspace elements ff_layernorm_bwd needs for dgamma / dbeta of a [rows, cols] input. */
FF_API int64_t ff_layernorm_bwd_ws_elems(int64_t rows, int64_t cols);

/*
 * Backward of ff_layernorm_i8's LayerNorm from its output gradient dy and input x (both bf16
 * [rows, cols], leading dims lddy, ldx) and the forward's mean and rstd:
 *   dx = bf16(rstd*(g - mean_c(g) - xhat*mean_c(g*xhat))),  g = dy*gamma, xhat = (x - mean)*rstd
 * (bf16, leading dim lddx; cols up to 4096), dgamma[c] = sum_r dy*xhat and dbeta[c] = sum_r dy
 * (fp32 [cols]), each output NULL when not wanted.  The column sums go per block of 64 rows and
 * then over the blocks in order (deterministic); ws: ff_layernorm_bwd_ws_elems(rows, cols)
 * floats when dgamma or dbeta is wanted.  cols and leading dims multiples of 8; dy, x, dx,
 * gamma, ws 16-byte aligned.
 */
FF_API int ff_layernorm_bwd(const uint16_t* dy, int64_t lddy, const uint16_t* x, int64_t ldx, int64_t rows,
                            int64_t cols, const float* mean, const float* rstd, const float* gamma, uint16_t* dx,
                            int64_t lddx, float* dgamma, float* dbeta, float* ws, void* stream);

/*
 * GELU, tanh form, as the GELU GEMM epilogues evaluate it: for n bf16 inputs x writes
 *   h[i] = 0.5*x*(1 + tanhf(b*(x + k*x^3)))                            (fp32, before rounding)
 *   d[i] = 0.5*(1 + t) + 0.5*x*(1 - t*t)*b*(1 + 3k*x^2),  t = tanhf(b*(x + k*x^3))
 * with b = sqrt(2/pi), k = 0.044715, every operation rounded once; the variant bits (0-63)
 * choose which multiply-add pairs are fused (1: x + k*x^3 in h; 16: the same in d; 2: 1 - t*t;
 * 4: 1 + 3k*x^2; 8: the final sum of d) and, with 32, the product order of d's second term
 * ((0.5x*(1 - t*t)) * (b*(1 + 3k*x^2)) instead of ((0.5x*(1 - t*t))*b) * (1 + 3k*x^2)).
 * h or d may be NULL.  The host compares the results
 * with its framework's GELU kernels over all 65536 bf16 inputs and passes the matching
 * variant to ff_gelu_gemm_i8 / ff_gelu_bwd_gemm_i8.
 */
FF_API int ff_gelu_eval(const uint16_t* x, int64_t n, int fwd_variant, int bwd_variant, float* h, float* d,
                        void* stream);

/*
 * The up GEMM of a GELU MLP block (BitLinear d -> F, GELU, BitLinear F -> d) with the
 * activation and the first pass of its quantiser in the epilogue.  A: int8 activation codes
 * [M, K], B: int8 weight [F, K].  Writes u (bf16 [M, F], leading dim ldu) exactly as
 * ff_gemm_i8 with FF_OUT_BF16 would (scale_a per row, scale_b per column, optional bias) and
 * h = bf16(gelu(u)) (ff_gelu_eval's h under `variant`, rounded to bf16; leading dim ldh),
 * then quantises h exactly as ff_quant_dual_i8 quantises a bf16 matrix (no colmul; outputs as
 * there; absmax_ws M + F floats).  Two kernels.  F a multiple of 32; u, h, scale_b and bias
 * 16-byte aligned, ldu and ldh multiples of 8.
 * Replaces the up projection's matmul (fireflykernels.py:167), the elementwise GELU and the
 * down projection's input quantisation.
 */
FF_API int ff_gelu_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                           const float* scale_b, const float* bias, uint16_t* u, int64_t ldu, uint16_t* h,
                           int64_t ldh, int64_t M, int64_t F, int64_t K, float eps, int variant, int8_t* q_rows,
                           int64_t ldq, float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                           float* absmax_ws, void* stream);

/*
 * The GEMM dh = dY * W_down of a GELU MLP block's backward with the GELU backward and the
 * first pass of the du quantiser in its epilogue.  A: int8 codes of dY * s_w [M, K], B: W_down
 * int8 [K, F] row-major (the K x N operand, as ff_gemm_i8_kn reads it), scale_a: fp32 [M].
 * With dh = bf16(acc * scale_a[m]) and u the saved up output (bf16 [M, F], leading dim ldu),
 * writes du = bf16(dh * gelu'(u)) (ff_gelu_eval's d under `variant`; leading dim lddu) and
 * quantises it exactly as ff_quant_dual_i8 quantises the bf16 matrix du with row_colmul =
 * colmul (NULL or fp32 [F], the up projection's weight scales); absmax_ws M + F floats.  dh is
 * not written.  F a multiple of 32; u, du and colmul 16-byte aligned, ldu and lddu multiples
 * of 8.
 * Replaces the down projection's dX matmul (fireflykernels.py:191), torch's GELU backward and
 * the up projection's backward operand preparation (fireflykernels.py:184-193).
 */
FF_API int ff_gelu_bwd_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, const float* scale_a,
                               const uint16_t* u, int64_t ldu, const float* colmul, uint16_t* du, int64_t lddu,
                               int64_t M, int64_t F, int64_t K, float eps, int variant, int8_t* q_rows, int64_t ldq,
                               float* s_rows, int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws,
                               void* stream);

/*
 * Backward of the SwiGLU activation fused with the dual quantiser of the gate/up
 * projection's output gradient.  With dh the gradient of h (bf16, leading dim ldh)
 * and g, u as in ff_swiglu_quant_i8, the gradient of the [rows, 2*cols] projection
 * output is the two column panels, formed in bf16 exactly as torch's autograd
 * forms them for F.silu(g) * u:
 *   panel 0 (gate): dg = bf16(bf16(dh*u) * s * (1 + g*(1 - s))),  s = 1/(1 + exp(-g))
 *   panel 1 (up):   du = bf16(dh * bf16(silu(g)))
 * It is written to dgu (bf16 [rows, lddgu], lddgu >= 2*cols) while its absmax values
 * are taken, then quantised exactly as ff_quant_dual_i8 quantises the bf16 matrix
 * dgu with row_colmul = colmul (NULL or fp32[2*cols], the projection's weight
 * scales): q_rows [rows, ldq >= 2*cols], s_rows [rows], q_cols_t [2*cols, ldqt],
 * s_cols [2*cols]; absmax_ws rows + 2*cols floats.  cols must be a multiple of 8.
 * Requires a passing ff_swiglu_selftest on the device.
 * Replaces torch's mul/silu backward between the down projection's dX and the
 * gate/up projection's backward operand preparation (fireflykernels.py:184-193).
 */
FF_API int ff_swiglu_bwd_quant_i8(const uint16_t* dh, int64_t ldh, const uint16_t* g, const uint16_t* u,
                                  int64_t ld, int64_t rows, int64_t cols, const float* colmul, float eps,
                                  uint16_t* dgu, int64_t lddgu, int8_t* q_rows, int64_t ldq, float* s_rows,
                                  int8_t* q_cols_t, int64_t ldqt, float* s_cols, float* absmax_ws, void* stream);

/*
 * int8 transpose: dst[c, r] = src[r, c] for r < rows, c < cols; dst entries
 * r in rows..ldd-1 are written 0.  Builds the K-major copy of W (Wᵀ) that
 * the dX GEMM reads; the reference keeps per-handle weight layouts in
 * _cached_weight_transform (fireflykernels.py:64-90).
 */
FF_API int ff_transpose_i8(const int8_t* src, int64_t rows, int64_t cols, int64_t lds,
                    int8_t* dst, int64_t ldd, void* stream);

/*
 * int8 tensor-core GEMM (tcgen05 kind::i8, int32 accumulation in TMEM).
 *   acc[m,n] = sum_k A[m,k] * B[n,k]    A: M x K (lda), B: N x K (ldb), both K-contiguous
 *   D[m,n]   = epilogue(acc) per out_kind (FF_OUT_*), D leading dim ldd.
 * scale_a: NULL or fp32[M]; scale_b: NULL or fp32[N]; bias: NULL or fp32[N].
 * Requirements: A, B 16-byte aligned; lda, ldb multiples of 16; K >= 1.
 * Replaces the GEMMs of fireflykernels.py:167 (forward), :191 (dX), :193 (dW)
 * and the dead cuBLASLt path igemmlt + mm_dequant (fireflykernels.py:132-156).
 */
FF_API int ff_gemm_i8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
               const float* scale_a, const float* scale_b, const float* bias,
               void* D, int64_t ldd, int out_kind, int64_t M, int64_t N, int64_t K,
               void* stream);

/*
 * Bytes of the split-K workspace that ff_gemm_i8_ws uses for an M x N x K problem, or 0
 * when that shape takes no workspace (M > 128).  No counterpart in the reference (its
 * GEMM went through bitsandbytes / cuBLASLt, fireflykernels.py:132-156, :164-176).
 */
FF_API int64_t ff_gemm_i8_ws_bytes(int64_t M, int64_t N, int64_t K);

/*
 * ff_gemm_i8 (same arguments and results, bit for bit) with a split-K workspace for skinny
 * problems (M <= 128 rows of A, which are a stream over B): the k-range of every 128-row tile
 * of B is divided over all SMs (stream-K) and the int32 partial sums are added in the
 * workspace, the last contributor of a tile applying the epilogue.  ws: at least
 * ff_gemm_i8_ws_bytes(M, N, K) bytes, 16-byte aligned, all zeros before the first call; every
 * call leaves it all zeros again (after a device timeout, FF_DEVICE_TIMEOUT, zero it before
 * reuse).  Calls that share a workspace must be ordered on one stream.  With M > 128 the
 * workspace is not used and the call is ff_gemm_i8.
 */
FF_API int ff_gemm_i8_ws(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                  const float* scale_a, const float* scale_b, const float* bias,
                  void* D, int64_t ldd, int out_kind, int64_t M, int64_t N, int64_t K,
                  void* ws, int64_t ws_bytes, void* stream);

/*
 * ff_gemm_i8 with B given as a K x N row-major matrix (N contiguous, leading dim ldb >= N,
 * ldb a multiple of 16): acc[m,n] = sum_k A[m,k] * B[k,n].  B is staged MN-major, so the
 * dX GEMM reads the int8 weight W[O, K_in] directly as its K x N operand (no transposed
 * copy).  Replaces torch.matmul(go_bf16, w_bf16) at fireflykernels.py:191.
 */
FF_API int ff_gemm_i8_kn(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                         const float* scale_a, const float* scale_b, const float* bias,
                         void* D, int64_t ldd, int out_kind, int64_t M, int64_t N, int64_t K,
                         void* stream);

/*
 * Column sums of a bf16 matrix in fp32, rounded to bf16: db[c] = bf16(sum_r x[r,c]).
 * Deterministic (fixed reduction order).  ws: fp32 workspace of
 * ff_colsum_ws_elems(rows, cols) elements.  Replaces go_bf16.sum(dim=0)
 * (fireflykernels.py:200).
 */
FF_API int64_t ff_colsum_ws_elems(int64_t rows, int64_t cols);
FF_API int ff_colsum_bf16(const uint16_t* x, int64_t rows, int64_t cols, int64_t ldx,
                   uint16_t* out, float* ws, void* stream);

/*
 * ff_quant_dual_i8 of a bf16 matrix (the output gradient dY) that also writes the bias
 * gradient db[c] = bf16(sum_r x[r,c]) from the same read of x: the column sums are
 * accumulated in fp32 inside the absmax pass (per 128-row block, even and odd rows each in
 * row order, then the two added) and a second small kernel adds the blocks in order and
 * rounds to bf16.  Deterministic.  db_ws: fp32 workspace of ff_quant_dual_db_ws_elems(rows,
 * cols) elements; the other arguments as ff_quant_dual_i8 (dtype bf16).  rows == 0 writes
 * db = 0.  Replaces the operand preparation of go_bf16 (fireflykernels.py:185) together
 * with go_bf16.sum(dim=0) (fireflykernels.py:200).
 */
FF_API int64_t ff_quant_dual_db_ws_elems(int64_t rows, int64_t cols);
FF_API int ff_quant_dual_i8_db(const uint16_t* x, int64_t rows, int64_t cols, int64_t ldx,
                               const float* row_colmul, float eps,
                               int8_t* q_rows, int64_t ldq, float* s_rows,
                               int8_t* q_cols_t, int64_t ldqt, float* s_cols,
                               float* absmax_ws, uint16_t* db, float* db_ws, void* stream);

/*
 * Block-wise 8-bit AdamW step of a dense (non-BitLinear) parameter, in place.
 * Replaces bitsandbytes' AdamW8bit, which steps the reference's dense parameters
 * (fireflyoptim.py:83, :124); the algorithm is the published one (Dettmers et al., ICLR
 * 2022): m and v stored as uint8 codes of 256-entry maps (qmap_s signed for m, qmap_u
 * unsigned for v, fp32, sorted ascending) scaled per block of 2048 elements by fp32
 * absmax arrays [ceil(n/2048)].  Per element, fp32, each operation rounded once:
 *   p *= 1 - lr*wd (if wd != 0);  m = b1*m + (1-b1)*g;  v = b2*v + ((1-b2)*g)*g;
 *   p -= a_t * (m / (sqrt(v) + e_t)),  a_t = lr*sqrt(bc2)/bc1, e_t = eps*sqrt(bc2),
 *   bc = 1 - beta^step (scalars in double, then fp32);
 * then each block's absmax of |m| and v and the nearest map code of value * (1/absmax)
 * (ties to the lower code; an all-zero block keeps absmax 0).  p: fp32 or bf16 (FF_DTYPE_*), g:
 * fp32 or bf16; all arrays have n elements; p and g 16-byte aligned, m_q and v_q
 * 8-byte aligned.
 */
FF_API int ff_adamw8_blockwise(void* p, int p_dtype, const void* g, int g_dtype, uint8_t* m_q, float* m_absmax,
                               uint8_t* v_q, float* v_absmax, int64_t n, double lr, double beta1, double beta2,
                               double eps, double weight_decay, int64_t step, const float* qmap_s,
                               const float* qmap_u, void* stream);

/* One dense parameter of ff_adamw32_multi (all pointers device memory, numel elements each). */
typedef struct FfAdamw32Tensor {
  void* param;          /* FF_DTYPE_F32 or FF_DTYPE_BF16 (param_dtype), updated in place */
  const void* grad;     /* FF_DTYPE_F32 or FF_DTYPE_BF16 (grad_dtype) */
  float* exp_avg;       /* fp32 first moment, updated in place */
  float* exp_avg_sq;    /* fp32 second moment, updated in place */
  int64_t numel;
  int32_t param_dtype;
  int32_t grad_dtype;
  float eps_term;       /* fp32(eps * sqrt(1 - beta2^step)) of this parameter's step */
  float step_scale;     /* fp32(lr * sqrt(1 - beta2^step) / (1 - beta1^step)) */
} FfAdamw32Tensor;

/*
 * AdamW with fp32 moments of `count` dense parameters in ceil(count / 64) launches: the
 * parameters that bitsandbytes' AdamW8bit keeps in 32 bits (fewer than min_8bit_size
 * elements: norm scales, biases; fireflyoptim.py:83, :124).  Per element, fp32, each
 * operation rounded once, in the order of the torch ops it replaces:
 *   p *= decay (if use_decay; decay = fp32(1 - lr*wd));
 *   m = m*beta1 + g*one_minus_beta1;  v = v*beta2 + (g*one_minus_beta2)*g;
 *   p -= (m / (sqrt(v) + eps_term)) * step_scale.
 * `tensors` is a HOST array of `count` descriptors (read during the call).
 */
FF_API int ff_adamw32_multi(const FfAdamw32Tensor* tensors, int32_t count, float decay, int32_t use_decay,
                            float beta1, float one_minus_beta1, float beta2, float one_minus_beta2, void* stream);

/*
 * Fused DQT-SR 8-bit AdamW update of one int8 weight tensor (one BitLinear).
 * Replaces FireFlyOptim.step's bit-module loop body fireflyoptim.py:137-209
 * together with update_int8_weight_ (fireflykernels.py:218-223) and the
 * mu-law codecs (fireflyoptim.py:22-80).  Per element (fp32 math):
 *   decode m (signed), v (unsigned), r (signed) from uint8 codes * block absmax;
 *   m = b1*m + (1-b1)*g;  v = b2*v + (1-b2)*g*g;
 *   a = (m/bc1) / (sqrt(v/bc2) + eps);   ws = max(wscale[row], eps)
 *   r += -lr*(a + wd*q*ws)/ws;
 *   dq = sign(r)*(floor|r| + [u < clamp(frac|r| + tanh(a)*sr_bias*sign(r), 0, 1)])
 *   q = clamp(q+dq, -127, 127);  r -= dq;
 *   re-encode r, m, v per block of `block` elements (new block absmax, clamp 1e-12).
 * Hyperparameters are doubles (python floats); each is rounded to fp32 where
 * the reference's torch op rounds it (1-beta is formed in double first).
 * numel elements of q/g/m/v/r; block must be 256; row_len = elements per
 * weight row (wscale index = (elem_base + i) / row_len).  bc1 = 1-b1^t,
 * bc2 = 1-b2^t for the step t being taken.
 * Uniforms: u != NULL -> u[i] (fp32, element i); u == NULL -> Philox4x32-10
 * keyed by (seed, step) at global element index rng_offset + i.
 * dec_s / dec_u: fp32[256] decode tables (x_norm of each code).
 * elem_base: element index of element 0 within its weight (0 unless a shard).
 */
FF_API int ff_dqt_adamw8(int8_t* q, const float* wscale, int64_t row_len, int64_t elem_base,
                  const uint16_t* g, uint8_t* m_q, float* m_absmax, uint8_t* v_q,
                  float* v_absmax, uint8_t* r_q, float* r_absmax, int64_t numel,
                  int64_t block, double lr, double beta1, double beta2, double eps, double wd,
                  double bc1, double bc2, double sr_bias, uint64_t seed, uint64_t step,
                  int64_t rng_offset, const float* u, const float* dec_s,
                  const float* dec_u, void* stream);

/*
 * ff_dqt_adamw8 for one rank of a data-parallel job, with the gradient reduction and the
 * weight gather in the same kernel (no reference counterpart: the reference trains on one
 * GPU).  The gradient of element i is the average of the n_srcs bf16 arrays g_srcs[k][i]
 * (every rank's gradient of the same elements, the other ranks' read over NVLink: device
 * pointers of this process, e.g. from ff_ipc_open), summed in fp32 in the order k = 0..n_srcs-1,
 * multiplied by 1/n_srcs and rounded to bf16; the new weight of element i is written to
 * q_dsts[k][i] for every k < n_dsts (every rank's copy of the weights; q itself is read for the
 * current weight and must be one of them).  g_out (or NULL) receives the averaged gradient.
 * 1 <= n_srcs, n_dsts <= FF_DQT_MAX_SOURCES; g_srcs 16-byte aligned, q_dsts 8-byte aligned.
 * The other arguments are ff_dqt_adamw8's (uniforms always from Philox).  The kernel does not
 * wait for the other ranks: the caller orders it after every rank's gradient is complete and
 * orders every rank's next use of the weights or gradients after it (e.g. a collective on the
 * stream before and after).
 */
#define FF_DQT_MAX_SOURCES 8
FF_API int ff_dqt_adamw8_peers(int8_t* q, const float* wscale, int64_t row_len, int64_t elem_base,
                               const uint16_t* const* g_srcs, int n_srcs, int8_t* const* q_dsts, int n_dsts,
                               uint16_t* g_out, uint8_t* m_q, float* m_absmax, uint8_t* v_q, float* v_absmax,
                               uint8_t* r_q, float* r_absmax, int64_t numel, int64_t block, double lr,
                               double beta1, double beta2, double eps, double wd, double bc1, double bc2,
                               double sr_bias, uint64_t seed, uint64_t step, int64_t rng_offset,
                               const float* dec_s, const float* dec_u, void* stream);

/*
 * Device memory shared between the processes of one node (CUDA IPC), for the data-parallel
 * arenas that ff_dqt_adamw8_peers reads and writes.  ff_ipc_alloc: one device allocation of the
 * current device (freed by ff_ipc_free); ff_ipc_get_handle writes its FF_IPC_HANDLE_BYTES-byte
 * handle; ff_ipc_open maps another process's allocation from its handle (peer access enabled),
 * ff_ipc_close unmaps it.
 */
#define FF_IPC_HANDLE_BYTES 64
FF_API int ff_ipc_alloc(int64_t bytes, void** ptr);
FF_API int ff_ipc_free(void* ptr);
FF_API int ff_ipc_get_handle(void* ptr, uint8_t* handle);
FF_API int ff_ipc_open(const uint8_t* handle, void** ptr);
FF_API int ff_ipc_close(void* ptr);

/*
 * update_int8_weight_ (fireflykernels.py:218-223): w = clamp(int16(w) + dq, -127, 127).
 * dq: int32[n].
 */
FF_API int ff_update_int8_weight(int8_t* w, const int32_t* dq, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FIREFLY_B200_H */
