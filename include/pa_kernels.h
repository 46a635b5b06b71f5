/*
 * pa_kernels.h - C ABI of the B200 (sm_100a) attention-block kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (pa_stream_t is a cudaStream_t; NULL = legacy default stream), enqueues its
 * kernels on that stream and returns a pa_status. Nothing here allocates
 * device memory: scratch space is passed in by the caller (query the size with
 * the matching *_workspace_size function). Calls never throw and never print.
 *
 * Kernels whose waits are bounded record a timeout in a per-device status
 * word instead of hanging; pa_device_status() reads (and optionally clears) it.
 *
 * Layouts follow the Pure-Attention boundary:
 *   q, k, v, o, dO, dq, dk, dv : [B, L, H, D] row-major (heads interleaved
 *                                along E = H*D, the reference's [N, L, E])
 *   lse                        : [B*H, L] fp32, natural-log log-sum-exp
 *   delta                      : [B, L, H] fp32
 *   matrices                   : row-major
 */
#ifndef PA_KERNELS_H
#define PA_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PA_ABI_VERSION 1

typedef enum pa_status {
  PA_OK = 0,
  PA_ERR_SHAPE = 1,       /* sizes are inconsistent or zero where not allowed */
  PA_ERR_DTYPE = 2,       /* dtype not supported by this entry point */
  PA_ERR_ALIGN = 3,       /* a pointer or stride breaks the 16-byte TMA rule */
  PA_ERR_UNSUPPORTED = 4, /* e.g. head_dim outside {32, 64, 128} */
  PA_ERR_LAUNCH = 5,      /* the CUDA launch itself failed */
  PA_ERR_TIMEOUT = 6,     /* a kernel's bounded wait ran out (device status) */
  PA_ERR_WORKSPACE = 7,   /* workspace missing or too small */
  PA_ERR_NULL = 8,        /* a required pointer is NULL */
  PA_ERR_DEVICE = 9       /* no sm_100 device current, or a CUDA runtime error */
} pa_status;

typedef enum pa_dtype { PA_F32 = 0, PA_BF16 = 1 } pa_dtype;

typedef void* pa_stream_t; /* cudaStream_t */

typedef struct pa_attn_desc {
  int32_t batch;       /* B (the reference calls it N) */
  int32_t seq_len;     /* L */
  int32_t num_heads;   /* H */
  int32_t head_dim;    /* D = E / H */
  int32_t dtype;       /* pa_dtype of q, k, v, o, dO, dq, dk, dv */
  float softmax_scale; /* <= 0 selects 1/sqrt(head_dim) */
} pa_attn_desc;

/* Arithmetic of the fp32 entry points (pa_matmul*, pa_linear_*, and
 * pa_attn_fwd / pa_attn_bwd with dtype PA_F32 and head_dim 64), set per
 * calling thread:
 *   PA_F32_MATH_SPLIT3 (default): operands split into bf16 hi/lo planes and
 *     every product taken as hi*hi + hi*lo + lo*hi (fp32-level accuracy,
 *     within 1e-3 of float64 where the reference computes in fp32);
 *   PA_F32_MATH_BF16: operands rounded to bf16, one product, fp32 accumulation
 *     and fp32 storage (mixed-precision training; about 3x fewer tensor-core
 *     cycles and half the operand traffic).
 * Not in the reference, which computes every product in fp32 SIMT code. */
typedef enum pa_f32_math { PA_F32_MATH_SPLIT3 = 0, PA_F32_MATH_BF16 = 1 } pa_f32_math;
int pa_set_f32_math(int mode); /* PA_OK, or PA_ERR_UNSUPPORTED for an unknown mode */
int pa_get_f32_math(void);

/* Library information and status. */
int pa_abi_version(void);
const char* pa_status_string(int status);
/* Synchronises `stream`, returns PA_OK or the first error recorded by a kernel
 * on the current device (PA_ERR_TIMEOUT), and resets the word when clear != 0. */
int pa_device_status(pa_stream_t stream, int clear);

/* Self-test of the failure detection (no counterpart in the reference, which
 * had none). Enqueues one small kernel that waits on an mbarrier with the same
 * bounded wait as the attention and GEMM kernels, but with a limit of
 * limit_ns (at most 5 s) instead of the kernels' 2 s. With arrive != 0 the
 * barrier completes first and the wait returns at once; with arrive == 0
 * nothing completes it, the wait runs out, and the kernel records
 * PA_ERR_TIMEOUT in the device status word and returns normally (the context
 * stays usable). While the word is set, the attention kernels skip their work;
 * pa_device_status(stream, 1) reads and clears it. */
int pa_wait_selftest(uint64_t limit_ns, int arrive, pa_stream_t stream);

/* ---------------------------------------------------------------- attention */

/* Bytes of workspace pa_attn_fwd needs for this shape (0 for bf16; the fp32
 * path keeps bf16 hi/lo planes of q, k, v there). */
size_t pa_attn_fwd_workspace_size(const pa_attn_desc* desc);

/* Flash-attention forward: o = softmax(q k^T * scale) v, lse = row log-sum-exp.
 * Replaces launch_flash_attention (include/backend/Launchers.cuh:159-167).
 * bf16: head_dim 64 or 128 (workspace may be NULL). f32: head_dim 32 or 64,
 * computed as bf16 hi/lo splits (three tensor-core products per GEMM). */
int pa_attn_fwd(const pa_attn_desc* desc, const void* q, const void* k, const void* v, void* o,
                float* lse, void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* Bytes of workspace pa_attn_bwd needs for this shape. */
size_t pa_attn_bwd_workspace_size(const pa_attn_desc* desc);

/* Flash-attention backward from the saved lse: dq, dk, dv (overwritten, or
 * added to when accumulate != 0). Replaces launch_flash_backward
 * (include/backend/Launchers.cuh:169-174), which allocated its scratch itself. */
int pa_attn_bwd(const pa_attn_desc* desc, const void* q, const void* k, const void* v,
                const void* o, const void* dO, const float* lse, void* dq, void* dk, void* dv,
                int accumulate, void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* pa_attn_bwd for PA_F32 tensors that reuses the bf16 operand planes of q, k, v
 * which pa_attn_fwd left in its workspace (`fwd_workspace`, made under f32 math
 * mode `fwd_mode`, and not written since): only dO is converted. A bf16-math
 * forward at head_dim 64 kept no lo planes, so a split3 backward converts q, k,
 * v again. With dtype PA_BF16 or a NULL fwd_workspace this is pa_attn_bwd. No
 * counterpart in the reference, whose backward reads its fp32 inputs again. */
int pa_attn_bwd_kept(const pa_attn_desc* desc, const void* q, const void* k, const void* v,
                     const void* o, const void* dO, const float* lse, void* dq, void* dk, void* dv,
                     int accumulate, const void* fwd_workspace, size_t fwd_workspace_bytes,
                     int fwd_mode, void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* Backward without a caller workspace, for callers that cannot allocate device
 * memory (e.g. plugins whose host framework owns all GPU memory, or runtimes
 * that forbid allocations once a model is resident). No counterpart in the
 * reference, which allocated its scratch inside the call.
 * Same arguments and results as pa_attn_bwd minus the workspace: the scratch
 * is a fixed PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE-byte array in the library's
 * device memory, held on every GPU that loads the library until exit. Shapes
 * whose pa_attn_bwd_workspace_size exceeds it return PA_ERR_WORKSPACE: about
 * 113 000 (batch*head, padded query) rows for bf16 at head_dim 64 (296 B per
 * row), about 25 000 for the fp32 path (its operand planes add ~1 KB per
 * row). All calls on a device share that array: calls that overlap on the
 * GPU race and must be serialised. The first call on each device looks up the array's
 * device address; make it before any stream capture on that device. */
#define PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE (32u << 20)
int pa_attn_bwd_noalloc(const pa_attn_desc* desc, const void* q, const void* k, const void* v,
                        const void* o, const void* dO, const float* lse, void* dq, void* dk,
                        void* dv, int accumulate, pa_stream_t stream);

/* delta = rowsum(dO * o) as [B, L, H] fp32. Replaces compute_delta_kernel
 * (include/backend/Kernels.cuh:132, launched inside launch_flash_backward). */
int pa_attn_delta(const pa_attn_desc* desc, const void* dO, const void* o, float* delta,
                  pa_stream_t stream);

/* ---------------------------------------------------------------- layer norm */

/* y = gamma * (x - mean) * rstd + beta over rows of length N; saves mean, rstd.
 * Replaces launch_layer_norm_forward (include/backend/Launchers.cuh:178-189). */
int pa_layer_norm_fwd(const float* x, const float* gamma, const float* beta, float* y,
                      float* mean, float* rstd, uint32_t M, uint32_t N, float epsilon,
                      pa_stream_t stream);

/* sum = x + r (written), then y = LayerNorm(sum) as pa_layer_norm_fwd: a
 * residual add fused in front of the norm, one pass over the rows instead of an
 * add pass plus a norm pass. The reference builds the same value from its
 * elementwise add launcher and launch_layer_norm_forward
 * (include/backend/Launchers.cuh:178-189) in sequence. sum may alias neither
 * x nor r. The backward is pa_add_layer_norm_bwd. */
int pa_add_layer_norm_fwd(const float* x, const float* r, float* sum, const float* gamma,
                          const float* beta, float* y, float* mean, float* rstd, uint32_t M,
                          uint32_t N, float epsilon, pa_stream_t stream);

/* pa_layer_norm_fwd (r and sum NULL) or pa_add_layer_norm_fwd that also writes
 * y's bf16 operand planes, so a projection that reads y next takes them
 * (pa_linear_fwd_planes with PA_LINEAR_KEPT_VALID) instead of converting y.
 * The planes are made under the calling thread's f32 math mode, in the layout
 * of `kept` for a projection with in_features = N: hi = bf16(y) and, under
 * split3 math, lo = bf16(y - hi), from the same values as y. y_planes:
 * 256-byte aligned, at least pa_linear_kept_size(M, N) bytes. The reference
 * has no counterpart: its LayerNorm writes fp32 only and every matmul reads
 * fp32. */
int pa_layer_norm_fwd_planes(const float* x, const float* r, float* sum, const float* gamma,
                             const float* beta, float* y, float* mean, float* rstd, uint32_t M,
                             uint32_t N, float epsilon, void* y_planes, size_t y_planes_bytes,
                             pa_stream_t stream);

size_t pa_layer_norm_bwd_workspace_size(uint32_t M, uint32_t N);

/* dx (overwritten), dgamma and dbeta (accumulated); a NULL output is skipped.
 * Replaces launch_layer_norm_backward (include/backend/Launchers.cuh:191-203). */
int pa_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                      const float* gamma, float* dx, float* dgamma, float* dbeta, uint32_t M,
                      uint32_t N, void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* As pa_layer_norm_bwd, but dx is accumulated (dx += dL/dx), for an input that
 * also feeds a residual branch whose gradient is already in dx: no temporary
 * and no extra add pass. (The reference's LayerNorm node hands the input's
 * gradient buffer to the overwriting kernel, source/core/Autograd.cpp:257-280,
 * which drops the other consumers' contributions.) */
int pa_layer_norm_bwd_accumulate(const float* dy, const float* x, const float* mean,
                                 const float* rstd, const float* gamma, float* dx, float* dgamma,
                                 float* dbeta, uint32_t M, uint32_t N, void* workspace,
                                 size_t workspace_bytes, pa_stream_t stream);

/* Backward of pa_add_layer_norm_fwd in one pass over the rows: with
 * G = dL/dsum = LayerNorm_bwd(dy) + dsum, where dsum is the gradient that
 * reached sum from its other consumers (NULL: none),
 *   dx = G (flags & PA_ADD_LN_ACC_DX: dx += G), dr likewise (PA_ADD_LN_ACC_DR),
 * and dgamma, dbeta accumulated as in pa_layer_norm_bwd; any output may be
 * NULL, and dx and dr may be the same buffer (sum = x + x). Replaces the
 * reference's LayerNorm backward (include/backend/Launchers.cuh:191-203)
 * followed by its two gradient-accumulate launches for the add
 * (tensor_add_grad_kernel.cu:4-9): the sum's gradient is never written. */
#define PA_ADD_LN_ACC_DX 1
#define PA_ADD_LN_ACC_DR 2
int pa_add_layer_norm_bwd(const float* dy, const float* dsum, const float* sum,
                          const float* mean, const float* rstd, const float* gamma, float* dx,
                          float* dr, float* dgamma, float* dbeta, uint32_t M, uint32_t N,
                          int flags, void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* ---------------------------------------------------------------- matmul */

/* fp32 GEMMs on the tensor cores: operands are split into bf16 hi/lo planes
 * in the workspace and each product is hi*hi + hi*lo + lo*hi (fp32-level
 * accuracy). Bytes of workspace any of the three calls below needs for these
 * M, N, K: */
size_t pa_matmul_workspace_size(int M, int N, int K);

/* C[M,N] = A[M,K] B[K,N]. Replaces launch_matmul_tiled (Launchers.cuh:15-23). */
int pa_matmul(const float* A, const float* B, float* C, int M, int N, int K, void* workspace,
              size_t workspace_bytes, pa_stream_t stream);

/* dX[M,N] += dY[M,K] W[N,K]^T. Replaces launch_matmul_grad_X (Launchers.cuh:64-72). */
int pa_matmul_grad_x(const float* dY, const float* W, float* dX, int M, int N, int K,
                     void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* dW[N,K] += X[M,N]^T dY[M,K]. Replaces launch_matmul_grad_W (Launchers.cuh:74-82). */
int pa_matmul_grad_w(const float* X, const float* dY, float* dW, int M, int N, int K,
                     void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* ---------------------------------------------------------------- fused projection
 * No single reference counterpart: one call does what the reference does in
 * separate passes around a projection - core::matmul + core::matadd + core::split
 * forward (Functional.cpp:12-52, Functional.cpp:205-252, matadd_kernel.cu:4-12,
 * split_forward_kernel.cu:4-21), and MatMulFunction + AddFunction +
 * SplitFunction backward (Autograd.cpp:9-59, 113-177; sum_rows_grad_kernel.cu,
 * split_backward_kernel.cu). fp32 in/out, same arithmetic as pa_matmul.
 * out_features must be a multiple of n_outs (n_outs, n_parts in 1..3). */
size_t pa_linear_workspace_size(int M, int in_features, int out_features);

/* Y = X[M,in] W[in,out] (+ bias[out] if bias is not NULL), written as n_outs
 * column blocks: outs (a HOST array of n_outs device pointers) receives
 * outs[c][M, out/n_outs] = Y[:, c*out/n_outs : (c+1)*out/n_outs]. */
int pa_linear_fwd(const float* X, const float* W, const float* bias, float* const* outs, int n_outs,
                  int M, int in_features, int out_features, void* workspace, size_t workspace_bytes,
                  pa_stream_t stream);

/* With dY the concatenation of the n_parts column blocks dy_parts (a HOST array
 * of device pointers, [M, out/n_parts] each): dX[M,in] += dY W^T,
 * dW[in,out] += X^T dY, dbias[out] += column sums of dY. dX, dW and dbias may
 * each be NULL (that gradient is skipped). */
int pa_linear_bwd(const float* X, const float* W, const float* const* dy_parts, int n_parts,
                  float* dX, float* dW, float* dbias, int M, int in_features, int out_features,
                  void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* Projection followed by a ReLU, Y = max(0, X W + bias) [M, out], the clamp in
 * the GEMM epilogue (the reference runs Linear then ReLU: matmul, matadd and
 * ReLU_kernel.cu:4-12 passes, tests/main_denoise.py:18-22). Its backward takes
 * that Y and the gradient dY of Y: dY is masked by Y > 0 while it is gathered
 * into the GEMM operands (ReLU_backward_kernel.cu:4-10 folded in), then
 * dX += dZ W^T, dW += X^T dZ, dbias += colsum(dZ) with dZ = dY * (Y > 0).
 * Same workspace as pa_linear_fwd / pa_linear_bwd. */
int pa_linear_relu_fwd(const float* X, const float* W, const float* bias, float* Y, int M,
                       int in_features, int out_features, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream);
int pa_linear_relu_bwd(const float* X, const float* W, const float* Y, const float* dY, float* dX,
                       float* dW, float* dbias, int M, int in_features, int out_features,
                       void* workspace, size_t workspace_bytes, pa_stream_t stream);

/* Keeping X's operand planes from a projection's forward for its backward, so
 * the backward does not convert X again (a graph node holds them in between).
 * Bytes under the calling thread's f32 math mode (one bf16 plane of X for
 * bf16 math, hi and lo for split3): */
size_t pa_linear_kept_size(int M, int in_features);
/* pa_linear_fwd (relu = 0) or pa_linear_relu_fwd (relu = 1, n_outs = 1) that
 * also leaves X's planes in `kept` (256-byte aligned, pa_linear_kept_size bytes). */
int pa_linear_fwd_keep(const float* X, const float* W, const float* bias, float* const* outs,
                       int n_outs, int relu, int M, int in_features, int out_features, void* kept,
                       size_t kept_bytes, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream);
/* pa_linear_fwd_keep with X's planes possibly made already and Y's planes
 * written too, so a projection that reads Y next needs no conversion of it:
 *  - flags & PA_LINEAR_KEPT_VALID: `kept` already holds X's planes, made under
 *    f32 math mode kept_mode (e.g. the y_planes of the projection that
 *    produced X); X is not converted again where they serve the current mode;
 *  - y_planes (n_outs = 1; may be NULL): Y's bf16 planes, in the layout of
 *    `kept` for a projection with in_features = out_features (256-byte
 *    aligned, pa_linear_kept_size(M, out_features) bytes): hi = bf16(Y) and,
 *    under split3 math, lo = bf16(Y - hi), written by the GEMM epilogue from
 *    the same values as Y. */
#define PA_LINEAR_KEPT_VALID 1
int pa_linear_fwd_planes(const float* X, const float* W, const float* bias, float* const* outs,
                         int n_outs, int relu, int M, int in_features, int out_features, void* kept,
                         size_t kept_bytes, int kept_mode, int flags, void* y_planes,
                         size_t y_planes_bytes, void* workspace, size_t workspace_bytes,
                         pa_stream_t stream);
/* pa_linear_bwd (Y = NULL) or pa_linear_relu_bwd (Y = the ReLU output,
 * n_parts = 1) reading X's planes from `kept`, written by pa_linear_fwd_keep
 * under f32 math mode `kept_mode`. Where they cannot serve the current mode
 * (a bf16 forward keeps no lo plane for a split3 backward) X is converted
 * again, as pa_linear_bwd does. flags & PA_LINEAR_DX_OVERWRITE: dX = dY W^T
 * (its old contents are neither read nor kept; for a gradient buffer nothing
 * has written yet, which then needs no zeroing) instead of dX += dY W^T. */
#define PA_LINEAR_DX_OVERWRITE 1
int pa_linear_bwd_kept(const float* X, const float* W, const void* kept, size_t kept_bytes,
                       int kept_mode, const float* Y, const float* const* dy_parts, int n_parts,
                       float* dX, float* dW, float* dbias, int M, int in_features,
                       int out_features, int flags, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream);

/* ---------------------------------------------------------------- elementwise */

/* out[M,N] = A[M,N] + bias[N]. Replaces launch_matadd_tiled (Launchers.cuh:25-32). */
int pa_bias_add(const float* A, const float* bias, float* out, int M, int N, pa_stream_t stream);

/* out = a + b elementwise over n values (same-shape residual add). */
int pa_add(const float* a, const float* b, float* out, size_t n, pa_stream_t stream);

/* dst += src over n values. Replaces launch_tensor_add_grad (Launchers.cuh:84-89). */
int pa_grad_accumulate(const float* src, float* dst, size_t n, pa_stream_t stream);

/* db[N] += column sums of dY[M,N]. Replaces launch_sum_rows_grad (Launchers.cuh:91-97). */
int pa_bias_grad(const float* dY, float* db, int M, int N, pa_stream_t stream);
/* The same sums split over the whole GPU in two deterministic stages, with a
 * workspace of pa_bias_grad_workspace_size(M, N) bytes (16-byte aligned). */
size_t pa_bias_grad_workspace_size(int M, int N);
int pa_bias_grad_ws(const float* dY, float* db, int M, int N, void* workspace,
                    size_t workspace_bytes, pa_stream_t stream);

/* Split [rows, parts*width] along the last dimension into `parts` arrays of
 * [rows, width]; outs is a HOST array of `parts` device pointers (parts <= 8).
 * Replaces launch_split_forward (Launchers.cuh:139-147). */
int pa_split_last_dim(const float* in, float* const* outs, uint32_t parts, uint32_t rows,
                      uint32_t width, pa_stream_t stream);

/* grad_in[rows, parts*width] += concatenation of part_grads (NULL parts are
 * treated as zero). Replaces launch_concat_backward (Launchers.cuh:149-157). */
int pa_concat_last_dim_grad(const float* const* part_grads, float* grad_in, uint32_t parts,
                            uint32_t rows, uint32_t width, pa_stream_t stream);

/* ---------------------------------------------------------------- training utilities
 * Kernels behind the rest of the operator surface (ReLU, MSE, Adam, init).
 * They sit off the attention path; gradient outputs are accumulated (+=). */

/* y = max(x, 0). Replaces launch_ReLU_tiled (Launchers.cuh:34-40). */
int pa_relu_fwd(const float* x, float* y, size_t n, pa_stream_t stream);
/* dx += dy * (x > 0). Replaces launch_relu_backward (Launchers.cuh:99-105). */
int pa_relu_bwd(const float* dy, const float* x, float* dx, size_t n, pa_stream_t stream);
/* loss[0] = mean((pred - target)^2), deterministic. Replaces launch_mse_forward (Launchers.cuh:116-122). */
int pa_mse_fwd(const float* pred, const float* target, float* loss, size_t n, pa_stream_t stream);
/* pa_mse_fwd computes the sum in one CTA (deterministic, slow for large n);
 * pa_mse_fwd_ws spreads it over the GPU in two deterministic stages using
 * pa_mse_fwd_workspace_size(n) bytes (16-byte aligned). */
size_t pa_mse_fwd_workspace_size(size_t n);
int pa_mse_fwd_ws(const float* pred, const float* target, float* loss, size_t n, void* workspace,
                  size_t workspace_bytes, pa_stream_t stream);
/* dpred += 2/n * (pred - target) * dloss[0]. Replaces launch_mse_backward (Launchers.cuh:107-114). */
int pa_mse_bwd(const float* pred, const float* target, const float* dloss, float* dpred, size_t n,
               pa_stream_t stream);
/* Adam update with host-computed bias corrections c1 = 1 - beta1^t, c2 = 1 - beta2^t.
 * Replaces launch_adam_step (Launchers.cuh:124-137). */
int pa_adam_step(float* param, const float* grad, float* m, float* v, size_t n, float lr,
                 float beta1, float beta2, float eps, float bias_corr1, float bias_corr2,
                 pa_stream_t stream);
/* The same update for `count` tensors (host arrays of device pointers and
 * sizes) in one launch per 48 tensors, instead of the reference's launch per
 * parameter (Adam.cpp:28-59). Elementwise results equal pa_adam_step's. */
int pa_adam_step_multi(float* const* params, const float* const* grads, float* const* m,
                       float* const* v, const size_t* sizes, int count, float lr, float beta1,
                       float beta2, float eps, float bias_corr1, float bias_corr2,
                       pa_stream_t stream);
/* x[i] ~ N(0, std_dev^2) from a counter-based generator keyed by seed
 * (reproducible). Replaces launch_normal_population (Launchers.cuh:56-62),
 * which seeded from the clock. */
int pa_fill_normal(float* x, size_t n, float std_dev, uint64_t seed, pa_stream_t stream);
/* x[i] = value. */
int pa_fill(float* x, size_t n, float value, pa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PA_KERNELS_H */
