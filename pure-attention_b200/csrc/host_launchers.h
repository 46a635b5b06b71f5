// Host launchers behind the C ABI (one definition per kernel translation unit).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include "attn_common.cuh"

namespace pa {

// fp32_split.cu: the calling thread's pa_f32_math mode
int f32_math();
void set_f32_math(int mode);

// attn_fwd.cu
int launch_attn_fwd_bf16(const AttnShape& sh, const void* q, const void* k, const void* v, void* o,
                         float* lse, uint32_t* status, cudaStream_t stream);
int launch_attn_fwd_f32(const AttnShape& sh, const void* q, const void* k, const void* v, void* o,
                        float* lse, void* ws, uint32_t* status, cudaStream_t stream);
size_t attn_fwd_workspace_bytes_f32(const AttnShape& sh);
int f32_plane_dim(int D);  // padded head dim of the fp32 path's bf16 planes (-1: unsupported)

// fp32_split.cu: x [rows, D] fp32 -> hi, lo [rows, Dp] bf16 (zero-padded).
int launch_split_planes(const float* x, void* hi, void* lo, size_t rows, int D, int Dp,
                        cudaStream_t s);
// Same, into columns [c0, c0 + Dp) of planes with row pitch ldp (elements).
int launch_split_planes_into(const float* x, void* hi, void* lo, size_t rows, int D, int Dp,
                             size_t ldp, int c0, cudaStream_t s);
// Same, x taken as zero where mask (same layout as x) <= 0.
int launch_split_planes_masked(const float* x, const float* mask, void* hi, void* lo, size_t rows,
                               int D, int Dp, size_t ldp, int c0, cudaStream_t s);

// attn_bwd.cu
size_t attn_bwd_workspace_bytes(const AttnShape& sh);
size_t attn_bwd_workspace_bytes_f32(const AttnShape& sh);
int launch_attn_bwd_bf16(const AttnShape& sh, const void* q, const void* k, const void* v,
                         const void* o, const void* dO, const float* lse, void* dq, void* dk,
                         void* dv, int accumulate, void* ws, uint32_t* status, cudaStream_t stream);
int launch_attn_bwd_f32(const AttnShape& sh, const void* q, const void* k, const void* v,
                        const void* o, const void* dO, const float* lse, void* dq, void* dk,
                        void* dv, int accumulate, void* ws, uint32_t* status, cudaStream_t stream,
                        const void* kept = nullptr, bool kept_lo = false);
int launch_attn_delta_bf16(const AttnShape& sh, const void* dO, const void* o, float* delta,
                           cudaStream_t stream);
int launch_attn_delta_f32(const AttnShape& sh, const void* dO, const void* o, float* delta,
                          cudaStream_t stream);

}  // namespace pa

namespace pa {

// layernorm.cu
// r == nullptr: y = LN(x); else sum = x + r and y = LN(sum). ph (and pl):
// y's bf16 hi (and lo) operand planes, row pitch pld = N rounded up to 8
// (zero padding), written from the same values as y.
int launch_layer_norm_fwd(const float* x, const float* r, float* sum, const float* g,
                          const float* b, float* y, float* mu, float* rs, uint32_t M, uint32_t N,
                          float eps, cudaStream_t s, void* ph = nullptr, void* pl = nullptr,
                          uint32_t pld = 0);
size_t layer_norm_bwd_workspace_bytes(uint32_t M, uint32_t N);
int launch_layer_norm_bwd(const float* dy, const float* x, const float* mu, const float* rs,
                          const float* g, float* dx, float* dg, float* db, uint32_t M, uint32_t N,
                          float* part, int accumulate_dx, cudaStream_t s);
// Backward of sum = x + r, y = LN(sum): dx (+)= G and dr (+)= G with
// G = LN_bwd(dy) + dsum (dsum may be null; dx or dr may be null).
int launch_add_layer_norm_bwd(const float* dy, const float* dsum, const float* x, const float* mu,
                              const float* rs, const float* g, float* dx, int acc_dx, float* dr,
                              int acc_dr, float* dg, float* db, uint32_t M, uint32_t N,
                              float* part, cudaStream_t s);

// elementwise.cu
int launch_bias_add(const float* a, const float* bias, float* out, uint32_t M, uint32_t N,
                    cudaStream_t s);
int launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t s);
int launch_bias_grad(const float* dy, float* db, uint32_t M, uint32_t N, cudaStream_t s);
// With ws (bias_grad_workspace_bytes): two stages over the whole GPU; without: one pass.
size_t bias_grad_workspace_bytes(uint32_t M, uint32_t N);
int launch_bias_grad_masked(const float* dy, const float* mask, float* db, uint32_t M, uint32_t N,
                            float* ws, cudaStream_t s);
// launch_split_planes_masked of dy [M, D] and db += its (masked) column sums,
// in one pass over dy when the shapes allow (ws: bias_grad_workspace_bytes(M, D)).
int launch_split_planes_colsum(const float* dy, const float* mask, void* hi, void* lo,
                               uint32_t M, int D, int Dp, size_t ldp, int c0, float* db,
                               float* ws, cudaStream_t s);
int launch_split_last_dim(const float* in, float* const* outs, uint32_t parts, uint32_t rows,
                          uint32_t width, cudaStream_t s);
int launch_concat_last_dim_grad(const float* const* grads, float* grad_in, uint32_t parts,
                                uint32_t rows, uint32_t width, cudaStream_t s);

// gemm.cu: C (=|+=) op(A) op(B), fp32 in/out.
//   mode 0: C[M,N]  = A[M,K] B[K,N]
//   mode 1: C[M,N] += A[M,K] B[N,K]^T   (grad X: A = dY, B = W)
//   mode 2: C[N,K] += A[M,N]^T B[M,K]   (grad W: A = X,  B = dY)
int launch_gemm_f32(int mode, const float* A, const float* B, float* C, int M, int N, int K,
                    void* ws, uint32_t* status, cudaStream_t s);
size_t gemm_workspace_bytes(int M, int N, int K);
// Projection Y[M, OUT] = X[M, IN] W[IN, OUT] (+ bias) written as n_outs column
// blocks of OUT / n_outs (n_outs <= 3); backward from n_parts column-block
// gradients, accumulating into dx, dw, dbias (each may be null).
size_t linear_workspace_bytes(int M, int IN, int OUT);
// relu: Y = max(0, X W + bias). relu_out (backward, n_parts = 1): that Y,
// whose sign masks dy.
// kept (optional): X's operand planes, written by the forward (linear_kept_bytes
// for the math mode) and read by the backward instead of converting X again.
// kept: X's planes (written here, or already there when kept_valid); y_planes:
// Y's planes too (single output), in the kept layout of a projection reading Y.
int launch_linear_fwd(const float* x, const float* w, const float* bias, float* const* outs,
                      int n_outs, int M, int IN, int OUT, int relu, void* ws, uint32_t* status,
                      cudaStream_t s, void* kept = nullptr, int kept_valid = 0,
                      void* y_planes = nullptr);
int launch_linear_bwd(const float* x, const float* w, const float* const* dy_parts, int n_parts,
                      const float* relu_out, float* dx, float* dw, float* dbias, int M, int IN,
                      int OUT, void* ws, uint32_t* status, cudaStream_t s,
                      const void* kept = nullptr, int dx_accumulate = 1);
size_t linear_kept_bytes(int M, int IN, int mode);

// training.cu
int launch_relu_fwd(const float* x, float* y, size_t n, cudaStream_t s);
int launch_adam_multi(float* const* w, const float* const* g, float* const* m, float* const* v,
                      const size_t* n, int count, float lr, float b1, float b2, float eps, float c1,
                      float c2, cudaStream_t s);
int launch_relu_bwd(const float* dy, const float* x, float* dx, size_t n, cudaStream_t s);
size_t mse_workspace_bytes(size_t n);
int launch_mse_fwd(const float* p, const float* t, float* loss, size_t n, float* ws, cudaStream_t s);
int launch_mse_bwd(const float* p, const float* t, const float* dl, float* dp, size_t n,
                   cudaStream_t s);
int launch_adam(float* w, const float* g, float* m, float* v, size_t n, float lr, float b1, float b2,
                float eps, float c1, float c2, cudaStream_t s);
int launch_fill_normal(float* x, size_t n, float std_dev, uint64_t seed, cudaStream_t s);
int launch_fill(float* x, size_t n, float value, cudaStream_t s);

}  // namespace pa
