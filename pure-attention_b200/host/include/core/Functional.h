// Functional ops: allocate the output, launch the forward kernel through the
// C ABI and attach the graph node. Names and signatures follow the
// reference's include/core/Functional.h:9-76.
#pragma once
#include <cuda_runtime.h>
#include <memory>
#include <utility>
#include <vector>
#include "core/Tensor.h"

namespace core {
// C = A B with A [..., K] flattened to rows and B [K, N] (2-D weights).
void matmul(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& B,
            std::shared_ptr<Tensor>& C, const cudaStream_t& stream);
// B = A + X: X of shape [1, N] (or [N]) is a row-broadcast bias; X with A's
// shape is added elementwise.
void matadd(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& X,
            std::shared_ptr<Tensor>& B, const cudaStream_t& stream);
std::shared_ptr<Tensor> relu(const std::shared_ptr<Tensor>& In, const cudaStream_t& stream);
void pop_data_zeros(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream);
void pop_grad_zeros(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream);
void pop_grad_zeros(Tensor* A, const cudaStream_t& stream);
void pop_grad_ones(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream);
void pop_grad_ones(Tensor* A, const cudaStream_t& stream);
void pop_data_normal(const std::shared_ptr<Tensor>& A, float std_dev, const cudaStream_t& stream);
std::shared_ptr<Tensor> mse_loss(const std::shared_ptr<Tensor>& preds,
                                 const std::shared_ptr<Tensor>& targets,
                                 const cudaStream_t& stream);
// Fused projection (no single reference counterpart: core::matmul + core::matadd
// + core::split in one pass, Functional.cpp:12-52, 205-252): parts receive the
// num_parts column blocks of A W + bias, with one LinearFunction node; with
// relu (num_parts = 1) the block is max(0, A W + bias).
void linear(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& W,
            const std::shared_ptr<Tensor>& bias, uint32_t num_parts,
            std::vector<std::shared_ptr<Tensor>>& parts, const cudaStream_t& stream,
            bool relu = false);

void split(const std::shared_ptr<Tensor>& A, uint32_t num_parts, int dim,
           std::vector<std::shared_ptr<Tensor>>& parts, const cudaStream_t& stream);
// Q, K, V [N, L, E] with E = num_heads * head_dim (head_dim 32 or 64, fp32).
void flash_attention(const std::shared_ptr<Tensor>& Q, const std::shared_ptr<Tensor>& K,
                     const std::shared_ptr<Tensor>& V, std::shared_ptr<Tensor>& O, int num_heads,
                     const cudaStream_t& stream);
std::shared_ptr<Tensor> layer_norm(const std::shared_ptr<Tensor>& input,
                                   const std::shared_ptr<Tensor>& gamma,
                                   const std::shared_ptr<Tensor>& beta, float epsilon,
                                   const cudaStream_t& stream);
// sum = x + r and y = LayerNorm(sum) in one kernel; returns {sum, y}. sum's
// node is the add (its gradient goes to x and r), y's the norm over sum.
std::pair<std::shared_ptr<Tensor>, std::shared_ptr<Tensor>> add_layer_norm(
    const std::shared_ptr<Tensor>& x, const std::shared_ptr<Tensor>& r,
    const std::shared_ptr<Tensor>& gamma, const std::shared_ptr<Tensor>& beta, float epsilon,
    const cudaStream_t& stream);
}  // namespace core
