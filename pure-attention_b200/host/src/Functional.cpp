#include "core/Functional.h"

#include <stdexcept>
#include <string>

#include "core/Autograd.h"
#include "device_util.h"

namespace core {

void matmul(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& B,
            std::shared_ptr<Tensor>& C, const cudaStream_t& stream) {
  const auto a = A->get_shape(), b = B->get_shape();
  if (b.size() != 2) throw std::runtime_error("Matmul: B (weights) must be 2D");
  if (a.empty() || a.back() != b[0])
    throw std::runtime_error("Matmul: Dimension mismatch A[..., K] and B[K, N]");
  const int K = static_cast<int>(b[0]), N = static_cast<int>(b[1]);
  const int M = static_cast<int>(A->numel() / K);
  auto cs = a;
  cs.back() = static_cast<uint32_t>(N);
  const bool g = A->requires_grad() || B->requires_grad();
  C = std::make_shared<Tensor>(cs, g, false);
  Scratch ws(pa_matmul_workspace_size(M, N, K), stream);
  check_status(pa_matmul(A->get_data_ptr(), B->get_data_ptr(), C->get_data_ptr(), M, N, K, ws.get(),
                         ws.size(), ps(stream)),
               "Matmul");
  if (g) C->set_grad_fn(std::make_shared<MatMulFunction>(A, B, C));
}

void matadd(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& X,
            std::shared_ptr<Tensor>& B, const cudaStream_t& stream) {
  const bool g = A->requires_grad() || X->requires_grad();
  B = std::make_shared<Tensor>(A->get_shape(), g, false);
  const size_t n = A->numel(), N = last_dim(*A);
  if (X->numel() == n) {
    check_status(pa_add(A->get_data_ptr(), X->get_data_ptr(), B->get_data_ptr(), n, ps(stream)),
                 "Add");
  } else if (X->numel() == N) {
    check_status(pa_bias_add(A->get_data_ptr(), X->get_data_ptr(), B->get_data_ptr(),
                             static_cast<int>(n / N), static_cast<int>(N), ps(stream)),
                 "Bias add");
  } else {
    throw std::runtime_error("Add: second operand must match the first or its last dimension");
  }
  if (g) B->set_grad_fn(std::make_shared<AddFunction>(A, X, B));
}

std::shared_ptr<Tensor> relu(const std::shared_ptr<Tensor>& In, const cudaStream_t& stream) {
  auto Out = std::make_shared<Tensor>(In->get_shape(), In->requires_grad(), false);
  check_status(pa_relu_fwd(In->get_data_ptr(), Out->get_data_ptr(), In->numel(), ps(stream)), "ReLU");
  if (In->requires_grad()) Out->set_grad_fn(std::make_shared<ReLUFunction>(In, Out));
  return Out;
}

void pop_data_zeros(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream) {
  cudaMemsetAsync(A->get_data_ptr(), 0, A->numel() * sizeof(float), stream);
}
void pop_grad_zeros(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream) {
  pop_grad_zeros(A.get(), stream);
}
void pop_grad_zeros(Tensor* A, const cudaStream_t& stream) {
  bool unwritten = false;
  if (float* g = A->gradient_for_write(&unwritten))
    cudaMemsetAsync(g, 0, A->numel() * sizeof(float), stream);
}
void pop_grad_ones(const std::shared_ptr<Tensor>& A, const cudaStream_t& stream) {
  pop_grad_ones(A.get(), stream);
}
void pop_grad_ones(Tensor* A, const cudaStream_t& stream) {
  bool unwritten = false;
  if (float* g = A->gradient_for_write(&unwritten))
    check_status(pa_fill(g, A->numel(), 1.0f, ps(stream)), "fill");
}
void pop_data_normal(const std::shared_ptr<Tensor>& A, float std_dev, const cudaStream_t& stream) {
  check_status(pa_fill_normal(A->get_data_ptr(), A->numel(), std_dev, CudaContext::nextSeed(),
                              ps(stream)),
               "fill_normal");
}

std::shared_ptr<Tensor> mse_loss(const std::shared_ptr<Tensor>& preds,
                                 const std::shared_ptr<Tensor>& targets,
                                 const cudaStream_t& stream) {
  if (preds->numel() != targets->numel())
    throw std::runtime_error("MSE: predictions and targets differ in size");
  auto loss = std::make_shared<Tensor>(std::vector<uint32_t>{1}, preds->requires_grad(), false);
  Scratch ws(pa_mse_fwd_workspace_size(preds->numel()), stream);
  check_status(pa_mse_fwd_ws(preds->get_data_ptr(), targets->get_data_ptr(), loss->get_data_ptr(),
                             preds->numel(), ws.get(), ws.size(), ps(stream)),
               "MSE");
  if (preds->requires_grad()) loss->set_grad_fn(std::make_shared<MSEFunction>(preds, targets, loss));
  return loss;
}

void linear(const std::shared_ptr<Tensor>& A, const std::shared_ptr<Tensor>& W,
            const std::shared_ptr<Tensor>& bias, uint32_t num_parts,
            std::vector<std::shared_ptr<Tensor>>& parts, const cudaStream_t& stream, bool relu) {
  const auto a = A->get_shape(), w = W->get_shape();
  if (w.size() != 2) throw std::runtime_error("Linear: W (weights) must be 2D");
  if (a.empty() || a.back() != w[0])
    throw std::runtime_error("Linear: Dimension mismatch A[..., K] and W[K, N]");
  const int K = static_cast<int>(w[0]), N = static_cast<int>(w[1]);
  if (bias->numel() != static_cast<size_t>(N))
    throw std::runtime_error("Linear: bias must have W's output dimension");
  if (num_parts < 1 || num_parts > 3 || N % num_parts || (relu && num_parts != 1))
    throw std::runtime_error("Linear: 1 to 3 parts, dividing the output dimension");
  const int M = static_cast<int>(A->numel() / K);
  const bool g = A->requires_grad() || W->requires_grad() || bias->requires_grad();
  auto ps_ = a;
  ps_.back() = static_cast<uint32_t>(N / num_parts);
  std::vector<std::shared_ptr<Tensor>> mine;
  std::vector<float*> outs;
  for (uint32_t i = 0; i < num_parts; ++i) {
    mine.push_back(std::make_shared<Tensor>(ps_, g, false));
    outs.push_back(mine.back()->get_data_ptr());
  }
  Scratch ws(pa_linear_workspace_size(M, K, N), stream);
  // X's operand planes: from X's producer where they serve this math mode (no
  // conversion), else converted here; with gradients the node keeps them for
  // the backward. A hidden layer (Linear + ReLU) also writes its output's
  // planes for the projection that reads it next.
  const int mode = pa_get_f32_math();
  const size_t need = pa_linear_kept_size(M, K);
  const bool have = A->operand_planes && A->operand_planes_bytes >= need &&
                    (mode == PA_F32_MATH_BF16 || A->operand_planes_mode == PA_F32_MATH_SPLIT3);
  std::shared_ptr<void> kept;
  size_t kept_bytes = need;
  int kept_mode = mode;
  if (have) {
    kept = A->operand_planes;
    kept_bytes = A->operand_planes_bytes;
    kept_mode = A->operand_planes_mode;
  } else if (g || relu) {
    kept = device_buffer(kept_bytes, stream, "Linear");
  }
  std::shared_ptr<void> y_planes;
  size_t y_bytes = 0;
  if (relu) {
    y_bytes = pa_linear_kept_size(M, N);
    y_planes = device_buffer(y_bytes, stream, "Linear + ReLU");
  }
  if (kept) {
    check_status(pa_linear_fwd_planes(A->get_data_ptr(), W->get_data_ptr(), bias->get_data_ptr(),
                                      outs.data(), static_cast<int>(num_parts), relu ? 1 : 0, M, K,
                                      N, kept.get(), kept_bytes, kept_mode,
                                      have ? PA_LINEAR_KEPT_VALID : 0, y_planes.get(), y_bytes,
                                      ws.get(), ws.size(), ps(stream)),
                 relu ? "Linear + ReLU" : "Linear");
  } else {
    check_status(pa_linear_fwd(A->get_data_ptr(), W->get_data_ptr(), bias->get_data_ptr(),
                               outs.data(), static_cast<int>(num_parts), M, K, N, ws.get(),
                               ws.size(), ps(stream)),
                 "Linear");
  }
  if (y_planes) {
    mine[0]->operand_planes = y_planes;
    mine[0]->operand_planes_bytes = y_bytes;
    mine[0]->operand_planes_mode = mode;
  }
  std::shared_ptr<LinearFunction> node;
  if (g) {
    node = std::make_shared<LinearFunction>(A, W, bias, mine, relu);
    node->kept = kept;
    node->kept_bytes = kept_bytes;
    node->kept_mode = kept_mode;
  }
  if (g) {
    for (auto& p : mine) p->set_grad_fn(node);
  }
  parts.insert(parts.end(), mine.begin(), mine.end());
}

void split(const std::shared_ptr<Tensor>& A, uint32_t num_parts, int dim,
           std::vector<std::shared_ptr<Tensor>>& parts, const cudaStream_t& stream) {
  auto shape = A->get_shape();
  const int rank = static_cast<int>(shape.size());
  while (dim < 0) dim += rank;
  if (dim != rank - 1) throw std::runtime_error("Only split on last dimension is currently supported!");
  if (num_parts == 0 || shape[dim] % num_parts)
    throw std::runtime_error("Split dimension must be divisible by num_parts");
  const uint32_t width = shape[dim] / num_parts;
  const uint32_t rows = static_cast<uint32_t>(A->numel() / shape[dim]);
  shape[dim] = width;
  std::vector<float*> outs;
  for (uint32_t i = 0; i < num_parts; ++i) {
    parts.push_back(std::make_shared<Tensor>(shape, A->requires_grad(), false));
    outs.push_back(parts.back()->get_data_ptr());
  }
  check_status(pa_split_last_dim(A->get_data_ptr(), outs.data(), num_parts, rows, width, ps(stream)),
               "Split");
  if (A->requires_grad()) {
    std::vector<std::shared_ptr<Tensor>> mine(parts.end() - num_parts, parts.end());
    auto node = std::make_shared<SplitFunction>(A, mine);
    for (auto& p : mine) p->set_grad_fn(node);
  }
}

void flash_attention(const std::shared_ptr<Tensor>& Q, const std::shared_ptr<Tensor>& K,
                     const std::shared_ptr<Tensor>& V, std::shared_ptr<Tensor>& O, int num_heads,
                     const cudaStream_t& stream) {
  const auto sh = Q->get_shape();
  if (sh.size() != 3 || K->get_shape() != sh || V->get_shape() != sh)
    throw std::runtime_error("FlashAttention: Q, K, V must share a [N, L, E] shape");
  if (num_heads <= 0 || sh[2] % num_heads)
    throw std::runtime_error("FlashAttention: embedding dim not divisible by num_heads");
  const bool g = Q->requires_grad() || K->requires_grad() || V->requires_grad();
  O = std::make_shared<Tensor>(sh, g, false);
  // One log-sum-exp per (batch, head, query row).
  auto L_cache = std::make_shared<Tensor>(
      std::vector<uint32_t>{sh[0] * static_cast<uint32_t>(num_heads), sh[1]}, false, false);
  pa_attn_desc d{static_cast<int32_t>(sh[0]), static_cast<int32_t>(sh[1]), num_heads,
                 static_cast<int32_t>(sh[2]) / num_heads, PA_F32, 0.f};
  // With gradients, the workspace (Q, K, V's bf16 operand planes) stays with
  // the graph node, so the backward does not convert them again.
  const size_t ws_bytes = pa_attn_fwd_workspace_size(&d);
  std::shared_ptr<void> ws;
  if (ws_bytes) {
    void* p = nullptr;
    retain_pool_memory();
    if (cudaMallocAsync(&p, ws_bytes, stream) != cudaSuccess)
      throw std::runtime_error("FlashAttention: cannot allocate the workspace");
    ws = std::shared_ptr<void>(p, [](void* q) { cudaFreeAsync(q, CudaContext::getStream()); });
  }
  const int st = pa_attn_fwd(&d, Q->get_data_ptr(), K->get_data_ptr(), V->get_data_ptr(),
                             O->get_data_ptr(), L_cache->get_data_ptr(), ws.get(), ws_bytes,
                             ps(stream));
  if (st == PA_ERR_UNSUPPORTED)
    throw std::runtime_error("FlashAttention: Unsupported Head Dimension");
  check_status(st, "FlashAttention");
  if (g) {
    auto node = std::make_shared<FlashAttentionFunction>(Q, K, V, O, L_cache, num_heads);
    node->kept = ws;
    node->kept_bytes = ws_bytes;
    node->kept_mode = pa_get_f32_math();
    O->set_grad_fn(node);
  }
}

// A LayerNorm output's operand planes (pa_layer_norm_fwd_planes), attached to
// it so that a projection reading it converts nothing. NULL where the plane
// layout cannot describe the shape (more than INT_MAX rows or columns): the
// norm then writes y alone and a projection converts it.
static std::shared_ptr<void> ln_planes(const std::shared_ptr<Tensor>& out, uint32_t M, uint32_t N,
                                       const cudaStream_t& stream) {
  if (M > 0x7fffffffu || N > 0x7fffffffu) return nullptr;
  const size_t bytes = pa_linear_kept_size(static_cast<int>(M), static_cast<int>(N));
  if (bytes == 0) return nullptr;
  auto planes = device_buffer(bytes, stream, "LayerNorm");
  out->operand_planes = planes;
  out->operand_planes_bytes = bytes;
  out->operand_planes_mode = pa_get_f32_math();
  return planes;
}

std::shared_ptr<Tensor> layer_norm(const std::shared_ptr<Tensor>& input,
                                   const std::shared_ptr<Tensor>& gamma,
                                   const std::shared_ptr<Tensor>& beta, float epsilon,
                                   const cudaStream_t& stream) {
  const uint32_t N = static_cast<uint32_t>(last_dim(*input));
  const uint32_t M = static_cast<uint32_t>(input->numel() / N);
  if (gamma->numel() != N || beta->numel() != N)
    throw std::runtime_error("LayerNorm: gamma/beta must have the normalized size");
  const bool g = input->requires_grad() || gamma->requires_grad() || beta->requires_grad();
  auto output = std::make_shared<Tensor>(input->get_shape(), g, false);
  auto mean = std::make_shared<Tensor>(std::vector<uint32_t>{M}, false);
  auto rstd = std::make_shared<Tensor>(std::vector<uint32_t>{M}, false);
  // y's bf16 operand planes from the same pass, for the projection that reads y next
  auto planes = ln_planes(output, M, N, stream);
  check_status(planes ? pa_layer_norm_fwd_planes(input->get_data_ptr(), nullptr, nullptr,
                                                 gamma->get_data_ptr(), beta->get_data_ptr(),
                                                 output->get_data_ptr(), mean->get_data_ptr(),
                                                 rstd->get_data_ptr(), M, N, epsilon, planes.get(),
                                                 output->operand_planes_bytes, ps(stream))
                      : pa_layer_norm_fwd(input->get_data_ptr(), gamma->get_data_ptr(),
                                          beta->get_data_ptr(), output->get_data_ptr(),
                                          mean->get_data_ptr(), rstd->get_data_ptr(), M, N, epsilon,
                                          ps(stream)),
               "LayerNorm");
  if (g)
    output->set_grad_fn(
        std::make_shared<LayerNormFunction>(input, gamma, beta, output, mean, rstd, M, N));
  return output;
}

std::pair<std::shared_ptr<Tensor>, std::shared_ptr<Tensor>> add_layer_norm(
    const std::shared_ptr<Tensor>& x, const std::shared_ptr<Tensor>& r,
    const std::shared_ptr<Tensor>& gamma, const std::shared_ptr<Tensor>& beta, float epsilon,
    const cudaStream_t& stream) {
  const uint32_t N = static_cast<uint32_t>(last_dim(*x));
  const uint32_t M = static_cast<uint32_t>(x->numel() / N);
  if (r->numel() != x->numel())
    throw std::runtime_error("Add+LayerNorm: the residual must have the input's size");
  if (gamma->numel() != N || beta->numel() != N)
    throw std::runtime_error("LayerNorm: gamma/beta must have the normalized size");
  const bool gs = x->requires_grad() || r->requires_grad();
  const bool g = gs || gamma->requires_grad() || beta->requires_grad();
  auto sum = std::make_shared<Tensor>(x->get_shape(), g, false);
  auto output = std::make_shared<Tensor>(x->get_shape(), g, false);
  auto mean = std::make_shared<Tensor>(std::vector<uint32_t>{M}, false);
  auto rstd = std::make_shared<Tensor>(std::vector<uint32_t>{M}, false);
  auto planes = ln_planes(output, M, N, stream);
  check_status(planes ? pa_layer_norm_fwd_planes(x->get_data_ptr(), r->get_data_ptr(),
                                                 sum->get_data_ptr(), gamma->get_data_ptr(),
                                                 beta->get_data_ptr(), output->get_data_ptr(),
                                                 mean->get_data_ptr(), rstd->get_data_ptr(), M, N,
                                                 epsilon, planes.get(), output->operand_planes_bytes,
                                                 ps(stream))
                      : pa_add_layer_norm_fwd(x->get_data_ptr(), r->get_data_ptr(),
                                              sum->get_data_ptr(), gamma->get_data_ptr(),
                                              beta->get_data_ptr(), output->get_data_ptr(),
                                              mean->get_data_ptr(), rstd->get_data_ptr(), M, N,
                                              epsilon, ps(stream)),
               "Add+LayerNorm");
  if (gs) {  // one backward pass writes both addends' gradients
    sum->set_grad_fn(std::make_shared<AddLayerNormFunction>(x, r, gamma, beta, sum, mean, rstd, M, N));
    output->set_grad_fn(std::make_shared<LayerNormOutFunction>(sum, output));
  } else if (g) {  // only gamma / beta need gradients
    output->set_grad_fn(
        std::make_shared<LayerNormFunction>(sum, gamma, beta, output, mean, rstd, M, N));
  }
  return {sum, output};
}

}  // namespace core
