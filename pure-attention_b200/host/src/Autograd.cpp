#include "core/Autograd.h"

#include <stdexcept>

#include "device_util.h"

namespace core {

namespace {
cudaStream_t stream() { return CudaContext::getStream(); }
size_t rows_of(const Tensor& t) { return t.numel() / last_dim(t); }
}  // namespace

MatMulFunction::MatMulFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> w,
                               std::shared_ptr<Tensor> y)
    : X_input(std::move(x)), W_input(std::move(w)), Y_output(y) {}

// X [..., in] flattened to M rows, W [in, out]: dX += dY W^T, dW += X^T dY.
void MatMulFunction::apply_backward() {
  auto Y = Y_output.lock();
  if (!Y || !Y->get_gradient_ptr()) return;
  const int in = static_cast<int>(W_input->get_shape()[0]);
  const int out = static_cast<int>(W_input->get_shape()[1]);
  const int M = static_cast<int>(rows_of(*X_input));
  Scratch ws(pa_matmul_workspace_size(M, in, out), stream());
  if (X_input->requires_grad())
    check_status(pa_matmul_grad_x(Y->get_gradient_ptr(), W_input->get_data_ptr(),
                                  X_input->get_gradient_ptr(), M, in, out, ws.get(), ws.size(),
                                  ps(stream())),
                 "matmul grad X");
  if (W_input->requires_grad())
    check_status(pa_matmul_grad_w(X_input->get_data_ptr(), Y->get_gradient_ptr(),
                                  W_input->get_gradient_ptr(), M, in, out, ws.get(), ws.size(),
                                  ps(stream())),
                 "matmul grad W");
}

AddFunction::AddFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> bias,
                         std::shared_ptr<Tensor> y)
    : X_input(std::move(x)), bias_input(std::move(bias)), Y_output(y) {}

void AddFunction::apply_backward() {
  auto Y = Y_output.lock();
  if (!Y || !Y->get_gradient_ptr()) return;
  const size_t n = Y->numel();
  if (X_input->requires_grad())
    check_status(pa_grad_accumulate(Y->get_gradient_ptr(), X_input->get_gradient_ptr(), n,
                                    ps(stream())),
                 "add grad");
  if (bias_input->requires_grad()) {
    if (bias_input->numel() == n) {
      check_status(pa_grad_accumulate(Y->get_gradient_ptr(), bias_input->get_gradient_ptr(), n,
                                      ps(stream())),
                   "add grad");
    } else {
      const int N = static_cast<int>(bias_input->numel());
      const int M = static_cast<int>(n / N);
      Scratch ws(pa_bias_grad_workspace_size(M, N), stream());
      check_status(pa_bias_grad_ws(Y->get_gradient_ptr(), bias_input->get_gradient_ptr(), M, N,
                                   ws.get(), ws.size(), ps(stream())),
                   "bias grad");
    }
  }
}

ReLUFunction::ReLUFunction(std::shared_ptr<Tensor> in, std::shared_ptr<Tensor> out)
    : Input(std::move(in)), Output(out) {}

void ReLUFunction::apply_backward() {
  auto Y = Output.lock();
  if (!Y || !Y->get_gradient_ptr() || !Input->requires_grad()) return;
  check_status(pa_relu_bwd(Y->get_gradient_ptr(), Input->get_data_ptr(), Input->get_gradient_ptr(),
                           Input->numel(), ps(stream())),
               "relu backward");
}

MSEFunction::MSEFunction(const std::shared_ptr<Tensor>& preds, const std::shared_ptr<Tensor>& targs,
                         const std::shared_ptr<Tensor>& out)
    : predictions(preds), targets(targs), output_loss(out) {}

void MSEFunction::apply_backward() {
  auto L = output_loss.lock();
  if (!L || !L->get_gradient_ptr() || !predictions->requires_grad()) return;
  check_status(pa_mse_bwd(predictions->get_data_ptr(), targets->get_data_ptr(),
                          L->get_gradient_ptr(), predictions->get_gradient_ptr(),
                          predictions->numel(), ps(stream())),
               "mse backward");
}

LinearFunction::LinearFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> w,
                               std::shared_ptr<Tensor> b, std::vector<std::shared_ptr<Tensor>> outs,
                               bool relu_)
    : X_input(std::move(x)), W_input(std::move(w)), bias_input(std::move(b)),
      Outputs(outs.begin(), outs.end()), relu(relu_) {}

// dX += dY W^T, dW += X^T dY, dbias += column sums of dY, with dY the column
// blocks' gradients (a block whose tensor has expired contributes zero).
void LinearFunction::apply_backward() {
  const int K = static_cast<int>(W_input->get_shape()[0]);
  const int N = static_cast<int>(W_input->get_shape()[1]);
  const int M = static_cast<int>(rows_of(*X_input));
  const int parts = static_cast<int>(Outputs.size());
  const size_t part_bytes = static_cast<size_t>(M) * (N / parts) * sizeof(float);
  float* dX = X_input->requires_grad() ? X_input->get_gradient_ptr() : nullptr;
  float* dW = W_input->requires_grad() ? W_input->get_gradient_ptr() : nullptr;
  float* db = bias_input->requires_grad() ? bias_input->get_gradient_ptr() : nullptr;
  if (relu) {  // the saved output's sign masks its gradient inside the call
    auto Y = Outputs[0].lock();
    if (!Y || !Y->get_gradient_ptr()) return;
    Scratch ws(pa_linear_workspace_size(M, K, N), stream());
    const float* dy = Y->get_gradient_ptr();
    check_status(pa_linear_bwd_kept(X_input->get_data_ptr(), W_input->get_data_ptr(), kept.get(),
                                    kept_bytes, kept_mode, Y->get_data_ptr(), &dy, 1, dX, dW, db,
                                    M, K, N, ws.get(), ws.size(), ps(stream())),
                 "linear + ReLU backward");
    return;
  }
  std::vector<const float*> grads;
  std::vector<std::unique_ptr<Scratch>> zeros;
  bool any = false;
  for (auto& w : Outputs) {
    auto t = w.lock();
    if (t && t->get_gradient_ptr()) {
      grads.push_back(t->get_gradient_ptr());
      any = true;
    } else {
      zeros.push_back(std::make_unique<Scratch>(part_bytes, stream()));
      cudaMemsetAsync(zeros.back()->get(), 0, part_bytes, stream());
      grads.push_back(static_cast<const float*>(zeros.back()->get()));
    }
  }
  if (!any) return;
  Scratch ws(pa_linear_workspace_size(M, K, N), stream());
  check_status(pa_linear_bwd_kept(X_input->get_data_ptr(), W_input->get_data_ptr(), kept.get(),
                                  kept_bytes, kept_mode, nullptr, grads.data(), parts, dX, dW, db,
                                  M, K, N, ws.get(), ws.size(), ps(stream())),
               "linear backward");
}

SplitFunction::SplitFunction(std::shared_ptr<Tensor> in, std::vector<std::shared_ptr<Tensor>> outs)
    : Input(std::move(in)), Outputs(outs.begin(), outs.end()) {}

void SplitFunction::apply_backward() {
  if (!Input->requires_grad()) return;
  std::vector<const float*> grads;
  uint32_t width = 0;
  for (auto& w : Outputs) {
    auto t = w.lock();
    grads.push_back(t ? t->get_gradient_ptr() : nullptr);  // expired part: zero gradient
    if (t) width = static_cast<uint32_t>(last_dim(*t));
  }
  if (width == 0) return;
  const uint32_t parts = static_cast<uint32_t>(Outputs.size());
  const uint32_t rows = static_cast<uint32_t>(Input->numel() / (static_cast<size_t>(width) * parts));
  check_status(pa_concat_last_dim_grad(grads.data(), Input->get_gradient_ptr(), parts, rows, width,
                                       ps(stream())),
               "split backward");
}

FlashAttentionFunction::FlashAttentionFunction(const std::shared_ptr<Tensor>& q,
                                               const std::shared_ptr<Tensor>& k,
                                               const std::shared_ptr<Tensor>& v,
                                               const std::shared_ptr<Tensor>& o,
                                               const std::shared_ptr<Tensor>& lcache, int heads)
    : Q_input(q), K_input(k), V_input(v), O_output(o), L_cache(lcache), num_heads(heads) {}

// Gradients are added straight into Q/K/V's grads (accumulate = 1): no
// temporaries, unlike the reference's three cudaMallocAsync'd buffers.
void FlashAttentionFunction::apply_backward() {
  auto O = O_output.lock();
  if (!O || !O->get_gradient_ptr()) return;
  const auto sh = Q_input->get_shape();
  pa_attn_desc d{static_cast<int32_t>(sh[0]), static_cast<int32_t>(sh[1]), num_heads,
                 static_cast<int32_t>(sh[2]) / num_heads, PA_F32, 0.f};
  Scratch ws(pa_attn_bwd_workspace_size(&d), stream());
  const size_t n = Q_input->numel();
  // Inputs without a gradient get a throwaway buffer.
  Scratch sink((Q_input->requires_grad() && K_input->requires_grad() && V_input->requires_grad())
                   ? 0
                   : n * sizeof(float),
               stream());
  auto g = [&](const std::shared_ptr<Tensor>& t) {
    return t->requires_grad() ? static_cast<void*>(t->get_gradient_ptr()) : sink.get();
  };
  check_status(pa_attn_bwd(&d, Q_input->get_data_ptr(), K_input->get_data_ptr(),
                           V_input->get_data_ptr(), O->get_data_ptr(), O->get_gradient_ptr(),
                           L_cache->get_data_ptr(), g(Q_input), g(K_input), g(V_input), 1, ws.get(),
                           ws.size(), ps(stream())),
               "FlashAttention Backward");
}

LayerNormFunction::LayerNormFunction(const std::shared_ptr<Tensor>& inp,
                                     const std::shared_ptr<Tensor>& g,
                                     const std::shared_ptr<Tensor>& b,
                                     const std::shared_ptr<Tensor>& out,
                                     const std::shared_ptr<Tensor>& m,
                                     const std::shared_ptr<Tensor>& r, uint32_t m_size,
                                     uint32_t n_size)
    : input(inp), gamma(g), beta(b), output(out), mean(m), rstd(r), M(m_size), N(n_size) {}

// dX is accumulated by the kernel into the input's gradient, which may
// already hold a residual branch's contribution (the reference's node
// overwrites it, source/core/Autograd.cpp:257-280).
void LayerNormFunction::apply_backward() {
  auto Y = output.lock();
  if (!Y || !Y->get_gradient_ptr()) return;
  Scratch ws(pa_layer_norm_bwd_workspace_size(M, N), stream());
  check_status(pa_layer_norm_bwd_accumulate(
                   Y->get_gradient_ptr(), input->get_data_ptr(), mean->get_data_ptr(),
                   rstd->get_data_ptr(), gamma->get_data_ptr(),
                   input->requires_grad() ? input->get_gradient_ptr() : nullptr,
                   gamma->requires_grad() ? gamma->get_gradient_ptr() : nullptr,
                   beta->requires_grad() ? beta->get_gradient_ptr() : nullptr, M, N, ws.get(),
                   ws.size(), ps(stream())),
               "LayerNorm backward");
}

}  // namespace core
