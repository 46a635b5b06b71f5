#include "core/Autograd.h"

#include <stdexcept>
#include <string>

#include "device_util.h"

namespace core {

namespace {
cudaStream_t stream() { return CudaContext::getStream(); }
size_t rows_of(const Tensor& t) { return t.numel() / last_dim(t); }

// The gradient that reached an output, or null when none did (the tensor has
// expired, has no gradient, or nothing has written its gradient: zero).
const float* grad_in(const std::shared_ptr<Tensor>& t) {
  if (!t || !t->requires_grad() || t->gradient_unwritten()) return nullptr;
  return t->get_gradient_ptr();
}

// t.grad += src (n floats), as a copy when nothing has written t.grad yet.
void add_into(const Tensor& t, const float* src, size_t n, const char* what) {
  bool unwritten = false;
  float* dst = t.gradient_for_write(&unwritten);
  if (unwritten) {
    if (cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToDevice, stream()) !=
        cudaSuccess)
      throw std::runtime_error(std::string(what) + ": cudaMemcpyAsync failed");
    return;
  }
  check_status(pa_grad_accumulate(src, dst, n, ps(stream())), what);
}
}  // namespace

MatMulFunction::MatMulFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> w,
                               std::shared_ptr<Tensor> y)
    : X_input(std::move(x)), W_input(std::move(w)), Y_output(y) {}

// X [..., in] flattened to M rows, W [in, out]: dX += dY W^T, dW += X^T dY.
void MatMulFunction::apply_backward() {
  auto Y = Y_output.lock();
  if (!grad_in(Y)) return;
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
  const float* dy = grad_in(Y);
  if (!dy) return;
  const size_t n = Y->numel();
  if (X_input->requires_grad()) add_into(*X_input, dy, n, "add grad");
  if (bias_input->requires_grad()) {
    if (bias_input->numel() == n) {
      add_into(*bias_input, dy, n, "add grad");
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
  if (!grad_in(Y) || !Input->requires_grad()) return;
  check_status(pa_relu_bwd(Y->get_gradient_ptr(), Input->get_data_ptr(), Input->get_gradient_ptr(),
                           Input->numel(), ps(stream())),
               "relu backward");
}

MSEFunction::MSEFunction(const std::shared_ptr<Tensor>& preds, const std::shared_ptr<Tensor>& targs,
                         const std::shared_ptr<Tensor>& out)
    : predictions(preds), targets(targs), output_loss(out) {}

void MSEFunction::apply_backward() {
  auto L = output_loss.lock();
  if (!grad_in(L) || !predictions->requires_grad()) return;
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
// blocks' gradients (a block whose tensor has expired, or that no gradient
// reached, contributes zero). dX is written outright when nothing has written
// it yet.
void LinearFunction::apply_backward() {
  const int K = static_cast<int>(W_input->get_shape()[0]);
  const int N = static_cast<int>(W_input->get_shape()[1]);
  const int M = static_cast<int>(rows_of(*X_input));
  const int parts = static_cast<int>(Outputs.size());
  const size_t part_bytes = static_cast<size_t>(M) * (N / parts) * sizeof(float);
  std::vector<const float*> grads;
  std::vector<std::unique_ptr<Scratch>> zeros;
  std::shared_ptr<Tensor> Y0;
  bool any = false;
  for (auto& w : Outputs) {
    auto t = w.lock();
    if (!Y0) Y0 = t;
    if (const float* g = grad_in(t)) {
      grads.push_back(g);
      any = true;
    } else {
      zeros.push_back(std::make_unique<Scratch>(part_bytes, stream()));
      cudaMemsetAsync(zeros.back()->get(), 0, part_bytes, stream());
      grads.push_back(static_cast<const float*>(zeros.back()->get()));
    }
  }
  if (!any) return;
  // the saved ReLU output's sign masks its gradient inside the call
  const float* y = relu ? Y0->get_data_ptr() : nullptr;
  bool dx_unwritten = false;
  float* dX = X_input->requires_grad() ? X_input->gradient_for_write(&dx_unwritten) : nullptr;
  float* dW = W_input->requires_grad() ? W_input->get_gradient_ptr() : nullptr;
  float* db = bias_input->requires_grad() ? bias_input->get_gradient_ptr() : nullptr;
  Scratch ws(pa_linear_workspace_size(M, K, N), stream());
  check_status(pa_linear_bwd_kept(X_input->get_data_ptr(), W_input->get_data_ptr(), kept.get(),
                                  kept_bytes, kept_mode, y, grads.data(), parts, dX, dW, db, M, K,
                                  N, dx_unwritten ? PA_LINEAR_DX_OVERWRITE : 0, ws.get(),
                                  ws.size(), ps(stream())),
               relu ? "linear + ReLU backward" : "linear backward");
}

SplitFunction::SplitFunction(std::shared_ptr<Tensor> in, std::vector<std::shared_ptr<Tensor>> outs)
    : Input(std::move(in)), Outputs(outs.begin(), outs.end()) {}

void SplitFunction::apply_backward() {
  if (!Input->requires_grad()) return;
  std::vector<const float*> grads;
  uint32_t width = 0;
  for (auto& w : Outputs) {
    auto t = w.lock();
    grads.push_back(grad_in(t));  // expired or unreached part: zero gradient
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

// Gradients go straight into Q/K/V's grads: written outright when nothing
// has written any of them yet (accumulate = 0), else added (accumulate = 1,
// after zeroing those still unwritten). No temporaries, unlike the
// reference's three cudaMallocAsync'd buffers. Q, K, V's bf16 planes come from
// the forward's kept workspace; only dO is converted.
void FlashAttentionFunction::apply_backward() {
  auto O = O_output.lock();
  const float* dO = grad_in(O);
  if (!dO) return;
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
  const std::shared_ptr<Tensor>* qkv[3] = {&Q_input, &K_input, &V_input};
  if (Q_input == K_input || K_input == V_input || Q_input == V_input) {
    // one tensor in two or three roles (self-attention on x itself): the kernels
    // write dQ, dK, dV concurrently, so they go to separate buffers first
    Scratch g3(3 * n * sizeof(float), stream());
    float* gp = static_cast<float*>(g3.get());
    check_status(pa_attn_bwd_kept(&d, Q_input->get_data_ptr(), K_input->get_data_ptr(),
                                  V_input->get_data_ptr(), O->get_data_ptr(), dO,
                                  L_cache->get_data_ptr(), gp, gp + n, gp + 2 * n, 0, kept.get(),
                                  kept_bytes, kept_mode, ws.get(), ws.size(), ps(stream())),
                 "FlashAttention Backward");
    for (int i = 0; i < 3; ++i)
      if ((*qkv[i])->requires_grad()) add_into(**qkv[i], gp + i * n, n, "FlashAttention Backward");
    return;
  }
  void* dst[3];
  bool unwritten[3] = {false, false, false};
  bool all_unwritten = true;
  for (int i = 0; i < 3; ++i) {
    const Tensor& t = **qkv[i];
    if (t.requires_grad()) {
      dst[i] = t.gradient_for_write(&unwritten[i]);
      all_unwritten = all_unwritten && unwritten[i];
    } else {
      dst[i] = sink.get();
    }
  }
  if (!all_unwritten)
    for (int i = 0; i < 3; ++i)
      if (unwritten[i]) cudaMemsetAsync(dst[i], 0, n * sizeof(float), stream());
  check_status(pa_attn_bwd_kept(&d, Q_input->get_data_ptr(), K_input->get_data_ptr(),
                                V_input->get_data_ptr(), O->get_data_ptr(), dO,
                                L_cache->get_data_ptr(), dst[0], dst[1], dst[2],
                                all_unwritten ? 0 : 1, kept.get(), kept_bytes, kept_mode,
                                ws.get(), ws.size(), ps(stream())),
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
// overwrites it, source/core/Autograd.cpp:257-280), or written outright when
// nothing has written that gradient yet.
void LayerNormFunction::apply_backward() {
  auto Y = output.lock();
  const float* dy = grad_in(Y);
  if (!dy) return;
  Scratch ws(pa_layer_norm_bwd_workspace_size(M, N), stream());
  bool unwritten = false;
  float* dx = input->requires_grad() ? input->gradient_for_write(&unwritten) : nullptr;
  float* dg = gamma->requires_grad() ? gamma->get_gradient_ptr() : nullptr;
  float* db = beta->requires_grad() ? beta->get_gradient_ptr() : nullptr;
  auto fn = unwritten ? pa_layer_norm_bwd : pa_layer_norm_bwd_accumulate;
  check_status(fn(dy, input->get_data_ptr(), mean->get_data_ptr(), rstd->get_data_ptr(),
                  gamma->get_data_ptr(), dx, dg, db, M, N, ws.get(), ws.size(), ps(stream())),
               "LayerNorm backward");
}

AddLayerNormFunction::AddLayerNormFunction(
    const std::shared_ptr<Tensor>& x, const std::shared_ptr<Tensor>& r,
    const std::shared_ptr<Tensor>& g, const std::shared_ptr<Tensor>& b,
    const std::shared_ptr<Tensor>& sum, const std::shared_ptr<Tensor>& m,
    const std::shared_ptr<Tensor>& rs, uint32_t m_size, uint32_t n_size)
    : x_input(x), r_input(r), gamma(g), beta(b), mean(m), rstd(rs), sum_output(sum), M(m_size),
      N(n_size) {}

void AddLayerNormFunction::apply_backward() {
  auto S = sum_output.lock();
  std::shared_ptr<Tensor> out = std::move(pending_out);
  pending_out.reset();
  const float* dsum = grad_in(S);
  const float* dy = grad_in(out);
  if (!dy && !dsum) return;
  const size_t n = static_cast<size_t>(M) * N;
  if (!dy) {  // only the sum's own consumers: each addend receives their gradient
    if (x_input->requires_grad()) add_into(*x_input, dsum, n, "add grad");
    if (r_input->requires_grad()) add_into(*r_input, dsum, n, "add grad");
    return;
  }
  bool ux = false, ur = false;
  float* dx = x_input->requires_grad() ? x_input->gradient_for_write(&ux) : nullptr;
  float* dr = r_input->requires_grad() ? r_input->gradient_for_write(&ur) : nullptr;
  float* dg = gamma->requires_grad() ? gamma->get_gradient_ptr() : nullptr;
  float* db = beta->requires_grad() ? beta->get_gradient_ptr() : nullptr;
  const int flags = (dx && !ux ? PA_ADD_LN_ACC_DX : 0) | (dr && !ur ? PA_ADD_LN_ACC_DR : 0);
  Scratch ws(pa_layer_norm_bwd_workspace_size(M, N), stream());
  // out's node holds the sum, so its values are alive whenever out's gradient is
  if (!S) throw std::runtime_error("Add+LayerNorm backward: the sum has expired");
  check_status(pa_add_layer_norm_bwd(dy, dsum, S->get_data_ptr(), mean->get_data_ptr(),
                                     rstd->get_data_ptr(), gamma->get_data_ptr(), dx, dr, dg, db,
                                     M, N, flags, ws.get(), ws.size(), ps(stream())),
               "Add+LayerNorm backward");
}

LayerNormOutFunction::LayerNormOutFunction(const std::shared_ptr<Tensor>& s,
                                           const std::shared_ptr<Tensor>& out)
    : sum(s), output(out) {}

void LayerNormOutFunction::apply_backward() {
  auto Y = output.lock();
  if (!grad_in(Y)) return;
  if (auto* node = dynamic_cast<AddLayerNormFunction*>(sum->grad_fn().get()))
    node->pending_out = Y;
}

}  // namespace core
