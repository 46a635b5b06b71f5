// Graph nodes. Each node keeps the reference's public members
// (include/core/Autograd.h:6-105) and computes the gradients of its inputs
// from its output's gradient, accumulating into them. Unlike the reference,
// apply_backward does not recurse into its inputs: Tensor::backward visits
// the nodes in reverse topological order using inputs().
#pragma once
#include <memory>
#include <vector>
#include "core/Tensor.h"

namespace core {

struct Function {
  virtual void apply_backward() = 0;
  virtual std::vector<std::shared_ptr<Tensor>> inputs() const = 0;
  virtual ~Function() = default;
};

struct MatMulFunction : public Function {
  std::shared_ptr<Tensor> X_input;
  std::shared_ptr<Tensor> W_input;
  std::weak_ptr<Tensor> Y_output;
  MatMulFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> w, std::shared_ptr<Tensor> y);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {X_input, W_input}; }
};

// Bias add (bias of shape [1, N] broadcast over rows) or same-shape add.
struct AddFunction : public Function {
  std::shared_ptr<Tensor> X_input;
  std::shared_ptr<Tensor> bias_input;
  std::weak_ptr<Tensor> Y_output;
  AddFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> bias, std::shared_ptr<Tensor> y);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {X_input, bias_input}; }
};

struct ReLUFunction : public Function {
  std::shared_ptr<Tensor> Input;
  std::weak_ptr<Tensor> Output;
  ReLUFunction(std::shared_ptr<Tensor> in, std::shared_ptr<Tensor> out);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {Input}; }
};

struct MSEFunction : public Function {
  std::shared_ptr<Tensor> predictions;
  std::shared_ptr<Tensor> targets;
  std::weak_ptr<Tensor> output_loss;
  MSEFunction(const std::shared_ptr<Tensor>& preds, const std::shared_ptr<Tensor>& targs,
              const std::shared_ptr<Tensor>& out);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {predictions}; }
};

// Fused projection X W + bias, output as column blocks (core::linear): one
// node for what MatMulFunction + AddFunction + SplitFunction do in three.
// With relu (one output), Y = max(0, X W + bias): one node for Linear + ReLU.
struct LinearFunction : public Function {
  std::shared_ptr<Tensor> X_input;
  std::shared_ptr<Tensor> W_input;
  std::shared_ptr<Tensor> bias_input;
  std::vector<std::weak_ptr<Tensor>> Outputs;
  bool relu;
  // X's operand planes written by the forward (pa_linear_fwd_keep) for the
  // backward, with the f32 math mode they were made under
  std::shared_ptr<void> kept;
  size_t kept_bytes = 0;
  int kept_mode = 0;
  LinearFunction(std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> w, std::shared_ptr<Tensor> b,
                 std::vector<std::shared_ptr<Tensor>> outs, bool relu_ = false);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override {
    return {X_input, W_input, bias_input};
  }
};

struct SplitFunction : public Function {
  std::shared_ptr<Tensor> Input;
  std::vector<std::weak_ptr<Tensor>> Outputs;
  SplitFunction(std::shared_ptr<Tensor> in, std::vector<std::shared_ptr<Tensor>> outs);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {Input}; }
};

struct FlashAttentionFunction : public Function {
  std::shared_ptr<Tensor> Q_input;
  std::shared_ptr<Tensor> K_input;
  std::shared_ptr<Tensor> V_input;
  std::weak_ptr<Tensor> O_output;
  std::shared_ptr<Tensor> L_cache;
  int num_heads;
  // the forward's workspace, holding the bf16 planes of Q, K, V it converted,
  // with the f32 math mode they were made under (the backward converts only dO)
  std::shared_ptr<void> kept;
  size_t kept_bytes = 0;
  int kept_mode = 0;
  FlashAttentionFunction(const std::shared_ptr<Tensor>& q, const std::shared_ptr<Tensor>& k,
                         const std::shared_ptr<Tensor>& v, const std::shared_ptr<Tensor>& o,
                         const std::shared_ptr<Tensor>& lcache, int heads);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override {
    return {Q_input, K_input, V_input};
  }
};

struct LayerNormFunction : public Function {
  std::shared_ptr<Tensor> input;
  std::shared_ptr<Tensor> gamma;
  std::shared_ptr<Tensor> beta;
  std::weak_ptr<Tensor> output;
  std::shared_ptr<Tensor> mean;
  std::shared_ptr<Tensor> rstd;
  uint32_t M;
  uint32_t N;
  LayerNormFunction(const std::shared_ptr<Tensor>& inp, const std::shared_ptr<Tensor>& g,
                    const std::shared_ptr<Tensor>& b, const std::shared_ptr<Tensor>& out,
                    const std::shared_ptr<Tensor>& m, const std::shared_ptr<Tensor>& r,
                    uint32_t m_size, uint32_t n_size);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {input, gamma, beta}; }
};

// Backward of core::add_layer_norm: sum = x + r, out = LayerNorm(sum). This
// node is sum's grad_fn, so it runs after every consumer of sum; out's grad_fn
// is a LayerNormOutFunction, which runs after every consumer of out and hands
// out's gradient to this node. The node then writes G = LN_bwd(dout) + dsum
// (dsum: the gradient sum received from its other consumers) straight into
// x's and r's gradients (pa_add_layer_norm_bwd): the sum's own gradient is
// never formed, and no separate add pass runs.
struct AddLayerNormFunction : public Function {
  std::shared_ptr<Tensor> x_input;
  std::shared_ptr<Tensor> r_input;
  std::shared_ptr<Tensor> gamma;
  std::shared_ptr<Tensor> beta;
  std::shared_ptr<Tensor> mean;
  std::shared_ptr<Tensor> rstd;
  std::weak_ptr<Tensor> sum_output;
  uint32_t M;
  uint32_t N;
  // out, set by out's node in the current backward when a gradient reached it
  std::shared_ptr<Tensor> pending_out;
  AddLayerNormFunction(const std::shared_ptr<Tensor>& x, const std::shared_ptr<Tensor>& r,
                       const std::shared_ptr<Tensor>& g, const std::shared_ptr<Tensor>& b,
                       const std::shared_ptr<Tensor>& sum, const std::shared_ptr<Tensor>& m,
                       const std::shared_ptr<Tensor>& rs, uint32_t m_size, uint32_t n_size);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override {
    return {x_input, r_input, gamma, beta};
  }
};

// out's node in core::add_layer_norm: holds the sum (whose values the
// backward reads) and passes out's gradient to the sum's AddLayerNormFunction,
// which runs after it.
struct LayerNormOutFunction : public Function {
  std::shared_ptr<Tensor> sum;
  std::weak_ptr<Tensor> output;
  LayerNormOutFunction(const std::shared_ptr<Tensor>& s, const std::shared_ptr<Tensor>& out);
  void apply_backward() override;
  std::vector<std::shared_ptr<Tensor>> inputs() const override { return {sum}; }
};

}  // namespace core
