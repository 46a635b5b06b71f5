// layers::LayerNorm over the last dimension; gamma = 1, beta = 0 (include/layers/LayerNorm.h).
#pragma once
#include "layers/Module.h"

namespace layers {
class LayerNorm : public Module {
 public:
  explicit LayerNorm(uint32_t normalized_shape, float epsilon = 1e-5f);
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& input) override;
  // {x + r, LayerNorm(x + r)} from one kernel (a residual add fused in front)
  std::pair<std::shared_ptr<core::Tensor>, std::shared_ptr<core::Tensor>> forward_add(
      const std::shared_ptr<core::Tensor>& x, const std::shared_ptr<core::Tensor>& r);
  std::vector<std::shared_ptr<core::Tensor>> parameters() override;
  std::shared_ptr<core::Tensor> get_gamma() const { return gamma; }
  std::shared_ptr<core::Tensor> get_beta() const { return beta; }

 private:
  std::shared_ptr<core::Tensor> gamma;
  std::shared_ptr<core::Tensor> beta;
  uint32_t normalized_shape;
  float epsilon;
};
}  // namespace layers
