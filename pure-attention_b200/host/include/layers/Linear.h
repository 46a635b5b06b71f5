// layers::Linear: y = x W + b with W [in, out], b [1, out] (include/layers/Linear.h).
#pragma once
#include "layers/Module.h"

namespace layers {
class Linear : public Module {
 public:
  std::shared_ptr<core::Tensor> weight;
  std::shared_ptr<core::Tensor> bias;
  Linear(uint32_t in_channels, uint32_t out_channels);
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& input) override;
  std::vector<std::shared_ptr<core::Tensor>> parameters() override;
};
}  // namespace layers
