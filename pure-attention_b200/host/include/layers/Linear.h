// layers::Linear: y = x W + b with W [in, out], b [1, out] (include/layers/Linear.h).
// relu (not in the reference): y = max(0, x W + b) in one fused node, for the
// Linear -> ReLU pair of a feed-forward block.
#pragma once
#include "layers/Module.h"

namespace layers {
class Linear : public Module {
 public:
  std::shared_ptr<core::Tensor> weight;
  std::shared_ptr<core::Tensor> bias;
  bool relu = false;
  Linear(uint32_t in_channels, uint32_t out_channels, bool relu_ = false);
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& input) override;
  std::vector<std::shared_ptr<core::Tensor>> parameters() override;
};
}  // namespace layers
