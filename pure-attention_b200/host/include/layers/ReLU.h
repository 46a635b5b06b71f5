#pragma once
#include "layers/Module.h"

namespace layers {
class ReLU : public Module {
 public:
  ReLU() = default;
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& In) override;
};
}  // namespace layers
