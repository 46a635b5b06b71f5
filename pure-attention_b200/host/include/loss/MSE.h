// loss::MSE: mean((pred - target)^2) (include/loss/MSE.h, source/loss/MSE.cpp:8-11).
#pragma once
#include "loss/Loss.h"

namespace loss {
class MSE : public Loss {
 public:
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& predictions,
                                        const std::shared_ptr<core::Tensor>& targets) override;
};
}  // namespace loss
