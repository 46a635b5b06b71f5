#pragma once
#include <memory>
#include "core/Tensor.h"

namespace loss {
class Loss {
 public:
  virtual ~Loss() = default;
  virtual std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& predictions,
                                                const std::shared_ptr<core::Tensor>& targets) = 0;
};
}  // namespace loss
