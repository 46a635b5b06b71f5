// optim::Adam - the reference's optimizer interface (include/core/Adam.h:9-33).
#pragma once
#include <memory>
#include <vector>
#include "core/Tensor.h"

namespace optim {
class Adam {
 public:
  Adam(std::vector<std::shared_ptr<core::Tensor>> params, float lr = 1e-3f, float beta1 = 0.9f,
       float beta2 = 0.999f, float eps = 1e-8f);
  void step();
  void zero_grad();
  // Optimizer state for checkpoints (not in the reference's interface).
  int steps() const { return step_count; }
  void set_steps(int n) { step_count = n; }
  const std::vector<std::shared_ptr<core::Tensor>>& first_moments() const { return m_states; }
  const std::vector<std::shared_ptr<core::Tensor>>& second_moments() const { return v_states; }

 private:
  std::vector<std::shared_ptr<core::Tensor>> parameters;
  std::vector<std::shared_ptr<core::Tensor>> m_states, v_states;
  float lr, beta1, beta2, epsilon;
  int step_count = 0;
};
}  // namespace optim
