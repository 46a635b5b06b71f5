#include "core/Adam.h"

#include <cmath>

#include "core/Functional.h"
#include "device_util.h"

namespace optim {

Adam::Adam(std::vector<std::shared_ptr<core::Tensor>> params, float lr_, float beta1_, float beta2_,
           float eps)
    : parameters(std::move(params)), lr(lr_), beta1(beta1_), beta2(beta2_), epsilon(eps) {
  const cudaStream_t s = CudaContext::getStream();
  for (auto& p : parameters) {
    m_states.push_back(std::make_shared<core::Tensor>(p->get_shape(), false));
    v_states.push_back(std::make_shared<core::Tensor>(p->get_shape(), false));
    core::pop_data_zeros(m_states.back(), s);
    core::pop_data_zeros(v_states.back(), s);
  }
}

// Same update as adam_step_kernel.cu:18-30 with bias corrections from Adam.cpp:28-33.
void Adam::step() {
  ++step_count;
  const float c1 = 1.0f - std::pow(beta1, static_cast<float>(step_count));
  const float c2 = 1.0f - std::pow(beta2, static_cast<float>(step_count));
  // every parameter in one multi-tensor launch (per 48 tensors)
  std::vector<float*> w, m, v;
  std::vector<const float*> g;
  std::vector<size_t> n;
  for (size_t i = 0; i < parameters.size(); ++i) {
    auto& p = parameters[i];
    if (!p->requires_grad() || !p->get_gradient_ptr()) continue;
    w.push_back(p->get_data_ptr());
    g.push_back(p->get_gradient_ptr());
    m.push_back(m_states[i]->get_data_ptr());
    v.push_back(v_states[i]->get_data_ptr());
    n.push_back(p->numel());
  }
  core::check_status(pa_adam_step_multi(w.data(), g.data(), m.data(), v.data(), n.data(),
                                        static_cast<int>(w.size()), lr, beta1, beta2, epsilon, c1,
                                        c2, core::ps(CudaContext::getStream())),
                     "Adam");
}

void Adam::zero_grad() {
  for (auto& p : parameters) p->zero_grad();
}

}  // namespace optim
