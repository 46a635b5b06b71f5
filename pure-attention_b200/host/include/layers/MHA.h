// layers::MultiheadAttention (include/layers/MHA.h:7-23): in_proj_weight
// [E, 3E], in_proj_bias [1, 3E], out_proj_weight [E, E], out_proj_bias [1, E].
#pragma once
#include "layers/Module.h"

namespace layers {
class MultiheadAttention : public Module {
 public:
  MultiheadAttention(uint32_t embed_dim, uint32_t num_heads);
  // self-attention: one [E, 3E] projection, split along the last dimension
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& input) override;
  // q, k, v projected by the three column blocks of in_proj_weight
  std::shared_ptr<core::Tensor> forward(const std::shared_ptr<core::Tensor>& query,
                                        const std::shared_ptr<core::Tensor>& key,
                                        const std::shared_ptr<core::Tensor>& value);
  std::vector<std::shared_ptr<core::Tensor>> parameters() override;

 private:
  std::shared_ptr<core::Tensor> in_proj_weight, in_proj_bias, out_proj_weight, out_proj_bias;
  const uint32_t embed_dim;
  const uint32_t num_heads;
};
}  // namespace layers
