#include "core/Tensor.h"

#include <algorithm>
#include <unordered_map>
#include <stdexcept>
#include <string>
#include <unordered_set>
#include <vector>

#include "core/Autograd.h"
#include "device_util.h"

namespace core {

void check_status(int status, const char* what) {
  if (status != PA_OK) throw std::runtime_error(std::string(what) + ": " + pa_status_string(status));
}

static float32_t* device_alloc(size_t n, cudaStream_t s) {
  void* p = nullptr;
  retain_pool_memory();
  const cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(n, 1) * sizeof(float32_t), s);
  if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA Error: ") + cudaGetErrorString(e));
  return static_cast<float32_t*>(p);
}

Tensor::Tensor(const std::vector<uint32_t>& shape_, bool requires_gradient_, bool is_leaf_)
    : shape(shape_), requires_gradient(requires_gradient_), is_leaf(is_leaf_) {
  size = 1;
  for (uint32_t s : shape) size *= s;
  const cudaStream_t s = CudaContext::getStream();
  data_ptr = device_alloc(size, s);
  if (requires_gradient) {
    gradient_ptr = device_alloc(size, s);
    if (is_leaf)
      cudaMemsetAsync(gradient_ptr, 0, size * sizeof(float32_t), s);  // gradients start at zero
    else
      grad_unwritten = true;  // zeroed (or overwritten) on first use
  }
}

float32_t* Tensor::get_gradient_ptr() const {
  if (grad_unwritten) {
    grad_unwritten = false;
    if (cudaMemsetAsync(gradient_ptr, 0, size * sizeof(float32_t), CudaContext::getStream()) !=
        cudaSuccess)
      throw std::runtime_error("gradient: cudaMemsetAsync failed");
  }
  return gradient_ptr;
}

float32_t* Tensor::gradient_for_write(bool* unwritten) const {
  *unwritten = grad_unwritten;
  grad_unwritten = false;
  return gradient_ptr;
}

Tensor::~Tensor() {
  const cudaStream_t s = CudaContext::getStream();
  if (data_ptr) cudaFreeAsync(data_ptr, s);
  if (gradient_ptr && owns_gradient) cudaFreeAsync(gradient_ptr, s);
}

void Tensor::to_device(const std::vector<float32_t>& host_data) const {
  if (host_data.size() != size)
    throw std::length_error("Size mismatch: CPU array has different size to GPU tensor.");
  operand_planes.reset();  // they described the old values
  const cudaStream_t s = CudaContext::getStream();
  if (cudaMemcpyAsync(data_ptr, host_data.data(), size * sizeof(float32_t), cudaMemcpyHostToDevice,
                      s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    throw std::runtime_error("To GPU error (Memcpy H2D)");
}

std::vector<float32_t> Tensor::to_host() const {
  std::vector<float32_t> out(size);
  const cudaStream_t s = CudaContext::getStream();
  if (cudaMemcpyAsync(out.data(), data_ptr, size * sizeof(float32_t), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    throw std::runtime_error("To CPU error (Memcpy D2H)");
  return out;
}

std::vector<float32_t> Tensor::grad_to_host() const {
  std::vector<float32_t> out(size, 0.f);
  if (!gradient_ptr || grad_unwritten) return out;
  const cudaStream_t s = CudaContext::getStream();
  if (cudaMemcpyAsync(out.data(), gradient_ptr, size * sizeof(float32_t), cudaMemcpyDeviceToHost,
                      s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    throw std::runtime_error("To CPU error (Memcpy D2H)");
  return out;
}

void Tensor::set_grad_fn(std::shared_ptr<Function> fn) {
  grad_function = std::move(fn);
  is_leaf = false;
}

void Tensor::set_gradient_storage(float32_t* external) {
  if (!requires_gradient) throw std::runtime_error("set_gradient_storage: tensor has no gradient");
  if (!external || (reinterpret_cast<uintptr_t>(external) & 15u) != 0)
    throw std::runtime_error("set_gradient_storage: pointer must be non-null and 16-byte aligned");
  const cudaStream_t s = CudaContext::getStream();
  if (gradient_ptr && owns_gradient) cudaFreeAsync(gradient_ptr, s);
  gradient_ptr = external;
  owns_gradient = false;
  grad_unwritten = false;
  if (cudaMemsetAsync(gradient_ptr, 0, size * sizeof(float32_t), s) != cudaSuccess)
    throw std::runtime_error("set_gradient_storage: cudaMemsetAsync failed");
}

void Tensor::zero_grad() const {
  if (gradient_ptr && !grad_unwritten)
    cudaMemsetAsync(gradient_ptr, 0, size * sizeof(float32_t), CudaContext::getStream());
}

void Tensor::backward(bool seed_with_ones) const { backward(seed_with_ones, LeafHook()); }

void Tensor::backward(bool seed_with_ones, const LeafHook& leaf_ready) const {
  if (!requires_gradient)
    throw std::runtime_error("Called backward() on a tensor that does not require gradients.");
  if (seed_with_ones) {
    grad_unwritten = false;
    check_status(pa_fill(gradient_ptr, size, 1.0f, ps(CudaContext::getStream())), "backward seed");
  }
  if (!grad_function) return;
  // Post-order DFS over the graph: a node is appended after every node that
  // produces one of its inputs, so the reversed list runs each node only once
  // all the nodes consuming its output have added their contributions.
  std::vector<Function*> order;
  std::unordered_set<Function*> seen;
  std::vector<std::pair<Function*, size_t>> stack;
  stack.emplace_back(grad_function.get(), 0);
  seen.insert(grad_function.get());
  while (!stack.empty()) {
    auto& [node, next] = stack.back();
    const auto ins = node->inputs();
    if (next < ins.size()) {
      const auto& in = ins[next++];
      Function* f = in ? in->grad_fn().get() : nullptr;
      if (f && in->requires_grad() && seen.insert(f).second) stack.emplace_back(f, 0);
    } else {
      order.push_back(node);
      stack.pop_back();
    }
  }
  if (!leaf_ready) {
    for (auto it = order.rbegin(); it != order.rend(); ++it) (*it)->apply_backward();
    return;
  }
  // For each gradient-requiring leaf, the last node (in execution order) that
  // takes it as an input; after that node the leaf's gradient is complete.
  std::vector<Function*> exec(order.rbegin(), order.rend());
  std::unordered_map<const Tensor*, size_t> last;
  std::vector<std::vector<std::shared_ptr<Tensor>>> ready_after(exec.size());
  for (size_t i = 0; i < exec.size(); ++i)
    for (const auto& in : exec[i]->inputs())
      if (in && in->requires_grad() && !in->grad_fn()) last[in.get()] = i;
  std::unordered_set<const Tensor*> queued;
  for (size_t i = 0; i < exec.size(); ++i)
    for (const auto& in : exec[i]->inputs())
      if (in && in->requires_grad() && !in->grad_fn() && last[in.get()] == i &&
          queued.insert(in.get()).second)
        ready_after[i].push_back(in);
  for (size_t i = 0; i < exec.size(); ++i) {
    exec[i]->apply_backward();
    for (const auto& leaf : ready_after[i]) leaf_ready(leaf);
  }
}

}  // namespace core
