// core::Tensor - fp32 device tensor with an optional gradient and a link to the
// graph node that produced it. Same interface as the reference's
// include/core/Tensor.h:22-53; storage is stream-ordered (cudaMallocAsync on
// the context stream) and gradients start at zero. A leaf's gradient is zeroed
// when it is allocated; an op output's is zeroed only when something first
// reads it or adds to it, and a graph node that writes every element of it
// first overwrites it instead, so most activations' gradients are written
// once and never memset.
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <vector>

namespace core {
using float32_t = float;

struct Function;

class Tensor : public std::enable_shared_from_this<Tensor> {
 public:
  explicit Tensor(const std::vector<uint32_t>& shape, bool requires_gradient = false,
                  bool is_leaf = true);
  ~Tensor();
  Tensor(const Tensor&) = delete;
  Tensor& operator=(const Tensor&) = delete;

  void to_device(const std::vector<float32_t>& host_data) const;
  std::vector<float32_t> to_host() const;
  std::vector<float32_t> grad_to_host() const;

  std::vector<uint32_t> get_shape() const { return shape; }
  float32_t* get_data_ptr() const { return data_ptr; }
  size_t numel() const { return size; }

  bool requires_grad() const { return requires_gradient; }
  bool leaf() const { return is_leaf; }
  // The gradient buffer, zeroed first if nothing has written it yet.
  float32_t* get_gradient_ptr() const;
  // For a graph node that writes the whole gradient: the buffer, and in
  // *unwritten whether nothing has written it yet - its contents are then
  // undefined (it stands for zero), and the node must overwrite every element
  // rather than add. Afterwards the gradient counts as written.
  float32_t* gradient_for_write(bool* unwritten) const;
  // True while the gradient stands for zero without having been written.
  bool gradient_unwritten() const { return grad_unwritten; }
  void set_grad_fn(std::shared_ptr<Function> fn);
  std::shared_ptr<Function> grad_fn() const { return grad_function; }
  void zero_grad() const;
  // Moves the gradient into caller-owned device memory of numel() floats
  // (16-byte aligned), zeroed on the context stream; the tensor's own buffer
  // is freed. The caller keeps that memory alive while the tensor uses it.
  // Lets a data-parallel reducer keep many gradients in one flat buffer and
  // all-reduce it in place.
  void set_gradient_storage(float32_t* external);

  // Seeds this tensor's gradient with ones (or keeps the gradient already
  // written there) and runs every graph node reachable from it once, in
  // reverse topological order, so shared inputs receive the sum of all
  // contributions before their own node runs.
  void backward(bool seed_with_ones = true) const;
  // As backward(), and `leaf_ready` is called for each gradient-requiring leaf
  // of the graph (a parameter or input) right after the last node that adds to
  // its gradient has been enqueued: its gradient is then final on the stream,
  // so a caller can start reducing it while the rest of the backward runs.
  using LeafHook = std::function<void(const std::shared_ptr<Tensor>&)>;
  void backward(bool seed_with_ones, const LeafHook& leaf_ready) const;

  // bf16 operand planes of this tensor's data, written by the op that produced
  // it (a projection's epilogue) under f32 math mode operand_planes_mode, in
  // the layout a projection reading the tensor keeps for its backward; that
  // projection takes them instead of converting the tensor. to_device drops
  // them; other writes into the data must reset them too.
  mutable std::shared_ptr<void> operand_planes;
  mutable size_t operand_planes_bytes = 0;
  mutable int operand_planes_mode = -1;

 private:
  float32_t* data_ptr = nullptr;
  float32_t* gradient_ptr = nullptr;
  std::vector<uint32_t> shape;
  size_t size = 0;
  bool requires_gradient = false;
  bool is_leaf = true;
  bool owns_gradient = true;
  mutable bool grad_unwritten = false;
  std::shared_ptr<Function> grad_function;
};

// Throws std::runtime_error("<what>: <status string>") for a non-zero pa_status.
void check_status(int status, const char* what);
}  // namespace core
