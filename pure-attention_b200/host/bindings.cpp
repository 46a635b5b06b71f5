// PureAttention Python module: the reference's surface (bindings.cpp:37-125)
// over the B200 host layer. Names, signatures and defaults match; additions
// include set_seed, device_status, set_stream, flash_attention and
// Tensor.zero_grad.
#include <pybind11/pybind11.h>
#include <string>
#include <pybind11/functional.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cmath>
#include <numeric>

#include "core/Adam.h"
#include "core/Context.h"
#include "core/Functional.h"
#include "core/Tensor.h"
#include "layers/LayerNorm.h"
#include "layers/Linear.h"
#include "layers/MHA.h"
#include "layers/Module.h"
#include "layers/ReLU.h"
#include "loss/MSE.h"
#include "pa_kernels.h"

namespace py = pybind11;
using core::Tensor;

class PyModule : public layers::Module {
 public:
  using layers::Module::Module;
  std::shared_ptr<Tensor> forward(const std::shared_ptr<Tensor>& input) override {
    PYBIND11_OVERRIDE_PURE(std::shared_ptr<Tensor>, layers::Module, forward, input);
  }
  std::vector<std::shared_ptr<Tensor>> parameters() override {
    PYBIND11_OVERRIDE(std::vector<std::shared_ptr<Tensor>>, layers::Module, parameters, );
  }
};

PYBIND11_MODULE(PureAttention, m) {
  m.doc() = "Pure-Attention operator surface over sm_100a kernels";

  // Zero-copy views for other CUDA libraries (torch.as_tensor, cupy): the
  // gradient of a tensor, kept alive by the view. Not in the reference's surface.
  struct GradView {
    std::shared_ptr<Tensor> owner;
  };
  auto cai = [](float* ptr, const std::vector<uint32_t>& shape) {
    py::dict d;
    py::tuple sh(shape.size());
    for (size_t i = 0; i < shape.size(); ++i) sh[i] = shape[i];
    d["shape"] = sh;
    d["typestr"] = "<f4";
    d["data"] = py::make_tuple(reinterpret_cast<uintptr_t>(ptr), false);
    d["version"] = 3;
    d["strides"] = py::none();
    return d;
  };
  py::class_<GradView>(m, "GradView")
      .def_property_readonly("__cuda_array_interface__", [cai](const GradView& g) {
        if (!g.owner->get_gradient_ptr()) throw std::runtime_error("tensor has no gradient");
        return cai(g.owner->get_gradient_ptr(), g.owner->get_shape());
      });

  py::class_<Tensor, std::shared_ptr<Tensor>>(m, "Tensor")
      .def(py::init([](std::vector<uint32_t> shape, bool requires_grad) {
             return std::make_shared<Tensor>(shape, requires_grad);
           }),
           py::arg("shape"), py::arg("requires_grad") = false)
      .def("backward", py::overload_cast<bool>(&Tensor::backward, py::const_),
           py::arg("seed_with_ones") = true)
      .def("backward", py::overload_cast<bool, const Tensor::LeafHook&>(&Tensor::backward, py::const_),
           py::arg("seed_with_ones"), py::arg("leaf_ready"),
           "backward(), calling leaf_ready(t) for each gradient-requiring leaf t as soon as its "
           "gradient is final on the stream")
      .def("to_host", &Tensor::to_host)
      .def("to_device", &Tensor::to_device)
      .def("grad_to_host", &Tensor::grad_to_host)
      .def("shape", &Tensor::get_shape)
      .def("zero_grad", &Tensor::zero_grad)
      .def("set_grad_storage",
           [](Tensor& t, uintptr_t ptr) { t.set_gradient_storage(reinterpret_cast<float*>(ptr)); },
           py::arg("device_ptr"),
           "Move the gradient into caller-owned device memory (numel() floats, 16-byte aligned, "
           "zeroed); the caller keeps it alive")
      .def_property_readonly("__cuda_array_interface__",
                             [cai](const Tensor& t) { return cai(t.get_data_ptr(), t.get_shape()); })
      .def("grad_view", [](const std::shared_ptr<Tensor>& t) { return GradView{t}; },
           "Zero-copy view of the gradient (has __cuda_array_interface__)")
      .def("get_grad_stats", [](const Tensor& t) {
        const std::vector<float> g = t.grad_to_host();
        py::dict d;
        if (g.empty()) return d;
        double s = 0.0, s2 = 0.0;
        for (float v : g) {
          s += v;
          s2 += static_cast<double>(v) * v;
        }
        const double mean = s / g.size();
        d["mean"] = mean;
        d["std"] = std::sqrt(std::max(0.0, s2 / g.size() - mean * mean));
        d["min"] = *std::min_element(g.begin(), g.end());
        d["max"] = *std::max_element(g.begin(), g.end());
        return d;
      }, "Gradient stats");

  py::class_<layers::Module, PyModule, std::shared_ptr<layers::Module>>(m, "Module")
      .def(py::init<>())
      .def("forward", &layers::Module::forward)
      .def("parameters", &layers::Module::parameters);

  py::class_<layers::Linear, layers::Module, std::shared_ptr<layers::Linear>>(m, "Linear")
      .def(py::init<uint32_t, uint32_t, bool>(), py::arg("in_channels"), py::arg("out_channels"),
           py::arg("relu") = false,
           "relu=True (not in the reference): y = max(0, x W + b) as one fused op")
      .def("forward", &layers::Linear::forward)
      .def("parameters", &layers::Linear::parameters)
      .def_readwrite("weight", &layers::Linear::weight)
      .def_readwrite("bias", &layers::Linear::bias);

  py::class_<layers::ReLU, layers::Module, std::shared_ptr<layers::ReLU>>(m, "ReLU")
      .def(py::init<>())
      .def("forward", &layers::ReLU::forward)
      .def("parameters", &layers::ReLU::parameters);

  py::class_<layers::MultiheadAttention, layers::Module, std::shared_ptr<layers::MultiheadAttention>>(
      m, "MultiheadAttention")
      .def(py::init<uint32_t, uint32_t>())
      .def("forward", py::overload_cast<const std::shared_ptr<Tensor>&>(
                          &layers::MultiheadAttention::forward))
      .def("forward",
           py::overload_cast<const std::shared_ptr<Tensor>&, const std::shared_ptr<Tensor>&,
                             const std::shared_ptr<Tensor>&>(&layers::MultiheadAttention::forward))
      .def("parameters", &layers::MultiheadAttention::parameters);

  py::class_<layers::LayerNorm, layers::Module, std::shared_ptr<layers::LayerNorm>>(m, "LayerNorm")
      .def(py::init<uint32_t, float>(), py::arg("normalized_shape"), py::arg("epsilon") = 1e-5f)
      .def("forward", &layers::LayerNorm::forward)
      .def("forward_add", &layers::LayerNorm::forward_add,
           "(x + r, LayerNorm(x + r)) from one fused kernel")
      .def("parameters", &layers::LayerNorm::parameters)
      .def_property_readonly("gamma", &layers::LayerNorm::get_gamma)
      .def_property_readonly("beta", &layers::LayerNorm::get_beta);

  py::class_<loss::MSE, std::shared_ptr<loss::MSE>>(m, "MSE")
      .def(py::init<>())
      .def("forward", &loss::MSE::forward)
      .def("__call__", &loss::MSE::forward);

  py::class_<optim::Adam, std::shared_ptr<optim::Adam>>(m, "Adam")
      .def(py::init<std::vector<std::shared_ptr<Tensor>>, float, float, float, float>(),
           py::arg("params"), py::arg("lr") = 0.001f, py::arg("beta1") = 0.9f,
           py::arg("beta2") = 0.999f, py::arg("eps") = 1e-8f)
      .def("step", &optim::Adam::step)
      .def("zero_grad", &optim::Adam::zero_grad)
      .def_property("step_count", &optim::Adam::steps, &optim::Adam::set_steps,
                    "Steps taken (drives the bias corrections); for checkpoints")
      .def("state", [](const optim::Adam& a) {
        return py::make_tuple(a.first_moments(), a.second_moments());
      }, "(first moments, second moments): one Tensor per parameter, for checkpoints");

  m.def("fill_normal", [](const std::shared_ptr<Tensor>& t, float std_dev) {
    core::pop_data_normal(t, std_dev, CudaContext::getStream());
  }, "Fill tensor with normal distribution", py::arg("tensor"), py::arg("std_dev") = 1.0f);

  m.def("add", [](const std::shared_ptr<Tensor>& a, const std::shared_ptr<Tensor>& b) {
    std::shared_ptr<Tensor> c;
    core::matadd(a, b, c, CudaContext::getStream());
    return c;
  }, "Element-wise addition (a [1, N] second operand is broadcast over rows)", py::arg("a"),
        py::arg("b"));

  m.def("set_float32_math", [](const std::string& mode) {
    int m_ = -1;
    if (mode == "split3") m_ = PA_F32_MATH_SPLIT3;
    if (mode == "bf16") m_ = PA_F32_MATH_BF16;
    if (m_ < 0 || pa_set_f32_math(m_) != PA_OK)
      throw std::invalid_argument("float32 math mode must be 'split3' or 'bf16'");
  }, "Products of the calling thread's matmuls and attention: 'split3' (default; bf16 hi/lo "
     "planes, fp32-level accuracy) or 'bf16' (one bf16 product, fp32 accumulation and storage). "
     "Not in the reference.", py::arg("mode"));
  m.def("get_float32_math", []() {
    return std::string(pa_get_f32_math() == PA_F32_MATH_BF16 ? "bf16" : "split3");
  });
  m.def("set_seed", &CudaContext::setSeed, "Seed of fill_normal and layer initialisation",
        py::arg("seed"));
  m.def("flash_attention", [](const std::shared_ptr<Tensor>& q, const std::shared_ptr<Tensor>& k,
                              const std::shared_ptr<Tensor>& v, int num_heads) {
    std::shared_ptr<Tensor> o;
    core::flash_attention(q, k, v, o, num_heads, CudaContext::getStream());
    return o;
  }, "core::flash_attention: softmax(q k^T / sqrt(d)) v per head of [N, L, E] fp32 tensors, with "
     "its graph node", py::arg("q"), py::arg("k"), py::arg("v"), py::arg("num_heads"));
  m.def("set_stream", [](uintptr_t handle) {
    CudaContext::setStream(reinterpret_cast<cudaStream_t>(handle));
  }, "Stream every operator, allocation and gradient of this module runs on from now on "
     "(a cudaStream_t handle, e.g. torch.cuda.Stream().cuda_stream; 0 = the legacy default "
     "stream). A non-default stream lets a step be captured into a CUDA graph.",
     py::arg("handle"));
  m.def("get_stream", []() { return reinterpret_cast<uintptr_t>(CudaContext::getStream()); });
  m.def("device_status", []() { return pa_device_status(CudaContext::getStream(), 1); },
        "Synchronise and return the kernels' status word (0 = ok)");
}
