// Internal helpers of the host layer: status checks and stream-ordered scratch.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include "core/Context.h"
#include "core/Tensor.h"
#include "pa_kernels.h"

namespace core {

// The device's default memory pool hands freed memory back to the driver at
// every synchronisation unless its release threshold is raised, and the next
// cudaMallocAsync then maps it again. A training step frees and re-allocates
// its activations every step, so the pool keeps what it has (this process's
// pool only; nothing outlives the process).
inline void retain_pool_memory() {
  static thread_local int set_for = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev == set_for) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  set_for = dev;
}

// Stream-ordered device scratch (cudaMallocAsync / cudaFreeAsync on `s`).
class Scratch {
 public:
  Scratch(size_t bytes, cudaStream_t s) : s_(s), n_(bytes) {
    if (bytes) {
      retain_pool_memory();
      const cudaError_t e = cudaMallocAsync(&p_, bytes, s);
      if (e != cudaSuccess)
        throw std::runtime_error(std::string("CUDA Error: ") + cudaGetErrorString(e));
    }
  }
  ~Scratch() {
    if (p_) cudaFreeAsync(p_, s_);
  }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  void* get() const { return p_; }
  size_t size() const { return n_; }

 private:
  void* p_ = nullptr;
  cudaStream_t s_;
  size_t n_;
};

inline pa_stream_t ps(cudaStream_t s) { return static_cast<pa_stream_t>(s); }

// Stream-ordered device memory owned by a shared_ptr (freed on the context
// stream when the last owner lets go).
inline std::shared_ptr<void> device_buffer(size_t bytes, cudaStream_t s, const char* what) {
  void* p = nullptr;
  retain_pool_memory();
  if (cudaMallocAsync(&p, bytes, s) != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": cannot allocate device memory");
  return std::shared_ptr<void>(p, [](void* q) { cudaFreeAsync(q, CudaContext::getStream()); });
}

inline size_t last_dim(const Tensor& t) {
  const auto sh = t.get_shape();
  return sh.empty() ? 1 : sh.back();
}

}  // namespace core
