// Small training kernels behind the operator surface (fp32, HBM-bound):
//   ReLU forward / backward      ReLU_kernel.cu:4-12, ReLU_backward_kernel.cu:4-10
//   MSE forward / backward       mse_forward_kernel.cu:4-13 (+ mse_div_kernel.cu), mse_backward_kernel.cu:4-19
//   Adam step                    adam_step_kernel.cu:4-31 (bias corrections computed by the host)
//   normal / constant fill       populate_normal_kernel.cu:4-15 (here seeded, not clock-seeded)
// Differences from the reference: the MSE sum is one deterministic block
// reduction (the reference issues one global atomicAdd per element), and the
// gradient kernels accumulate into their outputs (grads start at zero and a
// tensor may feed several ops).
#include <cuda_runtime.h>
#include <cstdint>
#include "host_launchers.h"

namespace pa {

namespace {

int sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}
unsigned grid(size_t n) {
  const size_t want = (n + 255) / 256, cap = static_cast<size_t>(sms()) * 8;
  return static_cast<unsigned>(want < cap ? (want ? want : 1) : cap);
}
#define GRID_STRIDE(i, n)                                                          \
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < (n); \
       i += static_cast<size_t>(gridDim.x) * blockDim.x)

__global__ void relu_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  GRID_STRIDE(i, n) y[i] = fmaxf(x[i], 0.f);
}
__global__ void relu_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                float* __restrict__ dx, size_t n) {
  GRID_STRIDE(i, n) if (x[i] > 0.f) dx[i] += dy[i];
}

// loss = sum((p - t)^2) / n in one CTA (fixed order: deterministic).
__global__ void __launch_bounds__(1024)
    mse_fwd_kernel(const float* __restrict__ p, const float* __restrict__ t, float* __restrict__ loss,
                   size_t n) {
  __shared__ float part[32];
  float acc = 0.f;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = p[i] - t[i];
    acc = fmaf(d, d, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) loss[0] = v / static_cast<float>(n);
  }
}
// dp += 2/n * (p - t) * dloss[0]
__global__ void mse_bwd_kernel(const float* __restrict__ p, const float* __restrict__ t,
                               const float* __restrict__ dloss, float* __restrict__ dp, size_t n) {
  const float s = 2.f * dloss[0] / static_cast<float>(n);
  GRID_STRIDE(i, n) dp[i] += s * (p[i] - t[i]);
}

__global__ void adam_kernel(float* __restrict__ w, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, size_t n, float lr, float b1, float b2, float eps,
                            float c1, float c2) {
  GRID_STRIDE(i, n) {
    const float gi = g[i];
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    w[i] -= lr * ((mi / c1) / (sqrtf(vi / c2) + eps));
  }
}

// Counter-based normal samples: splitmix64 of (seed, index) -> two uniforms ->
// Box-Muller. Reproducible for a given seed regardless of launch shape.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
__global__ void fill_normal_kernel(float* __restrict__ x, size_t n, float std_dev, uint64_t seed) {
  GRID_STRIDE(i, n) {
    const uint64_t r = mix64(seed * 0x100000001b3ull + i);
    const float u1 = (static_cast<float>(r >> 40) + 1.f) * (1.f / 16777217.f);  // (0, 1]
    const float u2 = static_cast<float>((r >> 16) & 0xffffffu) * (1.f / 16777216.f);
    x[i] = std_dev * sqrtf(-2.f * __logf(u1)) * __cosf(6.28318530718f * u2);
  }
}
__global__ void fill_kernel(float* __restrict__ x, size_t n, float value) {
  GRID_STRIDE(i, n) x[i] = value;
}

int ok() { return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH; }

}  // namespace

int launch_relu_fwd(const float* x, float* y, size_t n, cudaStream_t s) {
  relu_fwd_kernel<<<grid(n), 256, 0, s>>>(x, y, n);
  return ok();
}
int launch_relu_bwd(const float* dy, const float* x, float* dx, size_t n, cudaStream_t s) {
  relu_bwd_kernel<<<grid(n), 256, 0, s>>>(dy, x, dx, n);
  return ok();
}
int launch_mse_fwd(const float* p, const float* t, float* loss, size_t n, cudaStream_t s) {
  mse_fwd_kernel<<<1, 1024, 0, s>>>(p, t, loss, n);
  return ok();
}
int launch_mse_bwd(const float* p, const float* t, const float* dl, float* dp, size_t n,
                   cudaStream_t s) {
  mse_bwd_kernel<<<grid(n), 256, 0, s>>>(p, t, dl, dp, n);
  return ok();
}
int launch_adam(float* w, const float* g, float* m, float* v, size_t n, float lr, float b1, float b2,
                float eps, float c1, float c2, cudaStream_t s) {
  adam_kernel<<<grid(n), 256, 0, s>>>(w, g, m, v, n, lr, b1, b2, eps, c1, c2);
  return ok();
}
int launch_fill_normal(float* x, size_t n, float std_dev, uint64_t seed, cudaStream_t s) {
  fill_normal_kernel<<<grid(n), 256, 0, s>>>(x, n, std_dev, seed);
  return ok();
}
int launch_fill(float* x, size_t n, float value, cudaStream_t s) {
  fill_kernel<<<grid(n), 256, 0, s>>>(x, n, value);
  return ok();
}

}  // namespace pa
