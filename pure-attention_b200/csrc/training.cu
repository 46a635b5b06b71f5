// Small training kernels behind the operator surface (fp32, HBM-bound):
//   ReLU forward / backward      ReLU_kernel.cu:4-12, ReLU_backward_kernel.cu:4-10
//   MSE forward / backward       mse_forward_kernel.cu:4-13 (+ mse_div_kernel.cu), mse_backward_kernel.cu:4-19
//   Adam step                    adam_step_kernel.cu:4-31 (bias corrections computed by the host)
//   normal / constant fill       populate_normal_kernel.cu:4-15 (here seeded, not clock-seeded)
// Differences from the reference: the MSE sum is a deterministic two-stage
// reduction (the reference issues one global atomicAdd per element), and the
// gradient kernels accumulate into their outputs (grads start at zero and a
// tensor may feed several ops).
#include <cuda_runtime.h>
#include <cstdint>
#include "host_launchers.h"

namespace pa {

namespace {

int sms() { return device_sm_count(); }
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

// Sum of v over the CTA, valid in thread 0 (blockDim a multiple of 32).
__device__ __forceinline__ float block_sum(float v) {
  __shared__ float part[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  v = 0.f;
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  return v;
}

// MSE without workspace: one CTA (fixed order, deterministic, slow on large n).
__global__ void __launch_bounds__(1024)
    mse_fwd_kernel(const float* __restrict__ p, const float* __restrict__ t, float* __restrict__ loss,
                   size_t n) {
  float acc = 0.f;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = p[i] - t[i];
    acc = fmaf(d, d, acc);
  }
  acc = block_sum(acc);
  if (threadIdx.x == 0) loss[0] = acc / static_cast<float>(n);
}

// MSE, stage 1: CTA b sums (p - t)^2 over its grid-stride share into part[b].
// The grid depends only on n, so the summation order (and the loss) is
// deterministic.
__global__ void __launch_bounds__(256)
    mse_partial_kernel(const float* __restrict__ p, const float* __restrict__ t,
                       float* __restrict__ part, size_t n) {
  float acc = 0.f;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t first = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  size_t n4 = 0;
  if (((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(t)) & 15u) == 0) {
    n4 = n / 4;
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const float4* t4 = reinterpret_cast<const float4*>(t);
#pragma unroll 4
    for (size_t i = first; i < n4; i += stride) {
      const float4 a = p4[i], b = t4[i];
      const float d0 = a.x - b.x, d1 = a.y - b.y, d2 = a.z - b.z, d3 = a.w - b.w;
      acc += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
    }
  }
  for (size_t i = 4 * n4 + first; i < n; i += stride) {
    const float d = p[i] - t[i];
    acc = fmaf(d, d, acc);
  }
  acc = block_sum(acc);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}
// MSE, stage 2: loss = (sum of the partials in index order) / n.
__global__ void __launch_bounds__(1024)
    mse_final_kernel(const float* __restrict__ part, int nparts, float* __restrict__ loss, size_t n) {
  float acc = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) acc += part[i];
  acc = block_sum(acc);
  if (threadIdx.x == 0) loss[0] = acc / static_cast<float>(n);
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

// Multi-tensor Adam: one launch updates up to kAdamPack tensors. The element
// space of the pack is cut into chunks of kAdamChunk; chunk_start[t] is the
// first chunk of tensor t, so a CTA finds its tensor once per chunk.
constexpr int kAdamPack = 48;
constexpr int kAdamChunk = 4096;
struct AdamPack {
  float* w[kAdamPack];
  const float* g[kAdamPack];
  float* m[kAdamPack];
  float* v[kAdamPack];
  size_t n[kAdamPack];
  uint32_t chunk_start[kAdamPack + 1];
  int count;
};
__global__ void __launch_bounds__(256)
    adam_multi_kernel(const __grid_constant__ AdamPack pk, float lr, float b1, float b2, float eps,
                      float c1, float c2) {
  const uint32_t chunks = pk.chunk_start[pk.count];
  for (uint32_t ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
    int t = 0;
    while (t + 1 < pk.count && pk.chunk_start[t + 1] <= ch) ++t;
    const size_t i0 = static_cast<size_t>(ch - pk.chunk_start[t]) * kAdamChunk;
    const size_t i1 = min(pk.n[t], i0 + kAdamChunk);
    float* w = pk.w[t];
    const float* g = pk.g[t];
    float* m = pk.m[t];
    float* v = pk.v[t];
    const bool vec = ((pk.n[t] & 3) == 0) &&
                     (((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g) |
                        reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15u) == 0);
    if (vec) {
      for (size_t i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x) {
        const float4 gi = *reinterpret_cast<const float4*>(g + i);
        float4 mi = *reinterpret_cast<const float4*>(m + i);
        float4 vi = *reinterpret_cast<const float4*>(v + i);
        float4 wi = *reinterpret_cast<const float4*>(w + i);
        const float ga[4] = {gi.x, gi.y, gi.z, gi.w};
        float* ma[4] = {&mi.x, &mi.y, &mi.z, &mi.w};
        float* va[4] = {&vi.x, &vi.y, &vi.z, &vi.w};
        float* wa[4] = {&wi.x, &wi.y, &wi.z, &wi.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          *ma[e] = b1 * *ma[e] + (1.f - b1) * ga[e];
          *va[e] = b2 * *va[e] + (1.f - b2) * ga[e] * ga[e];
          *wa[e] -= lr * ((*ma[e] / c1) / (sqrtf(*va[e] / c2) + eps));
        }
        *reinterpret_cast<float4*>(m + i) = mi;
        *reinterpret_cast<float4*>(v + i) = vi;
        *reinterpret_cast<float4*>(w + i) = wi;
      }
    } else {
      for (size_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float gi = g[i];
        const float mi = b1 * m[i] + (1.f - b1) * gi;
        const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
        m[i] = mi;
        v[i] = vi;
        w[i] -= lr * ((mi / c1) / (sqrtf(vi / c2) + eps));
      }
    }
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
int mse_parts(size_t n) {
  const size_t want = (n + 4 * 256 - 1) / (4 * 256), cap = static_cast<size_t>(sms()) * 4;
  return static_cast<int>(want < cap ? (want ? want : 1) : cap);
}
size_t mse_workspace_bytes(size_t n) { return static_cast<size_t>(mse_parts(n)) * sizeof(float); }

// With a workspace (one float per stage-1 CTA): two launches over the whole GPU.
int launch_mse_fwd(const float* p, const float* t, float* loss, size_t n, float* ws,
                   cudaStream_t s) {
  if (!ws) {
    mse_fwd_kernel<<<1, 1024, 0, s>>>(p, t, loss, n);
    return ok();
  }
  const int parts = mse_parts(n);
  mse_partial_kernel<<<parts, 256, 0, s>>>(p, t, ws, n);
  mse_final_kernel<<<1, 1024, 0, s>>>(ws, parts, loss, n);
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
int launch_adam_multi(float* const* w, const float* const* g, float* const* m, float* const* v,
                      const size_t* n, int count, float lr, float b1, float b2, float eps, float c1,
                      float c2, cudaStream_t s) {
  for (int base = 0; base < count; base += kAdamPack) {
    AdamPack pk{};
    pk.count = 0;
    uint32_t chunks = 0;
    for (int i = base; i < count && pk.count < kAdamPack; ++i) {
      if (n[i] == 0) continue;
      const size_t c = (n[i] + kAdamChunk - 1) / kAdamChunk;
      if (chunks + c > 0x7fffffffu) return PA_ERR_SHAPE;
      pk.w[pk.count] = w[i];
      pk.g[pk.count] = g[i];
      pk.m[pk.count] = m[i];
      pk.v[pk.count] = v[i];
      pk.n[pk.count] = n[i];
      pk.chunk_start[pk.count] = chunks;
      chunks += static_cast<uint32_t>(c);
      ++pk.count;
    }
    pk.chunk_start[pk.count] = chunks;
    if (!pk.count) continue;
    const uint32_t cap = static_cast<uint32_t>(sms()) * 8;
    adam_multi_kernel<<<chunks < cap ? chunks : cap, 256, 0, s>>>(pk, lr, b1, b2, eps, c1, c2);
    if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  }
  return PA_OK;
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
