// LayerNorm forward / backward (fp32), HBM-bound.
//
// Forward restates layer_norm_forward_kernel.cu:40-82: per row, mean and
// biased variance, rstd = 1/sqrt(var + eps), y = gamma * (x - mean) * rstd + beta.
// Backward restates layer_norm_backward.cu:17-157:
//   dX = rstd/N * (N*dY*gamma - sum(dY*gamma) - xhat*sum(dY*gamma*xhat))  (overwrite)
//   dgamma += sum_rows dY*xhat, dbeta += sum_rows dY                       (accumulate)
//
// B200 layout: one warp per row, each lane owning 4-float (16-byte) columns
// lane*4 + 128*i, so every load is a coalesced 128-bit access and the row stays
// in registers between the statistics and the output pass (one HBM read of x).
// Row sums are warp shuffles (the reference's dX block sums race, D9 there).
// dgamma/dbeta are reduced deterministically: per-CTA partials to the
// workspace, then a fixed-order column sum.
#include <cuda_runtime.h>
#include <cstdint>
#include "host_launchers.h"

namespace pa {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int LN_WARPS = 8;  // rows in flight per CTA

// VPL = float4 vectors per lane (row length N <= 128 * VPL, N % 4 == 0).
template <int VPL>
__global__ void __launch_bounds__(LN_WARPS * 32)
    ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                  const float* __restrict__ beta, float* __restrict__ y, float* __restrict__ mean,
                  float* __restrict__ rstd, uint32_t M, uint32_t N, float eps) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nvec = N / 4;
  for (uint32_t row = blockIdx.x * LN_WARPS + threadIdx.x / 32; row < M;
       row += gridDim.x * LN_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * N);
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      v[i] = c < nvec ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    const float mu = warp_sum(s) / N;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float a = v[i].x - mu, b = v[i].y - mu, cc = v[i].z - mu, d = v[i].w - mu;
        s2 += (a * a + b * b) + (cc * cc + d * d);
      }
    }
    const float rs = rsqrtf(warp_sum(s2) / N + eps);
    if (lane == 0) {
      mean[row] = mu;
      rstd[row] = rs;
    }
    float4* yr = reinterpret_cast<float4*>(y + static_cast<size_t>(row) * N);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c], bb = b4[c];
        yr[c] = make_float4(g.x * (v[i].x - mu) * rs + bb.x, g.y * (v[i].y - mu) * rs + bb.y,
                            g.z * (v[i].z - mu) * rs + bb.z, g.w * (v[i].w - mu) * rs + bb.w);
      }
    }
  }
}

// Backward: dX per row; per-CTA partial dgamma/dbeta written to part[blockIdx][2][N].
template <int VPL>
__global__ void __launch_bounds__(LN_WARPS * 32)
    ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                  const float* __restrict__ mean, const float* __restrict__ rstd,
                  const float* __restrict__ gamma, float* __restrict__ dx,
                  float* __restrict__ part, uint32_t M, uint32_t N) {
  extern __shared__ float red[];  // [LN_WARPS][2][N]
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const uint32_t nvec = N / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4 pg[VPL], pb[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) pg[i] = pb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t row = blockIdx.x * LN_WARPS + warp; row < M; row += gridDim.x * LN_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * N);
    const float4* dr = reinterpret_cast<const float4*>(dy + static_cast<size_t>(row) * N);
    const float mu = mean[row], rs = rstd[row];
    float4 xh[VPL], t[VPL];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 xv = xr[c], dv = dr[c], g = g4[c];
        xh[i] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs, (xv.w - mu) * rs);
        t[i] = make_float4(dv.x * g.x, dv.y * g.y, dv.z * g.z, dv.w * g.w);
        s1 += (t[i].x + t[i].y) + (t[i].z + t[i].w);
        s2 += (t[i].x * xh[i].x + t[i].y * xh[i].y) + (t[i].z * xh[i].z + t[i].w * xh[i].w);
        pg[i].x += dv.x * xh[i].x; pg[i].y += dv.y * xh[i].y;
        pg[i].z += dv.z * xh[i].z; pg[i].w += dv.w * xh[i].w;
        pb[i].x += dv.x; pb[i].y += dv.y; pb[i].z += dv.z; pb[i].w += dv.w;
      }
    }
    if (dx) {
      s1 = warp_sum(s1);
      s2 = warp_sum(s2);
      const float inv_n = 1.f / N;
      const float fn = static_cast<float>(N);
      float4* xo = reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * N);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const uint32_t c = lane + 32 * i;
        if (c < nvec)
          xo[c] = make_float4((fn * t[i].x - s1 - xh[i].x * s2) * rs * inv_n,
                              (fn * t[i].y - s1 - xh[i].y * s2) * rs * inv_n,
                              (fn * t[i].z - s1 - xh[i].z * s2) * rs * inv_n,
                              (fn * t[i].w - s1 - xh[i].w * s2) * rs * inv_n);
      }
    }
  }
  if (!part) return;
  float4* rg = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N);
  float4* rb = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N + N);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint32_t c = lane + 32 * i;
    if (c < nvec) {
      rg[c] = pg[i];
      rb[c] = pb[i];
    }
  }
  __syncthreads();
  float* out = part + static_cast<size_t>(blockIdx.x) * 2 * N;
  for (uint32_t c = threadIdx.x; c < 2 * N; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < LN_WARPS; ++w) acc += red[static_cast<size_t>(w) * 2 * N + c];
    out[c] = acc;
  }
}

// dgamma[c] += sum_b part[b][0][c]; dbeta[c] += sum_b part[b][1][c] (fixed order).
__global__ void ln_param_reduce_kernel(const float* __restrict__ part, float* __restrict__ dgamma,
                                       float* __restrict__ dbeta, uint32_t nblk, uint32_t N) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  float g = 0.f, b = 0.f;
  for (uint32_t k = 0; k < nblk; ++k) {
    g += part[static_cast<size_t>(k) * 2 * N + c];
    b += part[static_cast<size_t>(k) * 2 * N + N + c];
  }
  if (dgamma) dgamma[c] += g;
  if (dbeta) dbeta[c] += b;
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] > 0 ? sms[dev] : 148;
}

uint32_t ln_bwd_blocks(uint32_t M) {
  const uint32_t want = (M + LN_WARPS - 1) / LN_WARPS;
  const uint32_t cap = static_cast<uint32_t>(num_sms()) * 4;
  return want < cap ? want : cap;
}

template <int VPL>
int ln_fwd_launch(const float* x, const float* g, const float* b, float* y, float* mu, float* rs,
                  uint32_t M, uint32_t N, float eps, cudaStream_t s) {
  const uint32_t blocks = (M + LN_WARPS - 1) / LN_WARPS;
  ln_fwd_kernel<VPL><<<blocks, LN_WARPS * 32, 0, s>>>(x, g, b, y, mu, rs, M, N, eps);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

template <int VPL>
int ln_bwd_launch(const float* dy, const float* x, const float* mu, const float* rs,
                  const float* g, float* dx, float* dg, float* db, uint32_t M, uint32_t N,
                  float* part, cudaStream_t s) {
  const uint32_t blocks = ln_bwd_blocks(M);
  const size_t smem = static_cast<size_t>(LN_WARPS) * 2 * N * sizeof(float);
  static uint64_t attr = 0;
  ensure_smem_attr(ln_bwd_kernel<VPL>, static_cast<int>(LN_WARPS * 2 * 128 * VPL * 4), attr);
  ln_bwd_kernel<VPL><<<blocks, LN_WARPS * 32, (dg || db) ? smem : 0, s>>>(
      dy, x, mu, rs, g, dx, (dg || db) ? part : nullptr, M, N);
  if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  if (dg || db) {
    ln_param_reduce_kernel<<<(N + 255) / 256, 256, 0, s>>>(part, dg, db, blocks, N);
    if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  }
  return PA_OK;
}

}  // namespace

int launch_layer_norm_fwd(const float* x, const float* g, const float* b, float* y, float* mu,
                          float* rs, uint32_t M, uint32_t N, float eps, cudaStream_t s) {
  if (N <= 128) return ln_fwd_launch<1>(x, g, b, y, mu, rs, M, N, eps, s);
  if (N <= 256) return ln_fwd_launch<2>(x, g, b, y, mu, rs, M, N, eps, s);
  if (N <= 512) return ln_fwd_launch<4>(x, g, b, y, mu, rs, M, N, eps, s);
  if (N <= 1024) return ln_fwd_launch<8>(x, g, b, y, mu, rs, M, N, eps, s);
  if (N <= 2048) return ln_fwd_launch<16>(x, g, b, y, mu, rs, M, N, eps, s);
  if (N <= 4096) return ln_fwd_launch<32>(x, g, b, y, mu, rs, M, N, eps, s);
  return PA_ERR_UNSUPPORTED;
}

size_t layer_norm_bwd_workspace_bytes(uint32_t M, uint32_t N) {
  return static_cast<size_t>(ln_bwd_blocks(M)) * 2 * N * sizeof(float);
}

int launch_layer_norm_bwd(const float* dy, const float* x, const float* mu, const float* rs,
                          const float* g, float* dx, float* dg, float* db, uint32_t M, uint32_t N,
                          float* part, cudaStream_t s) {
  if (N <= 128) return ln_bwd_launch<1>(dy, x, mu, rs, g, dx, dg, db, M, N, part, s);
  if (N <= 256) return ln_bwd_launch<2>(dy, x, mu, rs, g, dx, dg, db, M, N, part, s);
  if (N <= 512) return ln_bwd_launch<4>(dy, x, mu, rs, g, dx, dg, db, M, N, part, s);
  if (N <= 1024) return ln_bwd_launch<8>(dy, x, mu, rs, g, dx, dg, db, M, N, part, s);
  return PA_ERR_UNSUPPORTED;
}

}  // namespace pa
