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
// ADD: the row is x + r (a residual add fused in front of the norm), also
// written to sum, which the backward and the next residual add read.
template <int VPL, bool ADD>
__global__ void __launch_bounds__(LN_WARPS * 32)
    ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ r,
                  float* __restrict__ sum, const float* __restrict__ gamma,
                  const float* __restrict__ beta, float* __restrict__ y, float* __restrict__ mean,
                  float* __restrict__ rstd, uint32_t M, uint32_t N, float eps,
                  uint32_t* __restrict__ ph, uint32_t* __restrict__ pl, uint32_t pld) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nvec = N / 4;
  for (uint32_t row = blockIdx.x * LN_WARPS + threadIdx.x / 32; row < M;
       row += gridDim.x * LN_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * N);
    const float4* rr = reinterpret_cast<const float4*>(r + static_cast<size_t>(row) * N);
    float4* sr = reinterpret_cast<float4*>(sum + static_cast<size_t>(row) * N);
    float4 v[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      v[i] = c < nvec ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (ADD && c < nvec) {
        const float4 w = rr[c];
        v[i] = make_float4(v[i].x + w.x, v[i].y + w.y, v[i].z + w.z, v[i].w + w.w);
        sr[c] = v[i];
      }
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
    // operand planes: bf16 pairs, row pitch pld bf16 values (2 words per float4)
    const size_t prow = static_cast<size_t>(row) * (pld / 2);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c], bb = b4[c];
        const float4 o = make_float4(g.x * (v[i].x - mu) * rs + bb.x, g.y * (v[i].y - mu) * rs + bb.y,
                                     g.z * (v[i].z - mu) * rs + bb.z, g.w * (v[i].w - mu) * rs + bb.w);
        yr[c] = o;
        if (ph) {  // hi = bf16(y), lo = bf16(y - hi), from the values just stored
          const uint32_t h0 = pack_bf16x2(o.x, o.y), h1 = pack_bf16x2(o.z, o.w);
          *reinterpret_cast<uint2*>(ph + prow + 2 * c) = make_uint2(h0, h1);
          if (pl)
            *reinterpret_cast<uint2*>(pl + prow + 2 * c) =
                make_uint2(pack_bf16x2(o.x - __uint_as_float(h0 << 16), o.y - __uint_as_float(h0 & 0xffff0000u)),
                           pack_bf16x2(o.z - __uint_as_float(h1 << 16), o.w - __uint_as_float(h1 & 0xffff0000u)));
        }
      } else if (ph && c == nvec && 4 * nvec < pld) {  // the pitch's zero padding (N % 8 == 4)
        *reinterpret_cast<uint2*>(ph + prow + 2 * c) = make_uint2(0u, 0u);
        if (pl) *reinterpret_cast<uint2*>(pl + prow + 2 * c) = make_uint2(0u, 0u);
      }
    }
  }
}

// Backward: dX per row (one warp per row, x and dY held in registers, with
// ACC the old dX too); dgamma / dbeta partials accumulated per warp in shared
// memory (each warp owns its [2][N] slice, so the order is fixed), summed over
// the warps in index order and written to part[blockIdx][2][N]. Holding only
// the loaded rows keeps the kernel near 100 registers, so several CTAs share
// an SM and enough loads are in flight to stream HBM.
template <int VPL, bool ACC>
__global__ void __launch_bounds__(LN_WARPS * 32)
    ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                  const float* __restrict__ mean, const float* __restrict__ rstd,
                  const float* __restrict__ gamma, float* __restrict__ dx,
                  float* __restrict__ part, uint32_t M, uint32_t N) {
  extern __shared__ float red[];  // [LN_WARPS][2][N] when part != nullptr
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const uint32_t nvec = N / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4* rg = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N);
  float4* rb = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N + N);
  if (part)
    for (uint32_t c = lane; c < nvec; c += 32) rg[c] = rb[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float inv_n = 1.f / N;
  const float fn = static_cast<float>(N);
  for (uint32_t row = blockIdx.x * LN_WARPS + warp; row < M; row += gridDim.x * LN_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * N);
    const float4* dr = reinterpret_cast<const float4*>(dy + static_cast<size_t>(row) * N);
    float4* xo = dx ? reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * N) : nullptr;
    float4 xv[VPL], dv[VPL], ov[ACC ? VPL : 1];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      const bool in = c < nvec;
      xv[i] = in ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      dv[i] = in ? dr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (ACC) ov[i] = in && xo ? xo[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float mu = mean[row], rs = rstd[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float t0 = dv[i].x * g.x, t1 = dv[i].y * g.y, t2 = dv[i].z * g.z, t3 = dv[i].w * g.w;
        s1 += (t0 + t1) + (t2 + t3);
        s2 += (t0 * (xv[i].x - mu) + t1 * (xv[i].y - mu)) + (t2 * (xv[i].z - mu) + t3 * (xv[i].w - mu));
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2) * rs;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float h0 = (xv[i].x - mu) * rs, h1 = (xv[i].y - mu) * rs;
        const float h2 = (xv[i].z - mu) * rs, h3 = (xv[i].w - mu) * rs;
        if (xo) {
          float4 o = make_float4((fn * dv[i].x * g.x - s1 - h0 * s2) * rs * inv_n,
                                 (fn * dv[i].y * g.y - s1 - h1 * s2) * rs * inv_n,
                                 (fn * dv[i].z * g.z - s1 - h2 * s2) * rs * inv_n,
                                 (fn * dv[i].w * g.w - s1 - h3 * s2) * rs * inv_n);
          if constexpr (ACC) {
            o.x += ov[i].x; o.y += ov[i].y; o.z += ov[i].z; o.w += ov[i].w;
          }
          xo[c] = o;
        }
        if (part) {
          float4 a = rg[c], b = rb[c];
          a.x += dv[i].x * h0; a.y += dv[i].y * h1; a.z += dv[i].z * h2; a.w += dv[i].w * h3;
          b.x += dv[i].x; b.y += dv[i].y; b.z += dv[i].z; b.w += dv[i].w;
          rg[c] = a;
          rb[c] = b;
        }
      }
    }
  }
  if (!part) return;
  __syncthreads();
  float* out = part + static_cast<size_t>(blockIdx.x) * 2 * N;
  for (uint32_t c = threadIdx.x; c < 2 * N; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < LN_WARPS; ++w) acc += red[static_cast<size_t>(w) * 2 * N + c];
    out[c] = acc;
  }
}

// Backward of sum = x + r, y = LN(sum): G = LN_bwd(dY) + dS, with dS the
// gradient that reached the sum from its other consumers (null: none), goes
// to both addends' gradients in one pass: dx = G (+ old dx when acc_dx), dr =
// G (+ old dr when acc_dr); either may be null, and they may be the same
// buffer (x + x), which then receives 2G. dgamma / dbeta partials as in
// ln_bwd_kernel. dS and the old gradients are read only when the row is
// written, so the registers held across the row reductions are ln_bwd_kernel's.
template <int VPL>
__global__ void __launch_bounds__(LN_WARPS * 32)
    add_ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ dsum,
                      const float* __restrict__ x, const float* __restrict__ mean,
                      const float* __restrict__ rstd, const float* __restrict__ gamma, float* dx,
                      int acc_dx, float* dr, int acc_dr, float* __restrict__ part, uint32_t M,
                      uint32_t N) {
  extern __shared__ float red[];  // [LN_WARPS][2][N] when part != nullptr
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x / 32;
  const uint32_t nvec = N / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4* rg = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N);
  float4* rb = reinterpret_cast<float4*>(red + static_cast<size_t>(warp) * 2 * N + N);
  if (part)
    for (uint32_t c = lane; c < nvec; c += 32) rg[c] = rb[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float inv_n = 1.f / N;
  const float fn = static_cast<float>(N);
  auto add4 = [](float4 a, const float4 b) {
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    return a;
  };
  for (uint32_t row = blockIdx.x * LN_WARPS + warp; row < M; row += gridDim.x * LN_WARPS) {
    const size_t off = static_cast<size_t>(row) * N;
    const float4* xr = reinterpret_cast<const float4*>(x + off);
    const float4* dyr = reinterpret_cast<const float4*>(dy + off);
    const float4* dsr = dsum ? reinterpret_cast<const float4*>(dsum + off) : nullptr;
    float4* xo = dx ? reinterpret_cast<float4*>(dx + off) : nullptr;
    float4* ro = dr ? reinterpret_cast<float4*>(dr + off) : nullptr;
    // The sum's own gradient is loaded with x and dY, before the row sums, so
    // its latency hides behind theirs (read in the output pass it cost 17%).
    float4 xv[VPL], dv[VPL], sv[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      const bool in = c < nvec;
      xv[i] = in ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      dv[i] = in ? dyr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      sv[i] = in && dsr ? dsr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float mu = mean[row], rs = rstd[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float t0 = dv[i].x * g.x, t1 = dv[i].y * g.y, t2 = dv[i].z * g.z, t3 = dv[i].w * g.w;
        s1 += (t0 + t1) + (t2 + t3);
        s2 += (t0 * (xv[i].x - mu) + t1 * (xv[i].y - mu)) + (t2 * (xv[i].z - mu) + t3 * (xv[i].w - mu));
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2) * rs;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t c = lane + 32 * i;
      if (c < nvec) {
        const float4 g = g4[c];
        const float h0 = (xv[i].x - mu) * rs, h1 = (xv[i].y - mu) * rs;
        const float h2 = (xv[i].z - mu) * rs, h3 = (xv[i].w - mu) * rs;
        if (xo || ro) {
          float4 o = make_float4((fn * dv[i].x * g.x - s1 - h0 * s2) * rs * inv_n,
                                 (fn * dv[i].y * g.y - s1 - h1 * s2) * rs * inv_n,
                                 (fn * dv[i].z * g.z - s1 - h2 * s2) * rs * inv_n,
                                 (fn * dv[i].w * g.w - s1 - h3 * s2) * rs * inv_n);
          if (dsr) o = add4(o, sv[i]);
          if (xo) xo[c] = acc_dx ? add4(o, xo[c]) : o;
          if (ro) ro[c] = acc_dr ? add4(o, ro[c]) : o;
        }
        if (part) {
          float4 a = rg[c], b = rb[c];
          a.x += dv[i].x * h0; a.y += dv[i].y * h1; a.z += dv[i].z * h2; a.w += dv[i].w * h3;
          b.x += dv[i].x; b.y += dv[i].y; b.z += dv[i].z; b.w += dv[i].w;
          rg[c] = a;
          rb[c] = b;
        }
      }
    }
  }
  if (!part) return;
  __syncthreads();
  float* out = part + static_cast<size_t>(blockIdx.x) * 2 * N;
  for (uint32_t c = threadIdx.x; c < 2 * N; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < LN_WARPS; ++w) acc += red[static_cast<size_t>(w) * 2 * N + c];
    out[c] = acc;
  }
}

// dgamma[c] += sum_b part[b][0][c]; dbeta[c] += sum_b part[b][1][c] (fixed
// order). CTA = 32 of the 2N columns x 32 lanes over the partial rows.
__global__ void __launch_bounds__(1024)
    ln_param_reduce_kernel(const float* __restrict__ part, float* __restrict__ dgamma,
                           float* __restrict__ dbeta, uint32_t nblk, uint32_t N) {
  __shared__ float red[32][33];
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const uint32_t c = blockIdx.x * 32 + tx;
  float acc = 0.f;
  if (c < 2 * N)
    for (uint32_t k = ty; k < nblk; k += 32) acc += part[static_cast<size_t>(k) * 2 * N + c];
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < 2 * N) {
    float t = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) t += red[k][tx];
    float* out = c < N ? dgamma : dbeta;
    if (out) out[c < N ? c : c - N] += t;
  }
}

int num_sms() { return device_sm_count(); }

// One wave of CTAs: two per SM for rows of up to 1024 values (about 100-130
// registers per thread, 64 KB of partials), three for shorter rows.
uint32_t ln_bwd_blocks(uint32_t M, uint32_t N) {
  const uint32_t want = (M + LN_WARPS - 1) / LN_WARPS;
  const uint32_t cap = static_cast<uint32_t>(num_sms()) * (N > 512 ? 2 : 3);
  return want < cap ? want : cap;
}

template <int VPL>
int ln_fwd_launch(const float* x, const float* r, float* sum, const float* g, const float* b,
                  float* y, float* mu, float* rs, uint32_t M, uint32_t N, float eps, void* ph,
                  void* pl, uint32_t pld, cudaStream_t s) {
  const uint32_t blocks = (M + LN_WARPS - 1) / LN_WARPS;
  uint32_t* h = static_cast<uint32_t*>(ph);
  uint32_t* l = static_cast<uint32_t*>(pl);
  if (r)
    ln_fwd_kernel<VPL, true><<<blocks, LN_WARPS * 32, 0, s>>>(x, r, sum, g, b, y, mu, rs, M, N, eps,
                                                              h, l, pld);
  else
    ln_fwd_kernel<VPL, false><<<blocks, LN_WARPS * 32, 0, s>>>(x, nullptr, nullptr, g, b, y, mu, rs,
                                                               M, N, eps, h, l, pld);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

template <int VPL>
int ln_bwd_launch(const float* dy, const float* x, const float* mu, const float* rs,
                  const float* g, float* dx, float* dg, float* db, uint32_t M, uint32_t N,
                  float* part, int accumulate, cudaStream_t s) {
  const uint32_t blocks = ln_bwd_blocks(M, N);
  const size_t smem = static_cast<size_t>(LN_WARPS) * 2 * N * sizeof(float);
  float* p = (dg || db) ? part : nullptr;
  if (accumulate && dx) {
    static std::atomic<uint64_t> attr{0};
    if (!ensure_smem_attr(ln_bwd_kernel<VPL, true>, static_cast<int>(LN_WARPS * 2 * 128 * VPL * 4),
                          attr))
      return PA_ERR_LAUNCH;
    ln_bwd_kernel<VPL, true><<<blocks, LN_WARPS * 32, p ? smem : 0, s>>>(dy, x, mu, rs, g, dx, p,
                                                                          M, N);
  } else {
    static std::atomic<uint64_t> attr{0};
    if (!ensure_smem_attr(ln_bwd_kernel<VPL, false>, static_cast<int>(LN_WARPS * 2 * 128 * VPL * 4),
                          attr))
      return PA_ERR_LAUNCH;
    ln_bwd_kernel<VPL, false><<<blocks, LN_WARPS * 32, p ? smem : 0, s>>>(dy, x, mu, rs, g, dx, p,
                                                                           M, N);
  }
  if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  if (dg || db) {
    ln_param_reduce_kernel<<<(2 * N + 31) / 32, 1024, 0, s>>>(part, dg, db, blocks, N);
    if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  }
  return PA_OK;
}

template <int VPL>
int add_ln_bwd_launch(const float* dy, const float* dsum, const float* x, const float* mu,
                      const float* rs, const float* g, float* dx, int acc_dx, float* dr, int acc_dr,
                      float* dg, float* db, uint32_t M, uint32_t N, float* part, cudaStream_t s) {
  const uint32_t blocks = ln_bwd_blocks(M, N);
  const size_t smem = static_cast<size_t>(LN_WARPS) * 2 * N * sizeof(float);
  float* p = (dg || db) ? part : nullptr;
  static std::atomic<uint64_t> attr{0};
  if (!ensure_smem_attr(add_ln_bwd_kernel<VPL>, static_cast<int>(LN_WARPS * 2 * 128 * VPL * 4),
                        attr))
    return PA_ERR_LAUNCH;
  add_ln_bwd_kernel<VPL><<<blocks, LN_WARPS * 32, p ? smem : 0, s>>>(
      dy, dsum, x, mu, rs, g, dx, acc_dx, dr, acc_dr, p, M, N);
  if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  if (dg || db) {
    ln_param_reduce_kernel<<<(2 * N + 31) / 32, 1024, 0, s>>>(part, dg, db, blocks, N);
    if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;
  }
  return PA_OK;
}

}  // namespace

// r == nullptr: y = LN(x); else sum = x + r and y = LN(sum).
int launch_layer_norm_fwd(const float* x, const float* r, float* sum, const float* g,
                          const float* b, float* y, float* mu, float* rs, uint32_t M, uint32_t N,
                          float eps, cudaStream_t s, void* ph, void* pl, uint32_t pld) {
  if (ph && (pld < N || pld > N + 4 || pld % 4 != 0)) return PA_ERR_SHAPE;
  if (N <= 128) return ln_fwd_launch<1>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  if (N <= 256) return ln_fwd_launch<2>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  if (N <= 512) return ln_fwd_launch<4>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  if (N <= 1024) return ln_fwd_launch<8>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  if (N <= 2048) return ln_fwd_launch<16>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  if (N <= 4096) return ln_fwd_launch<32>(x, r, sum, g, b, y, mu, rs, M, N, eps, ph, pl, pld, s);
  return PA_ERR_UNSUPPORTED;
}

size_t layer_norm_bwd_workspace_bytes(uint32_t M, uint32_t N) {
  return static_cast<size_t>(ln_bwd_blocks(M, N)) * 2 * N * sizeof(float);
}

int launch_layer_norm_bwd(const float* dy, const float* x, const float* mu, const float* rs,
                          const float* g, float* dx, float* dg, float* db, uint32_t M, uint32_t N,
                          float* part, int acc, cudaStream_t s) {
  if (N <= 128) return ln_bwd_launch<1>(dy, x, mu, rs, g, dx, dg, db, M, N, part, acc, s);
  if (N <= 256) return ln_bwd_launch<2>(dy, x, mu, rs, g, dx, dg, db, M, N, part, acc, s);
  if (N <= 512) return ln_bwd_launch<4>(dy, x, mu, rs, g, dx, dg, db, M, N, part, acc, s);
  if (N <= 1024) return ln_bwd_launch<8>(dy, x, mu, rs, g, dx, dg, db, M, N, part, acc, s);
  return PA_ERR_UNSUPPORTED;
}

int launch_add_layer_norm_bwd(const float* dy, const float* dsum, const float* x, const float* mu,
                              const float* rs, const float* g, float* dx, int acc_dx, float* dr,
                              int acc_dr, float* dg, float* db, uint32_t M, uint32_t N,
                              float* part, cudaStream_t s) {
  if (N <= 128)
    return add_ln_bwd_launch<1>(dy, dsum, x, mu, rs, g, dx, acc_dx, dr, acc_dr, dg, db, M, N, part, s);
  if (N <= 256)
    return add_ln_bwd_launch<2>(dy, dsum, x, mu, rs, g, dx, acc_dx, dr, acc_dr, dg, db, M, N, part, s);
  if (N <= 512)
    return add_ln_bwd_launch<4>(dy, dsum, x, mu, rs, g, dx, acc_dx, dr, acc_dr, dg, db, M, N, part, s);
  if (N <= 1024)
    return add_ln_bwd_launch<8>(dy, dsum, x, mu, rs, g, dx, acc_dx, dr, acc_dr, dg, db, M, N, part, s);
  return PA_ERR_UNSUPPORTED;
}

}  // namespace pa
