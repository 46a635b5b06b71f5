// fp32 -> two bf16 planes (hi, lo) for the fp32 attention path.
//
// x = hi + lo + r with hi = bf16(x), lo = bf16(x - hi) (both round-to-nearest),
// so |r| <= 2^-17 |x|: about 16 mantissa bits. A product a*b is then taken as
// a_hi*b_hi + a_hi*b_lo + a_lo*b_hi on the bf16 tensor cores (the dropped
// a_lo*b_lo term is below 2^-16 relative), which keeps the fp32 path within
// 1e-3 of float64 where a single tf32 or bf16 pass would not. Rows of D
// values are written as rows of Dp >= D values, zero-padded, so the head
// dimension of the planes is a multiple of 64 (one 128-byte TMA box). The
// planes may also be a column block [c0, c0 + Dp) of wider planes with row
// pitch ldp, which gathers several [rows, D] operands into one. With a null lo
// pointer only the hi plane (the bf16 rounding of x) is written. With a mask
// (same layout as x), x is taken as zero where mask <= 0: the gradient of a
// ReLU whose output is the mask, folded into the gather.
#include <cuda_bf16.h>
#include "host_launchers.h"

namespace pa {

namespace {

// One thread per 4 output columns of one row (D % 4 == 0, 16-byte aligned x).
__global__ void split_planes_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi,
                                    __nv_bfloat16* __restrict__ lo, size_t rows, int D, int Dp,
                                    size_t ldp, int c0, const float* __restrict__ mask) {
  const int groups = Dp / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
       i < rows * groups; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / groups;
    const int c = static_cast<int>(i % groups) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < D) {
      const float4 f = *reinterpret_cast<const float4*>(x + r * D + c);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
      if (mask) {
        const float4 m = *reinterpret_cast<const float4*>(mask + r * D + c);
        v[0] = m.x > 0.f ? v[0] : 0.f;
        v[1] = m.y > 0.f ? v[1] : 0.f;
        v[2] = m.z > 0.f ? v[2] : 0.f;
        v[3] = m.w > 0.f ? v[3] : 0.f;
      }
    }
    uint32_t h2[2], l2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const uint32_t ph = pack_bf16x2(v[2 * e], v[2 * e + 1]);
      const float h0 = __uint_as_float(ph << 16), h1 = __uint_as_float(ph & 0xffff0000u);
      h2[e] = ph;
      l2[e] = pack_bf16x2(v[2 * e] - h0, v[2 * e + 1] - h1);
    }
    *reinterpret_cast<uint2*>(hi + r * ldp + c0 + c) = make_uint2(h2[0], h2[1]);
    if (lo) *reinterpret_cast<uint2*>(lo + r * ldp + c0 + c) = make_uint2(l2[0], l2[1]);
  }
}

// Any D: one thread per output element.
__global__ void split_planes_scalar_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi,
                                           __nv_bfloat16* __restrict__ lo, size_t rows, int D, int Dp,
                                           size_t ldp, int c0, const float* __restrict__ mask) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < rows * Dp;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / Dp;
    const int c = static_cast<int>(i % Dp);
    const float v = c < D && (!mask || mask[r * D + c] > 0.f) ? x[r * D + c] : 0.f;
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[r * ldp + c0 + c] = h;
    if (lo) lo[r * ldp + c0 + c] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

thread_local int t_f32_math = PA_F32_MATH_SPLIT3;

}  // namespace

int f32_math() { return t_f32_math; }
void set_f32_math(int mode) { t_f32_math = mode; }

int launch_split_planes(const float* x, void* hi, void* lo, size_t rows, int D, int Dp,
                        cudaStream_t s) {
  return launch_split_planes_into(x, hi, lo, rows, D, Dp, static_cast<size_t>(Dp), 0, s);
}

int launch_split_planes_into(const float* x, void* hi, void* lo, size_t rows, int D, int Dp,
                             size_t ldp, int c0, cudaStream_t s) {
  return launch_split_planes_masked(x, nullptr, hi, lo, rows, D, Dp, ldp, c0, s);
}

int launch_split_planes_masked(const float* x, const float* mask, void* hi, void* lo, size_t rows,
                               int D, int Dp, size_t ldp, int c0, cudaStream_t s) {
  if (D > Dp || D <= 0 || c0 < 0 || static_cast<size_t>(c0) + Dp > ldp) return PA_ERR_SHAPE;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (D % 4 != 0 || Dp % 4 != 0 || c0 % 4 != 0 || ldp % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(mask)) & 15u) != 0) {
    const size_t n = rows * Dp;
    size_t blocks = (n + 255) / 256;
    if (blocks > static_cast<size_t>(sms) * 16) blocks = static_cast<size_t>(sms) * 16;
    if (blocks == 0) blocks = 1;
    split_planes_scalar_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        x, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), rows, D, Dp, ldp, c0,
        mask);
    return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
  }
  const size_t work = rows * (Dp / 4);
  size_t blocks = (work + 255) / 256;
  if (blocks > static_cast<size_t>(sms) * 16) blocks = static_cast<size_t>(sms) * 16;
  if (blocks == 0) blocks = 1;
  split_planes_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      x, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), rows, D, Dp, ldp, c0,
      mask);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

}  // namespace pa
