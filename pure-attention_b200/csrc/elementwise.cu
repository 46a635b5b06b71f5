// Elementwise and reduction kernels of the attention block (fp32, HBM-bound):
//   bias add          matadd_kernel.cu:4-12        out[i,j] = a[i,j] + bias[j]
//   add               (same-shape residual add; the reference's pa.add only
//                      broadcast row 0, matadd_kernel.cu:10)
//   grad accumulate   tensor_add_grad_kernel.cu:4-9  dst += src
//   bias grad         sum_rows_grad_kernel.cu:4-13   db[j] += sum_i dY[i,j]
//   split / concat    split_forward_kernel.cu:4-21, split_backward_kernel.cu:4-22
// Vectorised with 16-byte accesses where the sizes allow; grids are sized in
// multiples of the SM count with grid-stride loops.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "host_launchers.h"

namespace pa {

namespace {

int sm_count() { return device_sm_count(); }

unsigned grid_for(size_t work, int threads) {
  const size_t want = (work + threads - 1) / threads;
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  return static_cast<unsigned>(want < cap ? (want > 0 ? want : 1) : cap);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__global__ void bias_add_vec_kernel(const float4* __restrict__ a, const float4* __restrict__ bias,
                                    float4* __restrict__ out, size_t n4, uint32_t n4_row) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 x = a[i], b = bias[i % n4_row];
    out[i] = make_float4(x.x + b.x, x.y + b.y, x.z + b.z, x.w + b.w);
  }
}
__global__ void bias_add_kernel(const float* __restrict__ a, const float* __restrict__ bias,
                                float* __restrict__ out, size_t n, uint32_t N) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = a[i] + bias[i % N];
}

// out = a + b (beta == 1) or out += a (b == out).
__global__ void add_vec_kernel(const float4* __restrict__ a, const float4* b, float4* out,
                               size_t n4) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 x = a[i], y = b[i];
    out[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
  }
}
__global__ void add_kernel(const float* __restrict__ a, const float* b, float* out, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = a[i] + b[i];
}

// Column sums: CTA = 32 columns x 32 row lanes; fixed-order reduction, then db += .
// (With a mask, rows of dy count only where mask > 0.)
__global__ void __launch_bounds__(1024)
    bias_grad_kernel(const float* __restrict__ dy, const float* __restrict__ mask,
                     float* __restrict__ db, uint32_t M, uint32_t N) {
  __shared__ float part[32][33];
  const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const uint32_t col = blockIdx.x * 32 + tx;
  float acc = 0.f;
  if (col < N)
    for (uint32_t r = ty; r < M; r += 32) {
      const size_t i = static_cast<size_t>(r) * N + col;
      if (!mask || mask[i] > 0.f) acc += dy[i];
    }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && col < N) {
    float s = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) s += part[k][tx];
    db[col] += s;
  }
}

// Column sums over many CTAs, stage 1: CTA (x, y) sums rows [y*rows_per,
// (y+1)*rows_per) of the 128 columns x*128.. (one float4 per lane, a warp per
// row, 8 rows in flight per CTA) into part[y][cols].
__global__ void __launch_bounds__(256)
    colsum_partial_kernel(const float* __restrict__ dy, const float* __restrict__ mask,
                          float* __restrict__ part, uint32_t M, uint32_t N, uint32_t rows_per) {
  __shared__ float4 red[8][32];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c4 = blockIdx.x * 32 + lane, n4 = N / 4;
  const uint32_t r0 = blockIdx.y * rows_per, r1 = min(M, r0 + rows_per);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c4 < n4) {
#pragma unroll 4
    for (uint32_t r = r0 + warp; r < r1; r += 8) {
      float4 v = reinterpret_cast<const float4*>(dy + static_cast<size_t>(r) * N)[c4];
      if (mask) {
        const float4 m = reinterpret_cast<const float4*>(mask + static_cast<size_t>(r) * N)[c4];
        v.x = m.x > 0.f ? v.x : 0.f;
        v.y = m.y > 0.f ? v.y : 0.f;
        v.z = m.z > 0.f ? v.z : 0.f;
        v.w = m.w > 0.f ? v.w : 0.f;
      }
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c4 < n4) {
    float4 t = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      const float4 v = red[w][lane];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    reinterpret_cast<float4*>(part + static_cast<size_t>(blockIdx.y) * N)[c4] = t;
  }
}

// colsum_partial_kernel fused with the bf16 gather of the same values: the
// projection backward's dY column block [M, D] (zero where mask <= 0) goes to
// columns [c0, c0 + Dp) of the hi (and lo) planes with row pitch ldp, columns
// D..Dp-1 as zeros, and its fp32 column sums per row chunk to part[y][D], in
// the same order as colsum_partial_kernel (so the bias gradient is the same
// bits). One read of dY (and the mask) serves both.
__global__ void __launch_bounds__(256)
    split_colsum_kernel(const float* __restrict__ dy, const float* __restrict__ mask,
                        __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo,
                        float* __restrict__ part, uint32_t M, uint32_t D, uint32_t Dp, size_t ldp,
                        uint32_t c0, uint32_t rows_per) {
  __shared__ float4 red[8][32];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c = (blockIdx.x * 32 + lane) * 4;
  const uint32_t r0 = blockIdx.y * rows_per, r1 = min(M, r0 + rows_per);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < Dp) {
#pragma unroll 4
    for (uint32_t r = r0 + warp; r < r1; r += 8) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < D) {
        v = *reinterpret_cast<const float4*>(dy + static_cast<size_t>(r) * D + c);
        if (mask) {
          const float4 m = *reinterpret_cast<const float4*>(mask + static_cast<size_t>(r) * D + c);
          v.x = m.x > 0.f ? v.x : 0.f;
          v.y = m.y > 0.f ? v.y : 0.f;
          v.z = m.z > 0.f ? v.z : 0.f;
          v.w = m.w > 0.f ? v.w : 0.f;
        }
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      const uint32_t h01 = pack_bf16x2(v.x, v.y), h23 = pack_bf16x2(v.z, v.w);
      const size_t o = static_cast<size_t>(r) * ldp + c0 + c;
      *reinterpret_cast<uint2*>(hi + o) = make_uint2(h01, h23);
      if (lo) {
        const uint32_t l01 = pack_bf16x2(v.x - __uint_as_float(h01 << 16),
                                         v.y - __uint_as_float(h01 & 0xffff0000u));
        const uint32_t l23 = pack_bf16x2(v.z - __uint_as_float(h23 << 16),
                                         v.w - __uint_as_float(h23 & 0xffff0000u));
        *reinterpret_cast<uint2*>(lo + o) = make_uint2(l01, l23);
      }
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < D) {
    float4 t = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      const float4 v = red[w][lane];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    *reinterpret_cast<float4*>(part + static_cast<size_t>(blockIdx.y) * D + c) = t;
  }
}

struct PtrPack {
  float* p[8];
};

// in[rows, parts*width] -> outs[p][rows, width]
__global__ void split_kernel(const float* __restrict__ in, PtrPack outs, uint32_t parts,
                             uint32_t width, size_t total) {
  const size_t inner = static_cast<size_t>(parts) * width;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / inner;
    const uint32_t col = static_cast<uint32_t>(i % inner);
    const uint32_t p = col / width, c = col % width;
    outs.p[p][row * width + c] = in[i];
  }
}
// grad_in[rows, parts*width] += part_grads[p][rows, width]
__global__ void concat_grad_kernel(PtrPack grads, float* __restrict__ grad_in, uint32_t parts,
                                   uint32_t width, size_t total) {
  const size_t inner = static_cast<size_t>(parts) * width;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / inner;
    const uint32_t col = static_cast<uint32_t>(i % inner);
    const uint32_t p = col / width, c = col % width;
    const float* g = grads.p[p];
    if (g) grad_in[i] += g[row * width + c];
  }
}

int done() { return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH; }

}  // namespace

int launch_bias_add(const float* a, const float* bias, float* out, uint32_t M, uint32_t N,
                    cudaStream_t s) {
  const size_t n = static_cast<size_t>(M) * N;
  if (N % 4 == 0 && al16(a) && al16(bias) && al16(out)) {
    bias_add_vec_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(
        reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(bias),
        reinterpret_cast<float4*>(out), n / 4, N / 4);
  } else {
    bias_add_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, bias, out, n, N);
  }
  return done();
}

int launch_add(const float* a, const float* b, float* out, size_t n, cudaStream_t s) {
  if (n % 4 == 0 && al16(a) && al16(b) && al16(out)) {
    add_vec_kernel<<<grid_for(n / 4, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(a),
                                                        reinterpret_cast<const float4*>(b),
                                                        reinterpret_cast<float4*>(out), n / 4);
  } else {
    add_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, out, n);
  }
  return done();
}

namespace {

// Row chunks of the two-stage column sum: about four CTAs per SM, at least
// 64 rows each; returns the rows per chunk and sets R, the chunk count.
uint32_t colsum_chunks(uint32_t M, uint32_t N, uint32_t* R) {
  const uint32_t col_blocks = (N + 127) / 128;
  uint32_t r = (4u * static_cast<uint32_t>(sm_count()) + col_blocks - 1) / col_blocks;
  if (r > (M + 63) / 64) r = (M + 63) / 64;
  if (r < 1) r = 1;
  const uint32_t rows_per = (M + r - 1) / r;
  *R = (M + rows_per - 1) / rows_per;
  return rows_per;
}

}  // namespace

size_t bias_grad_workspace_bytes(uint32_t M, uint32_t N) {
  uint32_t R = 1;
  colsum_chunks(M, N, &R);
  return static_cast<size_t>(R) * N * sizeof(float);
}

// db += column sums of dy (rows counted only where mask > 0, if given). With a
// workspace of bias_grad_workspace_bytes: rows split over enough CTAs to fill
// the GPU, partial rows to the workspace, then bias_grad_kernel sums them in
// fixed order. Without one (or for unaligned rows): one pass of 32-column CTAs.
// Deterministic for a given shape and device either way.
int launch_bias_grad(const float* dy, float* db, uint32_t M, uint32_t N, cudaStream_t s) {
  return launch_bias_grad_masked(dy, nullptr, db, M, N, nullptr, s);
}

int launch_bias_grad_masked(const float* dy, const float* mask, float* db, uint32_t M, uint32_t N,
                            float* ws, cudaStream_t s) {
  uint32_t R = 1;
  const uint32_t rows_per = colsum_chunks(M, N, &R);
  if (!ws || N % 4 != 0 || !al16(dy) || (mask && !al16(mask)) || !al16(ws) || R < 2) {
    bias_grad_kernel<<<(N + 31) / 32, 1024, 0, s>>>(dy, mask, db, M, N);
    return done();
  }
  colsum_partial_kernel<<<dim3((N + 127) / 128, R), 256, 0, s>>>(dy, mask, ws, M, N, rows_per);
  bias_grad_kernel<<<(N + 31) / 32, 1024, 0, s>>>(ws, nullptr, db, R, N);
  return done();
}

// The masked bf16 gather of launch_split_planes_masked and the bias gradient of
// launch_bias_grad_masked over the same dY block, in one read of dY: db[0, D)
// += column sums, planes as launch_split_planes_masked writes them. Shapes or
// alignments the fused kernel does not take run the two launches instead.
int launch_split_planes_colsum(const float* dy, const float* mask, void* hi, void* lo,
                               uint32_t M, int D, int Dp, size_t ldp, int c0, float* db,
                               float* ws, cudaStream_t s) {
  if (D > Dp || D <= 0 || c0 < 0 || static_cast<size_t>(c0) + Dp > ldp) return PA_ERR_SHAPE;
  uint32_t R = 1;
  const uint32_t rows_per = colsum_chunks(M, static_cast<uint32_t>(D), &R);
  if (!ws || D % 4 != 0 || Dp % 4 != 0 || c0 % 4 != 0 || ldp % 4 != 0 || !al16(dy) ||
      (mask && !al16(mask)) || !al16(ws) || R < 2) {
    const int st = launch_split_planes_masked(dy, mask, hi, lo, M, D, Dp, ldp, c0, s);
    if (st != PA_OK) return st;
    return launch_bias_grad_masked(dy, mask, db, M, static_cast<uint32_t>(D), ws, s);
  }
  split_colsum_kernel<<<dim3((Dp + 127) / 128, R), 256, 0, s>>>(
      dy, mask, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), ws, M,
      static_cast<uint32_t>(D), static_cast<uint32_t>(Dp), ldp, static_cast<uint32_t>(c0),
      rows_per);
  bias_grad_kernel<<<(D + 31) / 32, 1024, 0, s>>>(ws, nullptr, db, R, static_cast<uint32_t>(D));
  return done();
}

int launch_split_last_dim(const float* in, float* const* outs, uint32_t parts, uint32_t rows,
                          uint32_t width, cudaStream_t s) {
  PtrPack pk{};
  for (uint32_t i = 0; i < parts; ++i) pk.p[i] = outs[i];
  const size_t total = static_cast<size_t>(rows) * parts * width;
  split_kernel<<<grid_for(total, 256), 256, 0, s>>>(in, pk, parts, width, total);
  return done();
}

int launch_concat_last_dim_grad(const float* const* grads, float* grad_in, uint32_t parts,
                                uint32_t rows, uint32_t width, cudaStream_t s) {
  PtrPack pk{};
  for (uint32_t i = 0; i < parts; ++i) pk.p[i] = const_cast<float*>(grads[i]);
  const size_t total = static_cast<size_t>(rows) * parts * width;
  concat_grad_kernel<<<grid_for(total, 256), 256, 0, s>>>(pk, grad_in, parts, width, total);
  return done();
}

}  // namespace pa
