// C-ABI harness around the reference's OWN CUDA launchers, compiled together
// with the unmodified Pure-Attention sources into oracle/_ref/libpa_ref.so.
//
// TEST INFRASTRUCTURE ONLY: the GPU parity tests call it to compare the B200
// kernels (and the float64 oracle) with what the reference itself computes.
// Inputs and outputs are HOST fp32 arrays; each call allocates, uploads,
// launches the reference launcher, synchronises and downloads.
//
// Deviations from calling the reference unchanged, each forced by a defect:
//  - the LSE buffer passed to launch_flash_attention holds B*H*L floats (the
//    reference's own core::flash_attention allocates B*H*ceil(L/16), which the
//    kernel overruns; launcher_flash_attn_forward.cu:5-72 takes it from the caller);
//  - ref_flash_bwd_relaunch_d64 launches the reference's
//    flash_attn_backward_kernel<64,16,64> template with a grid and shared-memory
//    size computed for Bc = 64, because launch_flash_backward sizes both for
//    Bc = 32 while instantiating Bc = 64 (launcher_flash_attn_backward.cu:21-36),
//    which addresses shared memory past its allocation. The shipped d = 32 path
//    is called unchanged (ref_flash_bwd).
#include <cuda_runtime.h>
#include <memory>
#include <vector>
#include <backend/Kernels.cuh>
#include <backend/Launchers.cuh>
#include <core/Tensor.h>

namespace {

float* up(const float* h, size_t n) {
  float* d = nullptr;
  if (cudaMalloc(&d, n * sizeof(float)) != cudaSuccess) return nullptr;
  if (h) cudaMemcpy(d, h, n * sizeof(float), cudaMemcpyHostToDevice);
  else cudaMemset(d, 0, n * sizeof(float));
  return d;
}
void down(float* h, const float* d, size_t n) {
  if (h && d) cudaMemcpy(h, d, n * sizeof(float), cudaMemcpyDeviceToHost);
}
int finish() {
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

}  // namespace

extern "C" {

// launch_flash_attention (launcher_flash_attn_forward.cu:5-72) on [B, L, H*D].
int ref_flash_fwd(const float* q, const float* k, const float* v, float* o, float* lse, int B,
                  int L, int H, int D) {
  const uint32_t E = static_cast<uint32_t>(H * D);
  const std::vector<uint32_t> shp = {static_cast<uint32_t>(B), static_cast<uint32_t>(L), E};
  const size_t n = static_cast<size_t>(B) * L * E;
  auto Q = std::make_shared<core::Tensor>(shp, false);
  auto K = std::make_shared<core::Tensor>(shp, false);
  auto V = std::make_shared<core::Tensor>(shp, false);
  auto O = std::make_shared<core::Tensor>(shp, false);
  auto Lc = std::make_shared<core::Tensor>(
      std::vector<uint32_t>{static_cast<uint32_t>(B * H), static_cast<uint32_t>(L)}, false);
  Q->to_device(std::vector<float>(q, q + n));
  K->to_device(std::vector<float>(k, k + n));
  V->to_device(std::vector<float>(v, v + n));
  launch_flash_attention(Q, K, V, O, Lc, H, nullptr);
  const int st = finish();
  if (st) return st;
  auto ho = O->to_host();
  auto hl = Lc->to_host();
  cudaDeviceSynchronize();
  std::copy(ho.begin(), ho.end(), o);
  std::copy(hl.begin(), hl.end(), lse);
  return 0;
}

// launch_flash_backward (launcher_flash_attn_backward.cu:4-53), shipped path
// (only safe at D = 32). dq is the reference's debug stub and is returned as is.
int ref_flash_bwd(const float* q, const float* k, const float* v, const float* o, const float* dO,
                  const float* lse, float* dq, float* dk, float* dv, int B, int L, int H, int D) {
  if (D != 32) return -1;
  const size_t n = static_cast<size_t>(B) * L * H * D;
  float *Q = up(q, n), *K = up(k, n), *V = up(v, n), *O = up(o, n), *G = up(dO, n);
  float* Lv = up(lse, static_cast<size_t>(B) * H * L);
  float *dQ = up(nullptr, n), *dK = up(nullptr, n), *dV = up(nullptr, n);
  launch_flash_backward(Q, K, V, O, G, Lv, dQ, dK, dV, B, H, L, H * D, nullptr);
  const int st = finish();
  down(dq, dQ, n);
  down(dk, dK, n);
  down(dv, dV, n);
  for (float* p : {Q, K, V, O, G, Lv, dQ, dK, dV}) cudaFree(p);
  return st;
}

// The reference's compute_delta_kernel + flash_attn_backward_kernel<64,16,64>,
// relaunched with Bc = 64 geometry (grid ceil(L/64) x B*H, 64 threads,
// (4*64*72 + 2*16*72)*4 bytes of shared memory). Requires L % 64 == 0.
int ref_flash_bwd_relaunch_d64(const float* q, const float* k, const float* v, const float* o,
                               const float* dO, const float* lse, float* dk, float* dv, int B,
                               int L, int H) {
  const int D = 64, Bc = 64, Br = 16, PAD = 8;
  if (L % Bc != 0) return -1;
  const size_t n = static_cast<size_t>(B) * L * H * D;
  float *Q = up(q, n), *K = up(k, n), *V = up(v, n), *O = up(o, n), *G = up(dO, n);
  float* Lv = up(lse, static_cast<size_t>(B) * H * L);
  float *dQ = up(nullptr, n), *dK = up(nullptr, n), *dV = up(nullptr, n);
  float* Delta = up(nullptr, static_cast<size_t>(B) * H * L);
  const int threads = 256;
  const int blocks = (B * H * L + threads - 1) / threads;
  compute_delta_kernel<<<blocks, threads>>>(G, O, Delta, B, H, L, D);
  const size_t smem = (4 * Bc * (D + PAD) + 2 * Br * (D + PAD)) * sizeof(float);
  cudaFuncSetAttribute(flash_attn_backward_kernel<64, 16, 64>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  dim3 grid(L / Bc, B * H);
  flash_attn_backward_kernel<64, 16, 64><<<grid, 64, smem>>>(
      Q, K, V, O, G, Lv, Delta, dQ, dK, dV, L * H * D, D, H * D, L, 1.0f / 8.0f);
  const int st = finish();
  down(dk, dK, n);
  down(dv, dV, n);
  for (float* p : {Q, K, V, O, G, Lv, dQ, dK, dV, Delta}) cudaFree(p);
  return st;
}

// launch_layer_norm_forward (launcher_layer_norm_forward.cu:4-28).
int ref_layer_norm_fwd(const float* x, const float* gamma, const float* beta, float* y, float* mean,
                       float* rstd, int M, int N, float eps) {
  const size_t n = static_cast<size_t>(M) * N;
  float *X = up(x, n), *Gm = up(gamma, N), *Bt = up(beta, N), *Y = up(nullptr, n);
  float *Mu = up(nullptr, M), *Rs = up(nullptr, M);
  launch_layer_norm_forward(X, Gm, Bt, Y, Mu, Rs, M, N, eps, nullptr);
  const int st = finish();
  down(y, Y, n);
  down(mean, Mu, M);
  down(rstd, Rs, M);
  for (float* p : {X, Gm, Bt, Y, Mu, Rs}) cudaFree(p);
  return st;
}

// launch_layer_norm_backward (launcher_layer_norm_backward.cu:5-48); dgamma and
// dbeta start at zero (as after the reference's forward, Functional.cpp:318-324).
int ref_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                       const float* gamma, float* dx, float* dgamma, float* dbeta, int M, int N) {
  const size_t n = static_cast<size_t>(M) * N;
  float *dY = up(dy, n), *X = up(x, n), *Mu = up(mean, M), *Rs = up(rstd, M), *Gm = up(gamma, N);
  float *dX = up(nullptr, n), *dG = up(nullptr, N), *dB = up(nullptr, N);
  launch_layer_norm_backward(dY, X, Mu, Rs, Gm, dX, dG, dB, M, N, nullptr);
  const int st = finish();
  down(dx, dX, n);
  down(dgamma, dG, N);
  down(dbeta, dB, N);
  for (float* p : {dY, X, Mu, Rs, Gm, dX, dG, dB}) cudaFree(p);
  return st;
}

// launch_matmul_tiled (launcher_matmul_forward.cu:4-15): C = A B.
int ref_matmul(const float* a, const float* b, float* c, int M, int N, int K) {
  float *A = up(a, static_cast<size_t>(M) * K), *Bm = up(b, static_cast<size_t>(K) * N);
  float* C = up(nullptr, static_cast<size_t>(M) * N);
  launch_matmul_tiled(A, Bm, C, M, N, K, nullptr);
  const int st = finish();
  down(c, C, static_cast<size_t>(M) * N);
  for (float* p : {A, Bm, C}) cudaFree(p);
  return st;
}

// launch_matmul_grad_X (launcher_matmul_backward.cu:4-11): dX += dY W^T (dX in/out).
int ref_matmul_grad_x(const float* dy, const float* w, float* dx, int M, int N, int K) {
  float *dY = up(dy, static_cast<size_t>(M) * K), *W = up(w, static_cast<size_t>(N) * K);
  float* dX = up(dx, static_cast<size_t>(M) * N);
  launch_matmul_grad_X(dY, W, dX, M, N, K, nullptr);
  const int st = finish();
  down(dx, dX, static_cast<size_t>(M) * N);
  for (float* p : {dY, W, dX}) cudaFree(p);
  return st;
}

// launch_matmul_grad_W (launcher_matmul_backward.cu:13-20): dW += X^T dY (dW in/out).
int ref_matmul_grad_w(const float* x, const float* dy, float* dw, int M, int N, int K) {
  float *X = up(x, static_cast<size_t>(M) * N), *dY = up(dy, static_cast<size_t>(M) * K);
  float* dW = up(dw, static_cast<size_t>(N) * K);
  launch_matmul_grad_W(X, dY, dW, M, N, K, nullptr);
  const int st = finish();
  down(dw, dW, static_cast<size_t>(N) * K);
  for (float* p : {X, dY, dW}) cudaFree(p);
  return st;
}

}  // extern "C"

// ---------------------------------------------------------------- timing
// The reference's attention kernels timed on the GPU (CUDA events, after one
// untimed launch): launch_flash_attention, then the backward - the shipped
// launch_flash_backward at D = 32 (which allocates its temporaries inside each
// call), or at D = 64 compute_delta_kernel plus flash_attn_backward_kernel<64,16,64>
// with the in-bounds Bc = 64 geometry of ref_flash_bwd_relaunch_d64. Inputs are
// host fp32 [B, L, H*D]; the average milliseconds per call are written to
// fwd_ms and bwd_ms. Returns 0 or a CUDA error code.
extern "C" int ref_time_flash(const float* q, const float* k, const float* v, const float* dO,
                              int B, int L, int H, int D, int reps, float* fwd_ms,
                              float* bwd_ms) {
  if ((D != 32 && D != 64) || reps <= 0) return -1;
  if (D == 64 && L % 64 != 0) return -1;
  const uint32_t E = static_cast<uint32_t>(H * D);
  const std::vector<uint32_t> shp = {static_cast<uint32_t>(B), static_cast<uint32_t>(L), E};
  const size_t n = static_cast<size_t>(B) * L * E;
  auto Q = std::make_shared<core::Tensor>(shp, false);
  auto K = std::make_shared<core::Tensor>(shp, false);
  auto V = std::make_shared<core::Tensor>(shp, false);
  auto O = std::make_shared<core::Tensor>(shp, false);
  auto Lc = std::make_shared<core::Tensor>(
      std::vector<uint32_t>{static_cast<uint32_t>(B * H), static_cast<uint32_t>(L)}, false);
  Q->to_device(std::vector<float>(q, q + n));
  K->to_device(std::vector<float>(k, k + n));
  V->to_device(std::vector<float>(v, v + n));
  float* G = up(dO, n);
  float *dQ = up(nullptr, n), *dK = up(nullptr, n), *dV = up(nullptr, n);
  float* Delta = up(nullptr, static_cast<size_t>(B) * H * L);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  auto bwd = [&]() {
    if (D == 32) {
      launch_flash_backward(Q->get_data_ptr(), K->get_data_ptr(), V->get_data_ptr(),
                            O->get_data_ptr(), G, Lc->get_data_ptr(), dQ, dK, dV, B, H, L, H * D,
                            nullptr);
      return;
    }
    const int Bc = 64, Br = 16, PAD = 8;
    const int blocks = (B * H * L + 255) / 256;
    compute_delta_kernel<<<blocks, 256>>>(G, O->get_data_ptr(), Delta, B, H, L, D);
    const size_t smem = (4 * Bc * (D + PAD) + 2 * Br * (D + PAD)) * sizeof(float);
    cudaFuncSetAttribute(flash_attn_backward_kernel<64, 16, 64>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    flash_attn_backward_kernel<64, 16, 64><<<dim3(L / Bc, B * H), 64, smem>>>(
        Q->get_data_ptr(), K->get_data_ptr(), V->get_data_ptr(), O->get_data_ptr(), G,
        Lc->get_data_ptr(), Delta, dQ, dK, dV, L * H * D, D, H * D, L, 1.0f / 8.0f);
  };
  launch_flash_attention(Q, K, V, O, Lc, H, nullptr);
  bwd();
  int st = finish();
  if (st == 0) {
    cudaEventRecord(e0);
    for (int i = 0; i < reps; ++i) launch_flash_attention(Q, K, V, O, Lc, H, nullptr);
    cudaEventRecord(e1);
    st = finish();
    cudaEventElapsedTime(fwd_ms, e0, e1);
    *fwd_ms /= reps;
  }
  if (st == 0) {
    cudaEventRecord(e0);
    for (int i = 0; i < reps; ++i) bwd();
    cudaEventRecord(e1);
    st = finish();
    cudaEventElapsedTime(bwd_ms, e0, e1);
    *bwd_ms /= reps;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  for (float* p : {G, dQ, dK, dV, Delta}) cudaFree(p);
  return st;
}
