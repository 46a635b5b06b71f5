// extern "C" entry points of libpa_kernels.so (declared in include/pa_kernels.h).
// Validation, status mapping and dispatch only; the kernels live in the other
// translation units.
#include <cmath>
#include <cstdio>
#include "attn_common.cuh"
#include "host_launchers.h"

namespace {

// First error recorded by a bounded wait in any kernel on this device.
__device__ uint32_t g_pa_status = 0;

// Device address of g_pa_status on the current device, looked up once per
// device (atomically cached: host threads driving different GPUs may make
// their first calls at the same time).
uint32_t* status_word() {
  static std::atomic<uint32_t*> ptrs[pa::kMaxDevices];
  const int dev = pa::current_device();
  if (dev < 0) return nullptr;
  uint32_t* w = ptrs[dev].load(std::memory_order_acquire);
  if (!w) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_pa_status) != cudaSuccess) return nullptr;
    w = static_cast<uint32_t*>(p);
    ptrs[dev].store(w, std::memory_order_release);
  }
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Validates an attention descriptor; fills `sh`.
int check_attn(const pa_attn_desc* d, pa::AttnShape* sh) {
  if (!d) return PA_ERR_NULL;
  if (d->batch <= 0 || d->seq_len <= 0 || d->num_heads <= 0 || d->head_dim <= 0)
    return PA_ERR_SHAPE;
  if (d->dtype != PA_BF16 && d->dtype != PA_F32) return PA_ERR_DTYPE;
  if (d->dtype == PA_BF16 && d->head_dim != 64 && d->head_dim != 128) return PA_ERR_UNSUPPORTED;
  if (d->dtype == PA_F32 && d->head_dim != 32 && d->head_dim != 64) return PA_ERR_UNSUPPORTED;
  const long long Lp = (static_cast<long long>(d->seq_len) + 127) / 128 * 128;
  if (static_cast<long long>(d->batch) * d->num_heads * Lp > 0x7fffffffLL) return PA_ERR_SHAPE;
  sh->B = d->batch;
  sh->L = d->seq_len;
  sh->H = d->num_heads;
  sh->D = d->head_dim;
  sh->scale = d->softmax_scale > 0.f ? d->softmax_scale
                                     : 1.0f / std::sqrt(static_cast<float>(d->head_dim));
  return PA_OK;
}

}  // namespace

extern "C" {

int pa_set_f32_math(int mode) {
  if (mode != PA_F32_MATH_SPLIT3 && mode != PA_F32_MATH_BF16) return PA_ERR_UNSUPPORTED;
  pa::set_f32_math(mode);
  return PA_OK;
}
int pa_get_f32_math(void) { return pa::f32_math(); }

int pa_abi_version(void) { return PA_ABI_VERSION; }

const char* pa_status_string(int s) {
  switch (s) {
    case PA_OK: return "ok";
    case PA_ERR_SHAPE: return "invalid shape";
    case PA_ERR_DTYPE: return "unsupported dtype";
    case PA_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case PA_ERR_UNSUPPORTED: return "unsupported configuration (head dimension)";
    case PA_ERR_LAUNCH: return "kernel launch failed";
    case PA_ERR_TIMEOUT: return "a kernel wait timed out";
    case PA_ERR_WORKSPACE: return "workspace missing or too small";
    case PA_ERR_NULL: return "required pointer is NULL";
    case PA_ERR_DEVICE: return "CUDA device error";
    default: return "unknown status";
  }
}

int pa_device_status(pa_stream_t stream, int clear) {
  uint32_t* w = status_word();
  if (!w) return PA_ERR_DEVICE;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return PA_ERR_DEVICE;
  uint32_t v = 0;
  if (cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return PA_ERR_DEVICE;
  if (clear && v != 0 && cudaMemset(w, 0, sizeof(v)) != cudaSuccess) return PA_ERR_DEVICE;
  return v == 0 ? PA_OK : PA_ERR_TIMEOUT;
}

}  // extern "C"

namespace {
// One thread waits on an mbarrier of arrival count 1 with the kernels' bounded
// wait. Without the arrival nothing completes the phase: the wait gives up
// after limit_ns, records the timeout in the status word and the kernel ends.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int arrive, uint32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = pa::smem_u32(&bar);
  pa::mbar_init(b, 1);
  pa::fence_mbar_init();
  if (arrive) pa::mbar_arrive(b);
  pa::mbar_wait_for(b, 0, status, limit_ns);
}
}  // namespace

extern "C" {

int pa_wait_selftest(uint64_t limit_ns, int arrive, pa_stream_t stream) {
  constexpr uint64_t kMaxLimitNs = 5000000000ull;
  if (limit_ns == 0 || limit_ns > kMaxLimitNs) return PA_ERR_SHAPE;
  uint32_t* w = status_word();
  if (!w) return PA_ERR_DEVICE;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, arrive, w);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

size_t pa_attn_fwd_workspace_size(const pa_attn_desc* desc) {
  pa::AttnShape sh;
  if (check_attn(desc, &sh) != PA_OK) return 0;
  return desc->dtype == PA_BF16 ? 0 : pa::attn_fwd_workspace_bytes_f32(sh);
}

int pa_attn_fwd(const pa_attn_desc* desc, const void* q, const void* k, const void* v, void* o,
                float* lse, void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  pa::AttnShape sh;
  int st = check_attn(desc, &sh);
  if (st != PA_OK) return st;
  if (!q || !k || !v || !o || !lse) return PA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return PA_ERR_ALIGN;
  if (desc->dtype == PA_F32) {
    const size_t need = pa_attn_fwd_workspace_size(desc);
    if (!workspace || workspace_bytes < need) return PA_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PA_ERR_ALIGN;
  }
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == PA_BF16) return pa::launch_attn_fwd_bf16(sh, q, k, v, o, lse, status, s);
  return pa::launch_attn_fwd_f32(sh, q, k, v, o, lse, workspace, status, s);
}

size_t pa_attn_bwd_workspace_size(const pa_attn_desc* desc) {
  pa::AttnShape sh;
  if (check_attn(desc, &sh) != PA_OK) return 0;
  return desc->dtype == PA_BF16 ? pa::attn_bwd_workspace_bytes(sh)
                                : pa::attn_bwd_workspace_bytes_f32(sh);
}

int pa_attn_bwd(const pa_attn_desc* desc, const void* q, const void* k, const void* v,
                const void* o, const void* dO, const float* lse, void* dq, void* dk, void* dv,
                int accumulate, void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  pa::AttnShape sh;
  int st = check_attn(desc, &sh);
  if (st != PA_OK) return st;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv) return PA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dO) ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return PA_ERR_ALIGN;
  const size_t need = pa_attn_bwd_workspace_size(desc);
  if (!workspace || workspace_bytes < need) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PA_ERR_ALIGN;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == PA_BF16)
    return pa::launch_attn_bwd_bf16(sh, q, k, v, o, dO, lse, dq, dk, dv, accumulate, workspace,
                                    status, s);
  return pa::launch_attn_bwd_f32(sh, q, k, v, o, dO, lse, dq, dk, dv, accumulate, workspace,
                                 status, s);
}

int pa_attn_bwd_kept(const pa_attn_desc* desc, const void* q, const void* k, const void* v,
                     const void* o, const void* dO, const float* lse, void* dq, void* dk, void* dv,
                     int accumulate, const void* fwd_workspace, size_t fwd_workspace_bytes,
                     int fwd_mode, void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  if (!desc) return PA_ERR_NULL;
  if (desc->dtype != PA_F32 || !fwd_workspace)
    return pa_attn_bwd(desc, q, k, v, o, dO, lse, dq, dk, dv, accumulate, workspace,
                       workspace_bytes, stream);
  pa::AttnShape sh;
  int st = check_attn(desc, &sh);
  if (st != PA_OK) return st;
  if (fwd_mode != PA_F32_MATH_SPLIT3 && fwd_mode != PA_F32_MATH_BF16) return PA_ERR_SHAPE;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv) return PA_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dO) ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return PA_ERR_ALIGN;
  const size_t need = pa_attn_bwd_workspace_size(desc);
  if (!workspace || workspace_bytes < need) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return PA_ERR_ALIGN;
  if (fwd_workspace_bytes < pa_attn_fwd_workspace_size(desc)) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(fwd_workspace) & 255u) != 0) return PA_ERR_ALIGN;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  // a bf16-math forward at head dim 64 kept only the hi planes
  const bool kept_lo = !(desc->head_dim == 64 && fwd_mode == PA_F32_MATH_BF16);
  return pa::launch_attn_bwd_f32(sh, q, k, v, o, dO, lse, dq, dk, dv, accumulate, workspace,
                                 status, static_cast<cudaStream_t>(stream), fwd_workspace, kept_lo);
}

int pa_attn_delta(const pa_attn_desc* desc, const void* dO, const void* o, float* delta,
                  pa_stream_t stream) {
  pa::AttnShape sh;
  int st = check_attn(desc, &sh);
  if (st != PA_OK) return st;
  if (!dO || !o || !delta) return PA_ERR_NULL;
  if (!aligned16(dO) || !aligned16(o)) return PA_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (desc->dtype == PA_BF16) return pa::launch_attn_delta_bf16(sh, dO, o, delta, s);
  return pa::launch_attn_delta_f32(sh, dO, o, delta, s);
}

}  // extern "C"

// ------------------------------------------------------------------ layer norm, matmul, elementwise
namespace {
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" {

int pa_layer_norm_fwd(const float* x, const float* gamma, const float* beta, float* y,
                      float* mean, float* rstd, uint32_t M, uint32_t N, float epsilon,
                      pa_stream_t stream) {
  if (!x || !gamma || !beta || !y || !mean || !rstd) return PA_ERR_NULL;
  if (M == 0 || N == 0) return PA_ERR_SHAPE;
  if (N % 4 != 0) return PA_ERR_UNSUPPORTED;
  if (!al16(x) || !al16(gamma) || !al16(beta) || !al16(y)) return PA_ERR_ALIGN;
  return pa::launch_layer_norm_fwd(x, nullptr, nullptr, gamma, beta, y, mean, rstd, M, N, epsilon,
                                   static_cast<cudaStream_t>(stream));
}

int pa_add_layer_norm_fwd(const float* x, const float* r, float* sum, const float* gamma,
                          const float* beta, float* y, float* mean, float* rstd, uint32_t M,
                          uint32_t N, float epsilon, pa_stream_t stream) {
  if (!x || !r || !sum || !gamma || !beta || !y || !mean || !rstd) return PA_ERR_NULL;
  if (M == 0 || N == 0) return PA_ERR_SHAPE;
  if (N % 4 != 0) return PA_ERR_UNSUPPORTED;
  if (!al16(x) || !al16(r) || !al16(sum) || !al16(gamma) || !al16(beta) || !al16(y))
    return PA_ERR_ALIGN;
  if (sum == x || sum == r) return PA_ERR_SHAPE;
  return pa::launch_layer_norm_fwd(x, r, sum, gamma, beta, y, mean, rstd, M, N, epsilon,
                                   static_cast<cudaStream_t>(stream));
}

int pa_layer_norm_fwd_planes(const float* x, const float* r, float* sum, const float* gamma,
                             const float* beta, float* y, float* mean, float* rstd, uint32_t M,
                             uint32_t N, float epsilon, void* y_planes, size_t y_planes_bytes,
                             pa_stream_t stream) {
  if (!x || !gamma || !beta || !y || !mean || !rstd || !y_planes) return PA_ERR_NULL;
  if (!r != !sum) return PA_ERR_NULL;
  if (M == 0 || N == 0 || M > 0x7fffffffu || N > 0x7fffffffu) return PA_ERR_SHAPE;
  if (N % 4 != 0) return PA_ERR_UNSUPPORTED;
  if (!al16(x) || !al16(gamma) || !al16(beta) || !al16(y) || (r && (!al16(r) || !al16(sum))) ||
      (reinterpret_cast<uintptr_t>(y_planes) & 255u) != 0)
    return PA_ERR_ALIGN;
  if (r && (sum == x || sum == r)) return PA_ERR_SHAPE;
  const int mode = pa::f32_math();
  if (y_planes_bytes < pa::linear_kept_bytes(static_cast<int>(M), static_cast<int>(N), mode))
    return PA_ERR_SHAPE;
  uint8_t* hi = static_cast<uint8_t*>(y_planes);
  uint8_t* lo = mode == PA_F32_MATH_BF16
                    ? nullptr
                    : hi + pa::linear_kept_bytes(static_cast<int>(M), static_cast<int>(N),
                                                 PA_F32_MATH_BF16);  // one plane
  return pa::launch_layer_norm_fwd(x, r, sum, gamma, beta, y, mean, rstd, M, N, epsilon,
                                   static_cast<cudaStream_t>(stream), hi, lo, (N + 7) / 8 * 8);
}

size_t pa_layer_norm_bwd_workspace_size(uint32_t M, uint32_t N) {
  return pa::layer_norm_bwd_workspace_bytes(M, N);
}

static int layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                          const float* gamma, float* dx, float* dgamma, float* dbeta, uint32_t M,
                          uint32_t N, void* workspace, size_t workspace_bytes, int accumulate,
                          pa_stream_t stream) {
  if (!dy || !x || !mean || !rstd || !gamma) return PA_ERR_NULL;
  if (M == 0 || N == 0) return PA_ERR_SHAPE;
  if (N % 4 != 0) return PA_ERR_UNSUPPORTED;
  if (!al16(dy) || !al16(x) || !al16(gamma) || (dx && !al16(dx))) return PA_ERR_ALIGN;
  if ((dgamma || dbeta) &&
      (!workspace || workspace_bytes < pa::layer_norm_bwd_workspace_bytes(M, N)))
    return PA_ERR_WORKSPACE;
  return pa::launch_layer_norm_bwd(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, M, N,
                                   static_cast<float*>(workspace), accumulate,
                                   static_cast<cudaStream_t>(stream));
}

int pa_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd,
                      const float* gamma, float* dx, float* dgamma, float* dbeta, uint32_t M,
                      uint32_t N, void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  return layer_norm_bwd(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, M, N, workspace,
                        workspace_bytes, 0, stream);
}

int pa_layer_norm_bwd_accumulate(const float* dy, const float* x, const float* mean,
                                 const float* rstd, const float* gamma, float* dx, float* dgamma,
                                 float* dbeta, uint32_t M, uint32_t N, void* workspace,
                                 size_t workspace_bytes, pa_stream_t stream) {
  return layer_norm_bwd(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, M, N, workspace,
                        workspace_bytes, 1, stream);
}

int pa_add_layer_norm_bwd(const float* dy, const float* dsum, const float* sum,
                          const float* mean, const float* rstd, const float* gamma, float* dx,
                          float* dr, float* dgamma, float* dbeta, uint32_t M, uint32_t N,
                          int flags, void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  if (!dy || !sum || !mean || !rstd || !gamma) return PA_ERR_NULL;
  if (M == 0 || N == 0) return PA_ERR_SHAPE;
  if (N % 4 != 0) return PA_ERR_UNSUPPORTED;
  if ((flags & ~(PA_ADD_LN_ACC_DX | PA_ADD_LN_ACC_DR)) != 0) return PA_ERR_SHAPE;
  if (!al16(dy) || !al16(sum) || !al16(gamma) || (dsum && !al16(dsum)) || (dx && !al16(dx)) ||
      (dr && !al16(dr)))
    return PA_ERR_ALIGN;
  if ((dgamma || dbeta) &&
      (!workspace || workspace_bytes < pa::layer_norm_bwd_workspace_bytes(M, N)))
    return PA_ERR_WORKSPACE;
  return pa::launch_add_layer_norm_bwd(dy, dsum, sum, mean, rstd, gamma, dx,
                                       (flags & PA_ADD_LN_ACC_DX) ? 1 : 0, dr,
                                       (flags & PA_ADD_LN_ACC_DR) ? 1 : 0, dgamma, dbeta, M, N,
                                       static_cast<float*>(workspace),
                                       static_cast<cudaStream_t>(stream));
}

size_t pa_matmul_workspace_size(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return pa::gemm_workspace_bytes(M, N, K);
}

static int gemm_call(int mode, const float* A, const float* B, float* C, int M, int N, int K,
                     void* ws, size_t ws_bytes, pa_stream_t stream) {
  if (!A || !B || !C) return PA_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return PA_ERR_SHAPE;
  if (!ws || ws_bytes < pa::gemm_workspace_bytes(M, N, K)) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return PA_ERR_ALIGN;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_gemm_f32(mode, A, B, C, M, N, K, ws, status, static_cast<cudaStream_t>(stream));
}

int pa_matmul(const float* A, const float* B, float* C, int M, int N, int K, void* workspace,
              size_t workspace_bytes, pa_stream_t stream) {
  return gemm_call(0, A, B, C, M, N, K, workspace, workspace_bytes, stream);
}

int pa_matmul_grad_x(const float* dY, const float* W, float* dX, int M, int N, int K,
                     void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  return gemm_call(1, dY, W, dX, M, N, K, workspace, workspace_bytes, stream);
}

int pa_matmul_grad_w(const float* X, const float* dY, float* dW, int M, int N, int K,
                     void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  return gemm_call(2, X, dY, dW, M, N, K, workspace, workspace_bytes, stream);
}

size_t pa_linear_workspace_size(int M, int in_features, int out_features) {
  if (M <= 0 || in_features <= 0 || out_features <= 0) return 0;
  return pa::linear_workspace_bytes(M, in_features, out_features);
}

static int linear_check(int M, int in, int out, int n, void* ws, size_t ws_bytes) {
  if (M <= 0 || in <= 0 || out <= 0 || n < 1 || n > 3 || out % n != 0) return PA_ERR_SHAPE;
  if (!ws || ws_bytes < pa::linear_workspace_bytes(M, in, out)) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return PA_ERR_ALIGN;
  return PA_OK;
}

int pa_linear_fwd(const float* X, const float* W, const float* bias, float* const* outs, int n_outs,
                  int M, int in_features, int out_features, void* workspace, size_t workspace_bytes,
                  pa_stream_t stream) {
  if (!X || !W || !outs) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, n_outs, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i]) return PA_ERR_NULL;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_linear_fwd(X, W, bias, outs, n_outs, M, in_features, out_features, 0,
                               workspace, status, static_cast<cudaStream_t>(stream));
}

int pa_linear_relu_fwd(const float* X, const float* W, const float* bias, float* Y, int M,
                       int in_features, int out_features, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream) {
  if (!X || !W || !Y) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, 1, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  float* outs[1] = {Y};
  return pa::launch_linear_fwd(X, W, bias, outs, 1, M, in_features, out_features, 1, workspace,
                               status, static_cast<cudaStream_t>(stream));
}

int pa_linear_bwd(const float* X, const float* W, const float* const* dy_parts, int n_parts,
                  float* dX, float* dW, float* dbias, int M, int in_features, int out_features,
                  void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  if (!X || !W || !dy_parts) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, n_parts, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  for (int i = 0; i < n_parts; ++i)
    if (!dy_parts[i]) return PA_ERR_NULL;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_linear_bwd(X, W, dy_parts, n_parts, nullptr, dX, dW, dbias, M, in_features,
                               out_features, workspace, status, static_cast<cudaStream_t>(stream));
}

size_t pa_linear_kept_size(int M, int in_features) {
  if (M <= 0 || in_features <= 0) return 0;
  return pa::linear_kept_bytes(M, in_features, pa::f32_math());
}

int pa_linear_fwd_keep(const float* X, const float* W, const float* bias, float* const* outs,
                       int n_outs, int relu, int M, int in_features, int out_features, void* kept,
                       size_t kept_bytes, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream) {
  if (!X || !W || !outs || !kept) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, n_outs, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  if (relu && n_outs != 1) return PA_ERR_SHAPE;
  if (kept_bytes < pa::linear_kept_bytes(M, in_features, pa::f32_math())) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(kept) & 255u) != 0) return PA_ERR_ALIGN;
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i]) return PA_ERR_NULL;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_linear_fwd(X, W, bias, outs, n_outs, M, in_features, out_features, relu ? 1 : 0,
                               workspace, status, static_cast<cudaStream_t>(stream), kept);
}

int pa_linear_fwd_planes(const float* X, const float* W, const float* bias, float* const* outs,
                         int n_outs, int relu, int M, int in_features, int out_features, void* kept,
                         size_t kept_bytes, int kept_mode, int flags, void* y_planes,
                         size_t y_planes_bytes, void* workspace, size_t workspace_bytes,
                         pa_stream_t stream) {
  if (!X || !W || !outs || !kept) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, n_outs, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  if (relu && n_outs != 1) return PA_ERR_SHAPE;
  if ((flags & ~PA_LINEAR_KEPT_VALID) != 0) return PA_ERR_SHAPE;
  const int mode = pa::f32_math();
  if (kept_bytes < pa::linear_kept_bytes(M, in_features, mode)) return PA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(kept) & 255u) != 0) return PA_ERR_ALIGN;
  if (y_planes) {
    if (n_outs != 1) return PA_ERR_SHAPE;
    if (y_planes_bytes < pa::linear_kept_bytes(M, out_features, mode)) return PA_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(y_planes) & 255u) != 0) return PA_ERR_ALIGN;
  }
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i]) return PA_ERR_NULL;
  // planes made under bf16 math have no lo plane: a split3 call converts X again
  const bool valid = (flags & PA_LINEAR_KEPT_VALID) &&
                     (mode == PA_F32_MATH_BF16 || kept_mode == PA_F32_MATH_SPLIT3);
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_linear_fwd(X, W, bias, outs, n_outs, M, in_features, out_features, relu ? 1 : 0,
                               workspace, status, static_cast<cudaStream_t>(stream), kept,
                               valid ? 1 : 0, y_planes);
}

int pa_linear_bwd_kept(const float* X, const float* W, const void* kept, size_t kept_bytes,
                       int kept_mode, const float* Y, const float* const* dy_parts, int n_parts,
                       float* dX, float* dW, float* dbias, int M, int in_features,
                       int out_features, int flags, void* workspace, size_t workspace_bytes,
                       pa_stream_t stream) {
  if (!X || !W || !dy_parts) return PA_ERR_NULL;
  if ((flags & ~PA_LINEAR_DX_OVERWRITE) != 0) return PA_ERR_SHAPE;
  const int st = linear_check(M, in_features, out_features, n_parts, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  if (Y && n_parts != 1) return PA_ERR_SHAPE;
  for (int i = 0; i < n_parts; ++i)
    if (!dy_parts[i]) return PA_ERR_NULL;
  const int mode = pa::f32_math();
  // a split3 forward kept hi and lo (enough for either mode), a bf16 one only hi
  const bool usable = kept && (reinterpret_cast<uintptr_t>(kept) & 255u) == 0 &&
                      (mode == PA_F32_MATH_BF16 || kept_mode == PA_F32_MATH_SPLIT3) &&
                      kept_bytes >= pa::linear_kept_bytes(M, in_features, mode);
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  return pa::launch_linear_bwd(X, W, dy_parts, n_parts, Y, dX, dW, dbias, M, in_features,
                               out_features, workspace, status, static_cast<cudaStream_t>(stream),
                               usable ? kept : nullptr,
                               (flags & PA_LINEAR_DX_OVERWRITE) ? 0 : 1);
}

int pa_linear_relu_bwd(const float* X, const float* W, const float* Y, const float* dY, float* dX,
                       float* dW, float* dbias, int M, int in_features, int out_features,
                       void* workspace, size_t workspace_bytes, pa_stream_t stream) {
  if (!X || !W || !Y || !dY) return PA_ERR_NULL;
  const int st = linear_check(M, in_features, out_features, 1, workspace, workspace_bytes);
  if (st != PA_OK) return st;
  uint32_t* status = status_word();
  if (!status) return PA_ERR_DEVICE;
  const float* parts[1] = {dY};
  return pa::launch_linear_bwd(X, W, parts, 1, Y, dX, dW, dbias, M, in_features, out_features,
                               workspace, status, static_cast<cudaStream_t>(stream));
}

int pa_bias_add(const float* A, const float* bias, float* out, int M, int N, pa_stream_t stream) {
  if (!A || !bias || !out) return PA_ERR_NULL;
  if (M <= 0 || N <= 0) return PA_ERR_SHAPE;
  return pa::launch_bias_add(A, bias, out, M, N, static_cast<cudaStream_t>(stream));
}

int pa_add(const float* a, const float* b, float* out, size_t n, pa_stream_t stream) {
  if (!a || !b || !out) return PA_ERR_NULL;
  if (n == 0) return PA_OK;
  return pa::launch_add(a, b, out, n, static_cast<cudaStream_t>(stream));
}

int pa_grad_accumulate(const float* src, float* dst, size_t n, pa_stream_t stream) {
  if (!src || !dst) return PA_ERR_NULL;
  if (n == 0) return PA_OK;
  return pa::launch_add(src, dst, dst, n, static_cast<cudaStream_t>(stream));
}

int pa_bias_grad(const float* dY, float* db, int M, int N, pa_stream_t stream) {
  if (!dY || !db) return PA_ERR_NULL;
  if (M <= 0 || N <= 0) return PA_ERR_SHAPE;
  return pa::launch_bias_grad(dY, db, M, N, static_cast<cudaStream_t>(stream));
}

size_t pa_bias_grad_workspace_size(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return pa::bias_grad_workspace_bytes(static_cast<uint32_t>(M), static_cast<uint32_t>(N));
}

int pa_bias_grad_ws(const float* dY, float* db, int M, int N, void* workspace,
                    size_t workspace_bytes, pa_stream_t stream) {
  if (!dY || !db) return PA_ERR_NULL;
  if (M <= 0 || N <= 0) return PA_ERR_SHAPE;
  if (!workspace || workspace_bytes < pa::bias_grad_workspace_bytes(M, N)) return PA_ERR_WORKSPACE;
  if (!al16(workspace)) return PA_ERR_ALIGN;
  return pa::launch_bias_grad_masked(dY, nullptr, db, M, N, static_cast<float*>(workspace),
                                     static_cast<cudaStream_t>(stream));
}

int pa_split_last_dim(const float* in, float* const* outs, uint32_t parts, uint32_t rows,
                      uint32_t width, pa_stream_t stream) {
  if (!in || !outs) return PA_ERR_NULL;
  if (parts == 0 || parts > 8 || rows == 0 || width == 0) return PA_ERR_SHAPE;
  for (uint32_t i = 0; i < parts; ++i)
    if (!outs[i]) return PA_ERR_NULL;
  return pa::launch_split_last_dim(in, outs, parts, rows, width,
                                   static_cast<cudaStream_t>(stream));
}

int pa_concat_last_dim_grad(const float* const* part_grads, float* grad_in, uint32_t parts,
                            uint32_t rows, uint32_t width, pa_stream_t stream) {
  if (!part_grads || !grad_in) return PA_ERR_NULL;
  if (parts == 0 || parts > 8 || rows == 0 || width == 0) return PA_ERR_SHAPE;
  return pa::launch_concat_last_dim_grad(part_grads, grad_in, parts, rows, width,
                                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------------ training utilities
extern "C" {

int pa_relu_fwd(const float* x, float* y, size_t n, pa_stream_t stream) {
  if (!x || !y) return PA_ERR_NULL;
  return n ? pa::launch_relu_fwd(x, y, n, static_cast<cudaStream_t>(stream)) : PA_OK;
}
int pa_relu_bwd(const float* dy, const float* x, float* dx, size_t n, pa_stream_t stream) {
  if (!dy || !x || !dx) return PA_ERR_NULL;
  return n ? pa::launch_relu_bwd(dy, x, dx, n, static_cast<cudaStream_t>(stream)) : PA_OK;
}
int pa_mse_fwd(const float* pred, const float* target, float* loss, size_t n, pa_stream_t stream) {
  if (!pred || !target || !loss) return PA_ERR_NULL;
  if (n == 0) return PA_ERR_SHAPE;
  return pa::launch_mse_fwd(pred, target, loss, n, nullptr, static_cast<cudaStream_t>(stream));
}

size_t pa_mse_fwd_workspace_size(size_t n) { return n ? pa::mse_workspace_bytes(n) : 0; }

int pa_mse_fwd_ws(const float* pred, const float* target, float* loss, size_t n, void* workspace,
                  size_t workspace_bytes, pa_stream_t stream) {
  if (!pred || !target || !loss) return PA_ERR_NULL;
  if (n == 0) return PA_ERR_SHAPE;
  if (!workspace || workspace_bytes < pa::mse_workspace_bytes(n)) return PA_ERR_WORKSPACE;
  if (!al16(workspace)) return PA_ERR_ALIGN;
  return pa::launch_mse_fwd(pred, target, loss, n, static_cast<float*>(workspace),
                            static_cast<cudaStream_t>(stream));
}
int pa_mse_bwd(const float* pred, const float* target, const float* dloss, float* dpred, size_t n,
               pa_stream_t stream) {
  if (!pred || !target || !dloss || !dpred) return PA_ERR_NULL;
  if (n == 0) return PA_ERR_SHAPE;
  return pa::launch_mse_bwd(pred, target, dloss, dpred, n, static_cast<cudaStream_t>(stream));
}
int pa_adam_step(float* param, const float* grad, float* m, float* v, size_t n, float lr,
                 float beta1, float beta2, float eps, float bias_corr1, float bias_corr2,
                 pa_stream_t stream) {
  if (!param || !grad || !m || !v) return PA_ERR_NULL;
  if (bias_corr1 <= 0.f || bias_corr2 <= 0.f) return PA_ERR_SHAPE;
  return n ? pa::launch_adam(param, grad, m, v, n, lr, beta1, beta2, eps, bias_corr1, bias_corr2,
                             static_cast<cudaStream_t>(stream))
           : PA_OK;
}
int pa_adam_step_multi(float* const* params, const float* const* grads, float* const* m,
                       float* const* v, const size_t* sizes, int count, float lr, float beta1,
                       float beta2, float eps, float bias_corr1, float bias_corr2,
                       pa_stream_t stream) {
  if (count < 0) return PA_ERR_SHAPE;
  if (count == 0) return PA_OK;
  if (!params || !grads || !m || !v || !sizes) return PA_ERR_NULL;
  for (int i = 0; i < count; ++i)
    if (sizes[i] && (!params[i] || !grads[i] || !m[i] || !v[i])) return PA_ERR_NULL;
  if (bias_corr1 <= 0.f || bias_corr2 <= 0.f) return PA_ERR_SHAPE;
  return pa::launch_adam_multi(params, grads, m, v, sizes, count, lr, beta1, beta2, eps, bias_corr1,
                               bias_corr2, static_cast<cudaStream_t>(stream));
}
int pa_fill_normal(float* x, size_t n, float std_dev, uint64_t seed, pa_stream_t stream) {
  if (!x) return PA_ERR_NULL;
  return n ? pa::launch_fill_normal(x, n, std_dev, seed, static_cast<cudaStream_t>(stream)) : PA_OK;
}
int pa_fill(float* x, size_t n, float value, pa_stream_t stream) {
  if (!x) return PA_ERR_NULL;
  return n ? pa::launch_fill(x, n, value, static_cast<cudaStream_t>(stream)) : PA_OK;
}

}  // extern "C"
