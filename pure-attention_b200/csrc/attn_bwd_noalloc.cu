// pa_attn_bwd_noalloc: the flash-attention backward for callers that cannot
// allocate device memory.
//
// Some callers have no way to obtain scratch memory: code running under an
// allocator that forbids new device allocations once a model is resident,
// plugins whose host framework owns all GPU memory and hands out only the
// tensors of an op, or C callers without a CUDA memory manager. For them this
// entry point carries its own scratch: a fixed array in the library's device
// memory, reserved on every GPU that loads the library until the process exits.
//
// The array holds PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE bytes (32 MiB). A shape
// whose backward workspace (pa_attn_bwd_workspace_size) is larger is rejected
// with PA_ERR_WORKSPACE. At head_dim 64 that is about 127 000 (batch*head,
// padded query) rows, e.g. B=1, H=16, L=4096 fits and B=8, H=16, L=4096 does not.
//
// All calls on a device share the one array, and it keeps whatever the last
// call left in it. The backward clears what must start at zero (the fp32 dQ
// accumulator) and overwrites the rest before reading it, so stale contents do
// no harm - but two calls whose kernels overlap on the GPU (different streams,
// or different host threads) race on the array and corrupt each other's dQ.
// Serialise them.
//
// The device address of the array is looked up (cudaGetSymbolAddress) on the
// first call made while a given device is current; make that first call before
// any stream capture on that device.
#include <cstdint>
#include <cuda_runtime.h>
#include "pa_kernels.h"

namespace {

constexpr size_t kMaxWorkspace = PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE;

static __device__ __align__(256) unsigned char g_attn_bwd_scratch[kMaxWorkspace];

// Device address of g_attn_bwd_scratch on the current device (set up once per
// device). In host code the symbol itself is only a stand-in, never a device
// address, so it must not be passed to a kernel.
void* scratch_address() {
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_bwd_scratch) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace

extern "C" int pa_attn_bwd_noalloc(const pa_attn_desc* desc, const void* q, const void* k,
                                   const void* v, const void* o, const void* dO, const float* lse,
                                   void* dq, void* dk, void* dv, int accumulate,
                                   pa_stream_t stream) {
  if (!desc) return PA_ERR_NULL;
  const size_t need = pa_attn_bwd_workspace_size(desc);
  if (need == 0) {
    // invalid descriptor: let the regular entry point report why
    return pa_attn_bwd(desc, q, k, v, o, dO, lse, dq, dk, dv, accumulate, nullptr, 0, stream);
  }
  if (need > kMaxWorkspace) return PA_ERR_WORKSPACE;
  void* scratch = scratch_address();
  if (!scratch) return PA_ERR_DEVICE;
  return pa_attn_bwd(desc, q, k, v, o, dO, lse, dq, dk, dv, accumulate, scratch, kMaxWorkspace,
                     stream);
}
