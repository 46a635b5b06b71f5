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
// with PA_ERR_WORKSPACE. The bf16 head-dim-64 backward needs 296 bytes per
// (batch*head, padded query) row - LSE, Delta, a 64-float dQ accumulator row
// and its share of the 4 KB key-extension tile per 128 rows - so about
// 113 000 rows fit: B=1, H=16, L=4096 does, B=8, H=16, L=4096 does not. The
// fp32 path also keeps eight bf16 operand planes, about 1.3 KB per row in all,
// so only about 25 000 rows fit (B=1, H=4, L=4096, say). pa_attn_bwd_workspace_size
// gives the exact figure for a shape.
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
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>
#include "attn_common.cuh"

namespace {

constexpr size_t kMaxWorkspace = PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE;

static __device__ __align__(256) unsigned char g_attn_bwd_scratch[kMaxWorkspace];

// Device address of g_attn_bwd_scratch on the current device (set up once per
// device; atomically cached, since host threads driving different GPUs may
// make their first calls at the same time). In host code the symbol itself is
// only a stand-in, never a device address, so it must not be passed to a kernel.
void* scratch_address() {
  static std::atomic<void*> ptrs[pa::kMaxDevices];
  const int dev = pa::current_device();
  if (dev < 0) return nullptr;
  void* p = ptrs[dev].load(std::memory_order_acquire);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_attn_bwd_scratch) != cudaSuccess) return nullptr;
    ptrs[dev].store(p, std::memory_order_release);
  }
  return p;
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
