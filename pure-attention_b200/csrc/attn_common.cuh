// Shared pieces of the attention kernels: problem shape, constants, TMA maps.
#pragma once
#include <atomic>
#include <cuda_runtime.h>
#include "pa_kernels.h"
#include "ptx.cuh"
#include "tma_host.h"

namespace pa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnShape {
  int B, L, H, D;
  float scale;  // softmax scale applied to q.k
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + (((a + 1023u) & ~1023u) - a);
}

// 4-D TMA map over a [B, L, H, D] 16-bit tensor: dims (D, H, L, B), box of
// 64 columns (128 bytes, one swizzle row) x 1 head x `rows` rows x 1 batch.
inline bool make_qkv_map(CUtensorMap* m, const void* base, const AttnShape& sh, uint32_t rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(sh.D), static_cast<uint64_t>(sh.H),
                            static_cast<uint64_t>(sh.L), static_cast<uint64_t>(sh.B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(sh.D) * 2,
                               static_cast<uint64_t>(sh.H) * sh.D * 2,
                               static_cast<uint64_t>(sh.L) * sh.H * sh.D * 2};
  const uint32_t box[4] = {64, 1, rows, 1};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---------------------------------------------------------------- per-device host caches
// The C ABI may be called from one host thread per GPU at the same time, so
// every value cached per device is an atomic: concurrent first calls compute
// the same value and store it without a data race.
constexpr int kMaxDevices = 64;

// The calling thread's current device, or -1 (no device, or beyond the caches).
inline int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

// cache[dev], computed by `compute` on first use; a value <= 0 is not kept.
template <typename F>
inline int cached_per_device(std::atomic<int> (&cache)[kMaxDevices], int dev, F compute) {
  int v = cache[dev].load(std::memory_order_acquire);
  if (v <= 0) {
    v = compute();
    if (v > 0) cache[dev].store(v, std::memory_order_release);
  }
  return v;
}

// Streaming multiprocessors of the current device (148 if it cannot be read).
inline int device_sm_count() {
  static std::atomic<int> cache[kMaxDevices];
  const int dev = current_device();
  if (dev < 0) return 148;
  const int n = cached_per_device(cache, dev, [dev] {
    int sms = 0;
    return cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess ? sms : 0;
  });
  return n > 0 ? n : 148;
}

// Raise a kernel's dynamic shared memory limit on the current device, once per
// device. The bit is set only after cudaFuncSetAttribute succeeded; two
// threads may both set the attribute, which is harmless. Returns false when
// the attribute could not be set (the launch would fail).
template <typename K>
inline bool ensure_smem_attr(K kernel, int bytes, std::atomic<uint64_t>& done_mask) {
  const int dev = current_device();
  if (dev < 0) return false;
  const uint64_t bit = 1ull << dev;
  if (done_mask.load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();  // do not leave the error for the caller's launch check
    return false;
  }
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

}  // namespace pa
