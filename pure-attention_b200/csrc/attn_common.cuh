// Shared pieces of the attention kernels: problem shape, constants, TMA maps.
#pragma once
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

// Raise a kernel's dynamic shared memory limit once per device.
template <typename K>
inline void ensure_smem_attr(K kernel, int bytes, uint64_t& done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done_mask & bit)) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done_mask |= bit;
  }
}

}  // namespace pa
