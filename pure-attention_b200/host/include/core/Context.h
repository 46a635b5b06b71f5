// Stream and seed context of the host layer (the reference's
// include/core/Context.h:6-16 holds the stream; the seed is an addition so
// weight initialisation is reproducible).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

struct CudaContext {
  inline static cudaStream_t current_stream = nullptr;  // nullptr = legacy default stream
  inline static uint64_t seed = 0x5eed5eedull;

  static cudaStream_t getStream() { return current_stream; }
  static void setStream(cudaStream_t s) { current_stream = s; }
  static void setSeed(uint64_t s) { seed = s; }
  static uint64_t nextSeed() { return seed++; }
};
