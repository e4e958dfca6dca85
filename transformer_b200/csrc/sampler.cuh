// sampler.cuh — device sampler (generate.py:28-65 semantics).  Placeholder:
// the launcher reports "not supported" until the kernel lands.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b2d {
constexpr int kSamplerMaxVocab = 65536;

inline cudaError_t launch_sampler(const float*, int, int, const int32_t*, int, const int32_t*, const float*,
                                  double, double, double, int32_t*, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace b2d
