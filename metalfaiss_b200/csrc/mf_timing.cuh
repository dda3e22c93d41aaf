// Per-kernel event timing hooks (see mf_timing.cu).
#pragma once

#include "mf_common.cuh"

namespace mf {
bool timing_enabled();
void* timing_begin(const char* name, cudaStream_t s);
void timing_end(void* h, cudaStream_t s);

struct ScopedTiming {
  void* h;
  cudaStream_t s;
  ScopedTiming(const char* name, cudaStream_t st) : h(timing_begin(name, st)), s(st) {}
  ~ScopedTiming() { timing_end(h, s); }
};
}  // namespace mf
