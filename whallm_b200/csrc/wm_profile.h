// Profiler state (host only).
#pragma once

#include <cuda_runtime.h>

#include <utility>
#include <vector>

#include "wm_kernels.h"

namespace wm {

struct Profiler {
  bool enabled = false;
  cudaEvent_t open[kProfSlots] = {};
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending[kProfSlots];
  double total_ms[kProfSlots] = {};
  long long launches[kProfSlots] = {};
  std::vector<cudaEvent_t> pool;

  cudaEvent_t take();
  void collect();
  void reset();
  ~Profiler();
};

const char* prof_name(int slot);

}  // namespace wm
