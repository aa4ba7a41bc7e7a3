// Per-kernel-group timing with CUDA events, enabled by wm_profile_enable.
// Each timed group records a start and an end event on the launching stream;
// wm_profile_read waits for them and accumulates the elapsed times.
#include <vector>

#include "wm_kernels.h"
#include "wm_profile.h"

namespace wm {

cudaEvent_t Profiler::take() {
  if (!pool.empty()) {
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void Profiler::collect() {
  for (int s = 0; s < kProfSlots; ++s) {
    for (auto& pr : pending[s]) {
      cudaEventSynchronize(pr.second);
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, pr.first, pr.second) == cudaSuccess) {
        total_ms[s] += ms;
        launches[s] += 1;
      }
      pool.push_back(pr.first);
      pool.push_back(pr.second);
    }
    pending[s].clear();
  }
}

void Profiler::reset() {
  collect();
  for (int s = 0; s < kProfSlots; ++s) {
    total_ms[s] = 0.0;
    launches[s] = 0;
  }
}

Profiler::~Profiler() {
  collect();
  for (cudaEvent_t e : pool) cudaEventDestroy(e);
}

void prof_begin(Profiler* p, int slot, cudaStream_t s) {
  if (p == nullptr || !p->enabled) return;
  cudaEvent_t e = p->take();
  cudaEventRecord(e, s);
  p->open[slot] = e;
}

void prof_end(Profiler* p, int slot, cudaStream_t s) {
  if (p == nullptr || !p->enabled || p->open[slot] == nullptr) return;
  cudaEvent_t e = p->take();
  cudaEventRecord(e, s);
  p->pending[slot].emplace_back(p->open[slot], e);
  p->open[slot] = nullptr;
}

const char* prof_name(int slot) {
  static const char* names[kProfSlots] = {"router_logits", "router_topk", "plan",     "act_f16",     "gather_rows",
                                          "gemv_gate_up",  "gemv_down",   "gemm_gate_up", "gemm_down", "combine",
                                          "decode_gate_up", "decode_down", "rmsnorm",
                                          "ep_send", "ep_wait_dispatch", "ep_return", "ep_wait_return",
                                          "route_plan_quant", "decode_fused"};
  return slot >= 0 && slot < kProfSlots ? names[slot] : "?";
}

}  // namespace wm
