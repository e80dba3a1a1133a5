// Optional per-kernel timing with CUDA events (ai_attn_profile_enable /
// ai_attn_profile_read).  When enabled, every launch of this library is
// bracketed by two events recorded on the launch's own stream; reading
// synchronizes them and returns the summed elapsed time and the launch count
// per kernel kind.  Nothing is skipped or reordered; when disabled (the
// default) a launch costs one relaxed atomic load.

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "../../include/ai_attn.h"
#include "ai_kernels.h"

namespace ai {
namespace {

struct Pair {
  int kind;
  cudaEvent_t start, stop;
};

constexpr size_t kMaxPairs = 4096;
std::atomic<bool> g_on{false};
std::mutex g_mu;
std::vector<Pair> g_pool;  // events, reused across reads
size_t g_used = 0;

}  // namespace

int prof_begin(int kind, cudaStream_t st) {
  if (!g_on.load(std::memory_order_relaxed)) return -1;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_used >= kMaxPairs) return -1;
  if (g_used == g_pool.size()) {
    Pair p{0, nullptr, nullptr};
    if (cudaEventCreate(&p.start) != cudaSuccess || cudaEventCreate(&p.stop) != cudaSuccess) return -1;
    g_pool.push_back(p);
  }
  Pair& p = g_pool[g_used];
  p.kind = kind;
  if (cudaEventRecord(p.start, st) != cudaSuccess) return -1;
  return (int)g_used++;
}

void prof_end(int slot, cudaStream_t st) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_mu);
  if ((size_t)slot < g_used) cudaEventRecord(g_pool[slot].stop, st);
}

}  // namespace ai

extern "C" {

int ai_attn_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(ai::g_mu);
  ai::g_used = 0;
  ai::g_on.store(on != 0);
  return AI_OK;
}

int ai_attn_profile_read(float* ms_by_kind, int32_t* launches_by_kind) {
  if (!ms_by_kind || !launches_by_kind) return AI_ERR_NULL;
  std::lock_guard<std::mutex> lock(ai::g_mu);
  for (int k = 0; k < AI_PROF_KINDS; ++k) {
    ms_by_kind[k] = 0.f;
    launches_by_kind[k] = 0;
  }
  int rc = AI_OK;
  for (size_t i = 0; i < ai::g_used; ++i) {
    const ai::Pair& p = ai::g_pool[i];
    float ms = 0.f;
    if (cudaEventSynchronize(p.stop) != cudaSuccess || cudaEventElapsedTime(&ms, p.start, p.stop) != cudaSuccess) {
      rc = AI_ERR_LAUNCH;
      continue;
    }
    if (p.kind >= 0 && p.kind < AI_PROF_KINDS) {
      ms_by_kind[p.kind] += ms;
      launches_by_kind[p.kind] += 1;
    }
  }
  ai::g_used = 0;
  return rc;
}

}  // extern "C"
