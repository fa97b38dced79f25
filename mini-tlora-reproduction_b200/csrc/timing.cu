// Per-kernel device timing of the tensor-core launches (mlora_timing_*).
// Off by default; when on, each launch is bracketed by two CUDA events
// recorded on the launch stream, and mlora_timing_read folds the pending
// pairs into per-role totals.
#include <mutex>

#include "common.cuh"

namespace mlora {
namespace {

struct Pending {
  int kind;
  cudaEvent_t a, b;
};

std::mutex g_tmu;
std::atomic<bool> g_timing{false};
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_free;
double g_ms[kTimedKinds] = {0};
int64_t g_n[kTimedKinds] = {0};

cudaEvent_t get_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

int fold() {
  for (const Pending& p : g_pending) {
    if (cudaEventSynchronize(p.b) != cudaSuccess) return MLORA_ERR_CUDA;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, p.a, p.b) != cudaSuccess) return MLORA_ERR_CUDA;
    g_ms[p.kind] += ms;
    g_n[p.kind] += 1;
    g_free.push_back(p.a);
    g_free.push_back(p.b);
  }
  g_pending.clear();
  return MLORA_OK;
}

}  // namespace

bool timing_begin(cudaStream_t st, cudaEvent_t (&ev)[2]) {
  if (!g_timing.load(std::memory_order_relaxed)) return false;
  std::lock_guard<std::mutex> lk(g_tmu);
  ev[0] = get_event();
  ev[1] = get_event();
  if (!ev[0] || !ev[1]) return false;
  return cudaEventRecord(ev[0], st) == cudaSuccess;
}

void timing_end(int kind, cudaStream_t st, cudaEvent_t (&ev)[2]) {
  std::lock_guard<std::mutex> lk(g_tmu);
  if (cudaEventRecord(ev[1], st) == cudaSuccess && kind >= 0 && kind < kTimedKinds)
    g_pending.push_back({kind, ev[0], ev[1]});
}

}  // namespace mlora

using namespace mlora;

extern "C" int mlora_timing_enable(int32_t on) {
  g_timing.store(on != 0);
  return MLORA_OK;
}

extern "C" int mlora_timing_read(int32_t kind, double* total_ms, int64_t* launches) {
  if (kind < 0 || kind >= kTimedKinds || !total_ms || !launches) return MLORA_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_tmu);
  int s = fold();
  if (s != MLORA_OK) return s;
  *total_ms = g_ms[kind];
  *launches = g_n[kind];
  return MLORA_OK;
}

extern "C" int mlora_timing_reset(void) {
  std::lock_guard<std::mutex> lk(g_tmu);
  int s = fold();
  for (int k = 0; k < kTimedKinds; ++k) {
    g_ms[k] = 0;
    g_n[k] = 0;
  }
  return s;
}
