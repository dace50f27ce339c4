// Opt-in CUDA-event timing of the library's main kernels (instrumentation for the benchmark).
// When enabled, launchers bracket their dominant kernel with events recorded on the launch stream;
// atlb_timing_read() waits for those events and returns the summed device time per kernel name.
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace atlb {

namespace {
std::mutex g_mu;
bool g_enabled = false;
std::map<std::string, std::vector<std::pair<cudaEvent_t, cudaEvent_t>>> g_pending;
}  // namespace

cudaEvent_t timing_begin(cudaStream_t s) {
  if (!g_enabled) return nullptr;
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  cudaEventRecord(e, s);
  return e;
}

void timing_end(const char* name, cudaStream_t s, cudaEvent_t e0) {
  if (!e0) return;
  cudaEvent_t e1 = nullptr;
  if (cudaEventCreate(&e1) != cudaSuccess) return;
  cudaEventRecord(e1, s);
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending[name].emplace_back(e0, e1);
}

}  // namespace atlb

extern "C" {

int atlb_timing_enable(int on) {
  std::lock_guard<std::mutex> lk(atlb::g_mu);
  atlb::g_enabled = on != 0;
  return ATLB_OK;
}

int atlb_timing_read(const char* name, double* total_ms, int64_t* count, int reset) {
  std::lock_guard<std::mutex> lk(atlb::g_mu);
  double tot = 0.0;
  int64_t n = 0;
  auto it = atlb::g_pending.find(name ? name : "");
  if (it != atlb::g_pending.end()) {
    for (auto& pr : it->second) {
      if (cudaEventSynchronize(pr.second) != cudaSuccess) return atlb::launch_status("timing_read");
      float ms = 0.f;
      cudaEventElapsedTime(&ms, pr.first, pr.second);
      tot += ms;
      ++n;
    }
    if (reset) {
      for (auto& pr : it->second) {
        cudaEventDestroy(pr.first);
        cudaEventDestroy(pr.second);
      }
      it->second.clear();
    }
  }
  if (total_ms) *total_ms = tot;
  if (count) *count = n;
  return ATLB_OK;
}

}  // extern "C"
