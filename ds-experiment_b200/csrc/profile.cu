// Per-kernel GPU timing (diagnostics).  While enabled, each launcher brackets
// its main kernel with CUDA events on the launch stream; ds_profile_read
// waits for the recorded events and sums their elapsed times per name.
// Disabled (the default), a scope costs one relaxed atomic load.
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "common.cuh"
#include "profile.h"

namespace dsb {
namespace {

struct Span {
  cudaEvent_t start, stop;
};

std::atomic<bool> g_enabled{false};
std::mutex g_mu;
std::set<std::string> g_only;  // families recorded while enabled; empty: all
std::map<std::string, std::vector<Span>> g_spans;
std::vector<cudaEvent_t> g_free;

cudaEvent_t take_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

ProfileScope::ProfileScope(const char* name, cudaStream_t s) : name_(name), stream_(s) {
  if (!g_enabled.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_only.empty() && !g_only.count(name)) return;
  start_ = take_event();
  if (start_ && cudaEventRecord(start_, s) != cudaSuccess) {
    g_free.push_back(start_);
    start_ = nullptr;
  }
}

ProfileScope::~ProfileScope() {
  if (!start_) return;
  std::lock_guard<std::mutex> lock(g_mu);
  cudaEvent_t stop = take_event();
  if (stop && cudaEventRecord(stop, stream_) == cudaSuccess) {
    g_spans[name_].push_back(Span{start_, stop});
  } else {
    g_free.push_back(start_);
    if (stop) g_free.push_back(stop);
  }
}

}  // namespace dsb

using namespace dsb;

extern "C" {

void ds_profile_enable(int on) { g_enabled.store(on != 0); }

void ds_profile_select(const char* names) {
  std::lock_guard<std::mutex> lock(g_mu);
  g_only.clear();
  if (!names) return;
  const std::string all(names);
  size_t at = 0;
  while (at <= all.size()) {
    const size_t end = all.find(',', at);
    const std::string one = all.substr(at, end == std::string::npos ? std::string::npos : end - at);
    if (!one.empty()) g_only.insert(one);
    if (end == std::string::npos) break;
    at = end + 1;
  }
}

void ds_profile_reset(void) {
  std::lock_guard<std::mutex> lock(g_mu);
  for (auto& kv : g_spans)
    for (Span& sp : kv.second) {
      g_free.push_back(sp.start);
      g_free.push_back(sp.stop);
    }
  g_spans.clear();
}

int ds_profile_read(const char* name, double* total_ms, int64_t* launches) {
  std::lock_guard<std::mutex> lock(g_mu);
  double total = 0.0;
  int64_t count = 0;
  auto it = g_spans.find(name ? name : "");
  if (it != g_spans.end()) {
    for (Span& sp : it->second) {
      cudaError_t e = cudaEventSynchronize(sp.stop);
      if (e != cudaSuccess) return cuda_status(e);
      float ms = 0.0f;
      e = cudaEventElapsedTime(&ms, sp.start, sp.stop);
      if (e != cudaSuccess) return cuda_status(e);
      total += ms;
      ++count;
    }
  }
  if (total_ms) *total_ms = total;
  if (launches) *launches = count;
  return DS_OK;
}

}  // extern "C"
