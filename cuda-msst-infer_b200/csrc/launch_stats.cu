// launch_stats.cu — launch counting and per-kernel event timing (LaunchScope).
//
// Timing is off by default; then a scope costs one relaxed atomic increment.
// While on, every launch takes two events from a per-device pool and is recorded
// as {name, flop, bytes, start, stop}; msst_kernel_timing_report() waits for the
// stop events, aggregates by name and returns the events to the pool.
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace msst {
namespace {

struct Record {
  const char* name;
  double flop, bytes;
  int device;
  cudaEvent_t start, stop;
};

std::atomic<unsigned long long> g_launches{0};
std::atomic<bool> g_timing{false};
std::mutex g_mu;
std::vector<Record> g_records;
std::map<int, std::vector<cudaEvent_t>> g_pool;

cudaEvent_t take_event(int dev) {
  auto& v = g_pool[dev];
  if (!v.empty()) {
    cudaEvent_t e = v.back();
    v.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

LaunchScope::LaunchScope(const char* name, double flop, double bytes, cudaStream_t s) : slot_(-1), stream_(s) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_timing.load(std::memory_order_relaxed)) return;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaEvent_t a = take_event(dev), b = take_event(dev);
  if (!a || !b) {
    if (a) g_pool[dev].push_back(a);
    if (b) g_pool[dev].push_back(b);
    return;
  }
  if (cudaEventRecord(a, s) != cudaSuccess) {
    g_pool[dev].push_back(a);
    g_pool[dev].push_back(b);
    return;
  }
  slot_ = (long long)g_records.size();
  g_records.push_back(Record{name, flop, bytes, dev, a, b});
}

LaunchScope::~LaunchScope() {
  if (slot_ < 0) return;
  std::lock_guard<std::mutex> lk(g_mu);
  if (slot_ < (long long)g_records.size()) cudaEventRecord(g_records[slot_].stop, stream_);
}

unsigned long long launch_count(bool reset) { return reset ? g_launches.exchange(0) : g_launches.load(); }

void set_kernel_timing(bool on) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (on) {
    for (auto& r : g_records) {
      g_pool[r.device].push_back(r.start);
      g_pool[r.device].push_back(r.stop);
    }
    g_records.clear();
  }
  g_timing.store(on);
}

std::vector<KernelStat> kernel_timing_report() {
  std::lock_guard<std::mutex> lk(g_mu);
  std::vector<KernelStat> out;
  std::map<std::string, size_t> idx;
  for (auto& r : g_records) {
    MSST_CUDA(cudaEventSynchronize(r.stop));
    float ms = 0.f;
    MSST_CUDA(cudaEventElapsedTime(&ms, r.start, r.stop));
    auto it = idx.find(r.name);
    if (it == idx.end()) {
      it = idx.emplace(r.name, out.size()).first;
      out.push_back(KernelStat{r.name});
    }
    KernelStat& k = out[it->second];
    k.launches += 1;
    k.ms += ms;
    k.flop += r.flop;
    k.bytes += r.bytes;
  }
  return out;
}

}  // namespace msst
