// Per-launch CUDA-event profiler of the library's kernels (nsrl_profile_*).
#include <mutex>
#include <vector>

#include "internal.h"

namespace nsrl {
namespace {

struct Entry {
  const char* name;
  cudaEvent_t a, b;
  double ops, bytes;
};

std::mutex g_mu;
bool g_on = false;
std::vector<Entry> g_entries;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

}  // namespace

ProfScope::ProfScope(const char* name, cudaStream_t s, double ops, double bytes)
    : name_(name), stream_(s), ops_(ops), bytes_(bytes), ev_(nullptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_on) return;
  ev_ = take_event();
  cudaEventRecord(ev_, s);
}

ProfScope::~ProfScope() {
  if (!ev_) return;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaEvent_t e = take_event();
  cudaEventRecord(e, stream_);
  g_entries.push_back(Entry{name_, ev_, e, ops_, bytes_});
}

}  // namespace nsrl

using namespace nsrl;

extern "C" {

void nsrl_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_on = enable != 0;
}

void nsrl_profile_reset(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& e : g_entries) {
    g_pool.push_back(e.a);
    g_pool.push_back(e.b);
  }
  g_entries.clear();
}

size_t nsrl_profile_count(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  return g_entries.size();
}

nsrl_status nsrl_profile_entry(size_t i, const char** name, float* ms, double* ops, double* bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (i >= g_entries.size()) return NSRL_INVALID_SHAPE;
  const Entry& e = g_entries[i];
  cudaError_t err = cudaEventSynchronize(e.b);
  if (err != cudaSuccess) {
    set_error("profile: %s", cudaGetErrorString(err));
    return NSRL_CUDA_ERROR;
  }
  float t = 0.f;
  err = cudaEventElapsedTime(&t, e.a, e.b);
  if (err != cudaSuccess) {
    set_error("profile: %s", cudaGetErrorString(err));
    return NSRL_CUDA_ERROR;
  }
  if (name) *name = e.name;
  if (ms) *ms = t;
  if (ops) *ops = e.ops;
  if (bytes) *bytes = e.bytes;
  return NSRL_OK;
}

}  // extern "C"
