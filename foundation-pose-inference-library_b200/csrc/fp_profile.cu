// Stage timing / launch counting (see fp_profile.hpp and fpk_profile_* in fpk.h).
#include <atomic>
#include <mutex>
#include <vector>

#include "fp_profile.hpp"
#include "fpk.h"

namespace fpb {
namespace prof {

namespace {
struct Rec {
  cudaEvent_t a, b;
  double work;
  int kind;
};
std::mutex g_mu;
std::atomic<bool> g_on{false};
std::vector<Rec> g_pending;
std::vector<cudaEvent_t> g_pool;
double g_ms[kKinds] = {};
double g_work[kKinds] = {};
long long g_timed[kKinds] = {};
std::atomic<long long> g_launch[kKinds];

cudaEvent_t take() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void resolveLocked() {
  for (Rec& r : g_pending) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      g_ms[r.kind] += ms;
      g_work[r.kind] += r.work;
      g_timed[r.kind] += 1;
    }
    g_pool.push_back(r.a);
    g_pool.push_back(r.b);
  }
  g_pending.clear();
}
}  // namespace

void countLaunch(int kind, int n) { g_launch[kind].fetch_add(n, std::memory_order_relaxed); }
bool enabled() { return g_on.load(std::memory_order_relaxed); }

Scope::Scope(int kind, double work, cudaStream_t s) : kind_(kind), work_(work), s_(s) {
  if (!enabled()) return;
  std::lock_guard<std::mutex> lock(g_mu);
  a_ = take();
  cudaEventRecord(a_, s_);
}

Scope::~Scope() {
  if (a_ == nullptr) return;
  std::lock_guard<std::mutex> lock(g_mu);
  cudaEvent_t b = take();
  cudaEventRecord(b, s_);
  g_pending.push_back({a_, b, work_, kind_});
}

}  // namespace prof
}  // namespace fpb

extern "C" {

void fpk_profile_enable(int enable) { fpb::prof::g_on.store(enable != 0); }

void fpk_profile_reset(void) {
  using namespace fpb::prof;
  std::lock_guard<std::mutex> lock(g_mu);
  resolveLocked();
  for (int k = 0; k < kKinds; ++k) {
    g_ms[k] = g_work[k] = 0.0;
    g_timed[k] = 0;
    g_launch[k].store(0);
  }
}

int fpk_profile_read(double* ms, double* work, long long* timed, long long* launches) {
  using namespace fpb::prof;
  std::lock_guard<std::mutex> lock(g_mu);
  resolveLocked();
  for (int k = 0; k < kKinds; ++k) {
    if (ms) ms[k] = g_ms[k];
    if (work) work[k] = g_work[k];
    if (timed) timed[k] = g_timed[k];
    if (launches) launches[k] = g_launch[k].load();
  }
  return kKinds;
}

}  // extern "C"
