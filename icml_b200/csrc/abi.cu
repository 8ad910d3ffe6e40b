// Error reporting and version of the C-ABI (include/pgf.h).
#include "common.cuh"

#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

namespace pgf {

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

// ---------------------------------------------------------------------------------------------
// launch counter and event timing
// ---------------------------------------------------------------------------------------------
static std::atomic<long long> g_launches{0};
static std::atomic<bool> g_prof_on{false};
static std::mutex g_prof_mu;
struct ProfRec { int id; cudaEvent_t a, b; bool closed; double work; };
static std::vector<ProfRec> g_prof;
static std::vector<cudaEvent_t> g_pool;
static size_t g_pool_used = 0;
static int g_open[PROF_COUNT];

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static cudaEvent_t pool_event() {
  if (g_pool_used == g_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_pool.push_back(e);
  }
  return g_pool[g_pool_used++];
}

void prof_begin(int id, cudaStream_t s) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEvent_t a = pool_event(), b = pool_event();
  if (!a || !b) return;
  cudaEventRecord(a, s);
  g_open[id] = int(g_prof.size());
  g_prof.push_back({id, a, b, false, 0.0});
}

void prof_end(int id, cudaStream_t s, double work) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  int i = g_open[id];
  if (i < 0 || i >= int(g_prof.size()) || g_prof[i].closed || g_prof[i].id != id) return;
  cudaEventRecord(g_prof[i].b, s);
  g_prof[i].closed = true;
  g_prof[i].work = work;
  g_open[id] = -1;
}

}  // namespace pgf

extern "C" long long pgf_launch_count(void) { return pgf::g_launches.load(); }

extern "C" int pgf_profile(int enable) {
  std::lock_guard<std::mutex> lk(pgf::g_prof_mu);
  if (enable) {
    pgf::g_prof.clear();
    pgf::g_pool_used = 0;
    for (int i = 0; i < pgf::PROF_COUNT; ++i) pgf::g_open[i] = -1;
  }
  pgf::g_prof_on.store(enable != 0);
  return PGF_OK;
}

extern "C" int pgf_profile_read(int id, long long* count, double* total_ms, double* total_work) {
  std::lock_guard<std::mutex> lk(pgf::g_prof_mu);
  long long n = 0;
  double ms = 0.0, work = 0.0;
  for (auto& r : pgf::g_prof) {
    if (r.id != id || !r.closed) continue;
    if (cudaEventSynchronize(r.b) != cudaSuccess) { pgf::set_error("profile: event sync failed"); return PGF_ERR_CUDA; }
    float t = 0.f;
    if (cudaEventElapsedTime(&t, r.a, r.b) != cudaSuccess) { pgf::set_error("profile: elapsed failed"); return PGF_ERR_CUDA; }
    ++n;
    ms += t;
    work += r.work;
  }
  if (count) *count = n;
  if (total_ms) *total_ms = ms;
  if (total_work) *total_work = work;
  return PGF_OK;
}

extern "C" const char* pgf_last_error(void) { return pgf::g_err; }

extern "C" int pgf_version(void) { return 100; /* 0.1.0 */ }
