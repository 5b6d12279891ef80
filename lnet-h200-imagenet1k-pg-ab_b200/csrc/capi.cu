// Error plumbing, launch accounting and version of the lnet_b200 C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <vector>

#include "common.cuh"

namespace lnet {

static thread_local std::string g_last_error;
static thread_local int g_launches = 0;

// Optional per-launch device timing: when enabled, every launch is followed by
// an event on its stream; consecutive events bracket one kernel because the
// launches of one entry point are stream-ordered.
struct ProfRecord {
  const char *name;
  cudaEvent_t stop;
};
static bool g_prof_on = false;
static std::vector<ProfRecord> g_prof;
static std::vector<cudaEvent_t> g_prof_pool;
static thread_local cudaStream_t g_stream = nullptr;
static thread_local cudaEvent_t g_prev = nullptr;

static cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return LNET_OK;
  return fail(LNET_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

void reset_launches() { g_launches = 0; }

void begin_entry(cudaStream_t stream) {
  g_stream = stream;
  if (!g_prof_on) return;
  g_prev = prof_event();
  cudaEventRecord(g_prev, stream);
  g_prof.push_back({nullptr, g_prev});
}
void count_launch(int n) { g_launches += n; }
int launch_count() { return g_launches; }

int after_library(const char *what) {
  if (g_prof_on) {
    cudaEvent_t e = prof_event();
    cudaEventRecord(e, g_stream);
    g_prof.push_back({what, e});
  }
  return LNET_OK;
}

int after_launch(const char *what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(LNET_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(err));
  ++g_launches;
  if (g_prof_on) {
    cudaEvent_t e = prof_event();
    cudaEventRecord(e, g_stream);
    g_prof.push_back({what, e});
  }
  return LNET_OK;
}

}  // namespace lnet

extern "C" const char *lnet_b200_last_error(void) { return lnet::g_last_error.c_str(); }
extern "C" int lnet_b200_last_launch_count(void) { return lnet::g_launches; }
extern "C" const char *lnet_b200_version(void) { return "lnet_b200 0.1.0 (sm_100a)"; }

// Enable (1) or disable (0) per-launch timing; enabling clears old records.
extern "C" void lnet_b200_profile_enable(int on) {
  for (auto &r : lnet::g_prof) lnet::g_prof_pool.push_back(r.stop);
  lnet::g_prof.clear();
  lnet::g_prof_on = on != 0;
}

// Synchronise the recorded events and aggregate per kernel name.  Writes up
// to `max_entries` rows: names as '\n'-separated text in names_buf, total
// milliseconds and launch counts.  Returns the number of distinct kernels.
extern "C" int lnet_b200_profile_read(char *names_buf, int names_bytes, float *total_ms,
                                      int *launches, int max_entries) {
  std::map<std::string, std::pair<double, int>> agg;
  std::vector<std::string> order;
  cudaEvent_t prev = nullptr;
  for (auto &r : lnet::g_prof) {
    cudaEventSynchronize(r.stop);
    if (r.name == nullptr) {
      prev = r.stop;
      continue;
    }
    float ms = 0.f;
    if (prev) cudaEventElapsedTime(&ms, prev, r.stop);
    prev = r.stop;
    std::string key(r.name);
    if (!agg.count(key)) order.push_back(key);
    agg[key].first += ms;
    agg[key].second += 1;
  }
  int n = 0;
  std::string names;
  for (auto &k : order) {
    if (n >= max_entries) break;
    total_ms[n] = (float)agg[k].first;
    launches[n] = agg[k].second;
    names += k + "\n";
    ++n;
  }
  if (names_buf && names_bytes > 0) {
    snprintf(names_buf, names_bytes, "%s", names.c_str());
  }
  return n;
}
