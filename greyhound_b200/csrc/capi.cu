// Library-wide C-ABI plumbing: version, last-error string, launch counter.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace gh {

static thread_local char g_err[512] = "";
static std::atomic<long long> g_launches{0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GH_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return GH_OK;
}

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace gh

extern "C" int gh_abi_version(void) { return 1; }
extern "C" const char* gh_last_error_string(void) { return gh::g_err; }
extern "C" long long gh_launch_count(void) { return gh::g_launches.load(); }
extern "C" size_t gh_workspace_status_offset(void) { return 0; }

// ---------------------------------------------------------------------------
// Optional per-kernel-class timing with CUDA events (for the benchmark's
// roofline figures). Off by default; when on, every launch of a timed class
// is bracketed by two events on its stream.
#include <mutex>
#include <vector>

namespace gh {
namespace {
struct TimedLaunch {
  int cls;
  cudaEvent_t a, b;
};
std::mutex g_prof_mu;
std::vector<TimedLaunch> g_prof;
std::vector<cudaEvent_t> g_free_events;
std::atomic<int> g_prof_on{0};

cudaEvent_t take_event() {
  if (!g_free_events.empty()) {
    cudaEvent_t e = g_free_events.back();
    g_free_events.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}
}  // namespace

ProfScope::ProfScope(int cls, cudaStream_t st) : cls_(cls), st_(st), a_(nullptr) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  a_ = take_event();
  cudaEventRecord(static_cast<cudaEvent_t>(a_), st_);
}
ProfScope::~ProfScope() {
  if (!a_) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEvent_t b = take_event();
  cudaEventRecord(b, st_);
  g_prof.push_back({cls_, static_cast<cudaEvent_t>(a_), b});
}
}  // namespace gh

extern "C" void gh_profile_enable(int on) { gh::g_prof_on.store(on ? 1 : 0); }

extern "C" int gh_profile_read(double* ms_out, long long* count_out, int n_classes, int reset) {
  using namespace gh;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (int i = 0; i < n_classes; ++i) {
    ms_out[i] = 0.0;
    count_out[i] = 0;
  }
  for (auto& t : g_prof) {
    cudaError_t e = cudaEventSynchronize(t.b);
    if (e != cudaSuccess) return set_error(GH_ECUDA, "gh_profile_read: %s", cudaGetErrorString(e));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, t.a, t.b);
    if (t.cls >= 0 && t.cls < n_classes) {
      ms_out[t.cls] += ms;
      count_out[t.cls] += 1;
    }
  }
  if (reset) {
    for (auto& t : g_prof) {
      g_free_events.push_back(t.a);
      g_free_events.push_back(t.b);
    }
    g_prof.clear();
  }
  return GH_OK;
}
