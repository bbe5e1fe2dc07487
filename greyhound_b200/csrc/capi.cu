// Library-wide C-ABI plumbing: version, last-error string, launch counter.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

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

// ---------------------------------------------------------------------------
// Sticky device-error bits, one int per device index, in pinned host memory
// that the GPU writes directly. Every entry point that owns a workspace status
// word ends with publish_status(): a one-thread kernel that ORs a non-zero
// status into this device's slot (nothing crosses the bus when the status is
// zero). The host reads and clears a slot with gh_take_device_errors() without
// synchronising, so a problem recorded by call k is seen at call k + 1 or
// later, once the GPU has run call k.
namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_slots_once;
int* g_slots = nullptr;

__global__ void publish_status_kernel(const int* __restrict__ status, int* slot) {
  const int v = *reinterpret_cast<const volatile int*>(status);
  if (v) {
    volatile int* h = slot;
    *h = *h | v;
  }
}
}  // namespace

int* error_slots() {
  std::call_once(g_slots_once, [] {
    void* p = nullptr;
    if (cudaHostAlloc(&p, kMaxDevices * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess) {
      memset(p, 0, kMaxDevices * sizeof(int));
      g_slots = static_cast<int*>(p);
    } else {
      cudaGetLastError();
    }
  });
  return g_slots;
}

int publish_status(const int* status, cudaStream_t st) {
  if (!status) return GH_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(GH_EUNSUPPORTED, "device index %d out of range", dev);
  int* slots = error_slots();
  if (!slots) return set_error(GH_ECUDA, "could not allocate the pinned device-error slots");
  void* dslot = nullptr;
  e = cudaHostGetDevicePointer(&dslot, slots + dev, 0);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
  publish_status_kernel<<<1, 1, 0, st>>>(status, static_cast<int*>(dslot));
  count_launch(1);
  return check_launch("publish_status");
}

}  // namespace gh

extern "C" int gh_take_device_errors(int device) {
  if (device < 0 || device >= gh::kMaxDevices || !gh::g_slots) return 0;
  return __atomic_exchange_n(&gh::g_slots[device], 0, __ATOMIC_SEQ_CST);
}

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
