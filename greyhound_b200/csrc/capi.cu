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
