// Host-side plumbing of the C ABI: version, per-thread error messages, launch counter and the
// opt-in for large dynamic shared memory.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <set>
#include <utility>

#include "zn_common.cuh"

namespace zn {

static thread_local char g_error[512];
static std::atomic<uint64_t> g_launches{0};

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ZN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ZN_OK;
}

void count_launch(int n) { g_launches.fetch_add(uint64_t(n), std::memory_order_relaxed); }

int set_max_smem(const void* func, int bytes) {
  // The attribute is per function and device; remember which pairs are done.
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  if (bytes <= 48 * 1024 || done.count({func, dev})) return ZN_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return set_error(ZN_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  done.insert({func, dev});
  return ZN_OK;
}

}  // namespace zn

extern "C" {

int zn_version(void) { return ZN_ABI_VERSION; }
const char* zn_last_error(void) { return zn::g_error; }
uint64_t zn_launch_count(void) { return zn::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
