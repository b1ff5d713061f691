// Host-side plumbing of the C ABI: version, per-thread error messages, launch counter, the opt-in
// for large dynamic shared memory, NVTX ranges and the opt-in kernel timing.
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>

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
  // The opt-in limit covers static and dynamic shared memory together.
  cudaFuncAttributes fa{};
  int optin = 0;
  cudaError_t e = cudaFuncGetAttributes(&fa, func);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e == cudaSuccess) {
    if (bytes > optin - int(fa.sharedSizeBytes))
      return set_error(ZN_ERR_CUDA, "kernel needs %d bytes of shared memory, the device allows %d", bytes,
                       optin - int(fa.sharedSizeBytes));
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - int(fa.sharedSizeBytes));
  }
  if (e != cudaSuccess) return set_error(ZN_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  done.insert({func, dev});
  return ZN_OK;
}

// ---- opt-in kernel timing -----------------------------------------------------------------

struct Timing {
  std::mutex mu;
  std::string kernel;  // "" = disabled, "*" = every kernel kind
  struct Rec {
    std::string kernel;
    cudaEvent_t start, stop;
  };
  std::vector<Rec> pending;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pool;
};
static Timing g_timing;

NvtxScope::NvtxScope(const char* name) { nvtxRangePushA(name); }
NvtxScope::~NvtxScope() { nvtxRangePop(); }

TimedLaunch::TimedLaunch(const char* kernel, cudaStream_t s) : slot(-1), stream(s) {
  nvtxRangePushA(kernel);  // a host range around each kernel stage's launch (no-op without a tool)
  std::lock_guard<std::mutex> lock(g_timing.mu);
  if (g_timing.kernel.empty() || (g_timing.kernel != "*" && g_timing.kernel != kernel)) return;
  std::pair<cudaEvent_t, cudaEvent_t> ev;
  if (!g_timing.pool.empty()) {
    ev = g_timing.pool.back();
    g_timing.pool.pop_back();
  } else if (cudaEventCreate(&ev.first) != cudaSuccess || cudaEventCreate(&ev.second) != cudaSuccess) {
    return;
  }
  cudaEventRecord(ev.first, s);
  slot = int(g_timing.pending.size());
  g_timing.pending.push_back({kernel, ev.first, ev.second});
}

TimedLaunch::~TimedLaunch() {
  nvtxRangePop();
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_timing.mu);
  if (slot < int(g_timing.pending.size())) cudaEventRecord(g_timing.pending[slot].stop, stream);
}

}  // namespace zn

extern "C" {

int zn_timing_enable(const char* kernel, int enable) {
  std::lock_guard<std::mutex> lock(zn::g_timing.mu);
  zn::g_timing.kernel = enable && kernel ? kernel : "";
  return ZN_OK;
}

int zn_timing_read(const char* kernel, double* total_ms, int64_t* launches) {
  std::lock_guard<std::mutex> lock(zn::g_timing.mu);
  // Launches of one kind may overlap (callers that launch on several streams or threads), so the
  // time is the union of their [start, stop] intervals, measured from the kind's first start
  // event: the time during which at least one of them ran.
  std::vector<std::pair<double, double>> iv;
  std::vector<zn::Timing::Rec> keep;
  cudaEvent_t origin = nullptr;
  for (auto& r : zn::g_timing.pending) {
    if (kernel && r.kernel != kernel) {
      keep.push_back(r);
      continue;
    }
    float a = 0, b = 0;
    if (cudaEventSynchronize(r.stop) != cudaSuccess)
      return zn::set_error(ZN_ERR_CUDA, "zn_timing_read: %s", cudaGetErrorString(cudaGetLastError()));
    if (!origin) origin = r.start;
    if (cudaEventElapsedTime(&a, origin, r.start) != cudaSuccess || cudaEventElapsedTime(&b, origin, r.stop) != cudaSuccess)
      return zn::set_error(ZN_ERR_CUDA, "zn_timing_read: %s", cudaGetErrorString(cudaGetLastError()));
    iv.push_back({double(a), double(b)});
    zn::g_timing.pool.push_back({r.start, r.stop});
  }
  zn::g_timing.pending.swap(keep);
  std::sort(iv.begin(), iv.end());
  double sum = 0, lo = 0, hi = 0;
  bool open = false;
  for (auto& x : iv) {
    if (!open || x.first > hi) {
      if (open) sum += hi - lo;
      lo = x.first;
      hi = x.second;
      open = true;
    } else if (x.second > hi) {
      hi = x.second;
    }
  }
  if (open) sum += hi - lo;
  if (launches) *launches = int64_t(iv.size());
  if (total_ms) *total_ms = sum;
  return ZN_OK;
}

int zn_version(void) { return ZN_ABI_VERSION; }
const char* zn_last_error(void) { return zn::g_error; }
uint64_t zn_launch_count(void) { return zn::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
