// Host runtime pieces of the C ABI: status strings, per-thread error detail,
// device-property and occupancy caches.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <set>
#include <tuple>
#include <unordered_map>

#include "launch.cuh"

namespace bysj {

namespace {
thread_local char g_last_error[512] = {0};

std::mutex g_mutex;
DeviceInfo g_devices[64];
bool g_device_ready[64] = {false};

struct OccKey {
  const void* kernel;
  int device;
  size_t smem;
  int threads;
  bool operator==(const OccKey& o) const {
    return kernel == o.kernel && device == o.device && smem == o.smem && threads == o.threads;
  }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return std::hash<const void*>()(k.kernel) ^ (size_t(k.device) << 40) ^
           (k.smem << 8) ^ (size_t(k.threads) << 52);
  }
};
std::unordered_map<OccKey, int, OccHash> g_occupancy;
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return status;
}

void clear_error() { g_last_error[0] = 0; }

int cuda_check(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return BYSJ_OK;
  return fail(BYSJ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int launch_check(const char* kernel) {
  const cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) return BYSJ_OK;
  return fail(BYSJ_ERR_LAUNCH, "launch of %s failed: %s", kernel,
              cudaGetErrorString(err));
}

const DeviceInfo& current_device_info() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    device = 0;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_device_ready[device]) {
    DeviceInfo info;
    info.device = device;
    int value = 0;
    if (cudaDeviceGetAttribute(&value, cudaDevAttrMultiProcessorCount,
                               device) == cudaSuccess && value > 0)
      info.sm_count = value;
    if (cudaDeviceGetAttribute(&value,
                               cudaDevAttrMaxThreadsPerMultiProcessor,
                               device) == cudaSuccess && value > 0)
      info.max_threads_per_sm = value;
    g_devices[device] = info;
    g_device_ready[device] = true;
  }
  return g_devices[device];
}

int allow_dynamic_smem(const void* kernel, size_t bytes) {
  if (bytes == 0) return BYSJ_OK;
  static std::mutex m;
  static std::set<std::tuple<const void*, int, size_t>> done;
  const DeviceInfo& info = current_device_info();
  std::lock_guard<std::mutex> lock(m);
  const auto key = std::make_tuple(kernel, info.device, bytes);
  if (done.count(key)) return BYSJ_OK;
  // The default limit is 48 KB of static and dynamic shared memory together.
  cudaFuncAttributes attr{};
  int st = cuda_check(cudaFuncGetAttributes(&attr, kernel), "kernel attributes");
  if (st != BYSJ_OK) return st;
  if (attr.sharedSizeBytes + bytes > 48 * 1024)
    st = cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(bytes)),
                    "opt in to dynamic shared memory");
  if (st == BYSJ_OK) done.insert(key);
  return st;
}

int resident_blocks(const void* kernel, size_t dynamic_smem, int threads) {
  const DeviceInfo& info = current_device_info();
  OccKey key{kernel, info.device, dynamic_smem, threads};
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) return it->second;
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &blocks, kernel, threads, dynamic_smem) != cudaSuccess ||
      blocks < 1) {
    cudaGetLastError();
    blocks = 1;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  g_occupancy[key] = blocks;
  return blocks;
}

}  // namespace bysj

extern "C" {

int bysj_version(void) { return 10000; }

const char* bysj_status_string(int status) {
  switch (status) {
    case BYSJ_OK: return "ok";
    case BYSJ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BYSJ_ERR_WORKSPACE: return "workspace missing or too small";
    case BYSJ_ERR_UNSUPPORTED: return "unsupported shape";
    case BYSJ_ERR_CUDA: return "CUDA runtime error";
    case BYSJ_ERR_LAUNCH: return "kernel launch failed";
    case BYSJ_ERR_TOO_LARGE: return "size beyond a fixed capacity";
    default: return "unknown status";
  }
}

const char* bysj_last_error(void) { return bysj::g_last_error; }

}  // extern "C"
