// Status reporting and small helpers of the C ABI (include/gsplat_b200.h).
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace gsb {

namespace {
thread_local char g_error[512] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace gsb

extern "C" {

const char* gs_status_string(int status) {
  switch (status) {
    case GS_OK: return "ok";
    case GS_ERR_INVALID: return "invalid argument";
    case GS_ERR_UNSUPPORTED: return "unsupported";
    case GS_ERR_OVERFLOW: return "index overflow";
    case GS_ERR_CUDA: return "cuda error";
    case GS_ERR_WORKSPACE: return "workspace missing or too small";
    case GS_ERR_DEVICE: return "on-device check failed";
    default: return "unknown status";
  }
}

const char* gs_last_error(void) { return gsb::g_error; }

int gs_version(void) { return 100; }

// gsplat_intersect.cpp:60-65: floor(log2(float(value))) + 1.
int32_t gs_floor_log2_plus_one(int32_t value) {
  if (value <= 0) return -1;
  return static_cast<int32_t>(std::floor(std::log2(static_cast<float>(value)))) + 1;
}

}  // extern "C"
