// Library-level C-ABI entry points (version, status text).
#include <atomic>

#include "gsplat_b200.h"
#include "gsb_host.cuh"

namespace gsb {
static std::atomic<uint64_t> g_launches{0};
void note_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
}  // namespace gsb

extern "C" uint64_t gsb_kernel_launches(void) { return gsb::g_launches.load(std::memory_order_relaxed); }

extern "C" int gsb_version(void) { return 100; }  // 0.1.0

extern "C" const char* gsb_status_string(int code) {
  switch (code) {
    case GSB_OK: return "ok";
    case GSB_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, bad shape or bad config)";
    case GSB_ERR_UNSUPPORTED: return "unsupported configuration (tile_size must be 16)";
    case GSB_ERR_WORKSPACE: return "workspace smaller than the *_workspace_size query";
    case GSB_ERR_CAPACITY:
      return "size exceeds capacity (pair count beyond the int32 index range, or beyond the fixed maximum "
             "of an allocation-free entry point)";
    case GSB_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait ran out";
    case GSB_ERR_CUDA: return "CUDA runtime error";
    case GSB_ERR_DEVICE_BOUNDS: return "device-side bounds check failed";
    default: return "unknown status code";
  }
}
