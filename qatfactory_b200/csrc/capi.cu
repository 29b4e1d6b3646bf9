// Library-level entry points of libqatf.so: version, status strings and the launch count.
#include <atomic>

#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {
static std::atomic<unsigned long long> g_launches{0};
int launched(int status) {
  if (status == QATF_OK) g_launches.fetch_add(1, std::memory_order_relaxed);
  return status;
}
}  // namespace qatf

extern "C" int qatf_version(void) { return 100; }

extern "C" uint64_t qatf_launch_count(void) { return qatf::g_launches.load(std::memory_order_relaxed); }

extern "C" const char* qatf_status_string(int status) {
  switch (status) {
    case QATF_OK:
      return "ok";
    case QATF_ERR_INVALID:
      return "invalid argument (null pointer, shape or stride)";
    case QATF_ERR_DTYPE:
      return "unsupported dtype code";
    case QATF_ERR_LAUNCH:
      return "CUDA launch or runtime call failed";
    case QATF_ERR_DEVICE:
      return "current device is not an sm_100 GPU";
    case QATF_ERR_TIMEOUT:
      return "device-side bounded wait expired";
    case QATF_ERR_UNSUPPORTED:
      return "shape not supported by this entry point";
    default:
      return "unknown status";
  }
}
