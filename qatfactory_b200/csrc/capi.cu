// Library-level entry points of libqatf.so: version and status strings.
#include "qatf.h"

extern "C" int qatf_version(void) { return 100; }

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
