// Library identification and error names of the rfm C ABI.
#include "rfm_common.cuh"

extern "C" const char* rfm_version(void) { return "rfm 0.1.0 sm_100a"; }

extern "C" const char* rfm_error_string(int code) {
  switch (code) {
    case RFM_OK: return "ok";
    case RFM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RFM_ERR_UNSUPPORTED: return "outside the supported envelope";
    case RFM_ERR_LAUNCH: return "CUDA launch error";
    case RFM_ERR_NO_DEVICE: return "no usable CUDA device";
    default: return "unknown error";
  }
}
