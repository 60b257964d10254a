// Library identification, error names and context identification of the rfm C ABI.
#include <cuda.h>  // CUresult / CUcontext types; the driver entry point is resolved at run time

#include "rfm_common.cuh"

extern "C" const char* rfm_version(void) { return "rfm 0.2.0 sm_100a"; }

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

namespace rfm {

unsigned long long current_context_id() {
  // cuCtxGetId through the runtime's driver entry-point lookup, so the library
  // does not link libcuda itself (it loads on machines without a driver)
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static const GetId get_id = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<GetId>(nullptr);
    }
    return reinterpret_cast<GetId>(fn);
  }();
  if (get_id == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(nullptr, &id) == CUDA_SUCCESS ? id : 0;
}

}  // namespace rfm
