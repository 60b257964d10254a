// Peer memory and the per-step barrier of the sharded sweep's pushed exchange.
//
// A batch split by image over the ranks (one process per GPU) needs every
// rank's pairs on every rank.  The solver's epilogue stores each pair into
// every rank's gathered buffer (rfm_lsap_push): plain stores to peer memory
// over NVLink, mapped into this process with CUDA IPC.  No multicast object is
// created and no TMA or bulk copy reads peer memory.  peer_sync_kernel is the
// step's barrier: one warp, lane j raising this rank's flag on rank j and then
// waiting for rank j's flag here, every wait bounded.  No counterpart in the
// reference, which matches on one GPU.
#include <string.h>

#include "rfm_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");

namespace rfm {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The kernels before this one on the stream (the solver and its pushes) have
// completed; the system-scope fence orders their stores before the release
// store of the flag, and a peer that acquires the flag sees them.
__global__ void peer_sync_kernel(const __grid_constant__ rfm_peer_sync_args a) {
  const int j = static_cast<int>(threadIdx.x);
  const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(a.epoch) + 1u;
  if (j < a.world) {
    __threadfence_system();
    st_release_sys(a.arrive[j], target);
    int64_t polls = 0;
    unsigned ns = 64;
    // flags only grow; a peer already one step ahead also satisfies the wait
    while (static_cast<int32_t>(ld_acquire_sys(a.flags + j) - target) < 0) {
      if (++polls >= a.spin_limit) {
        atomicExch(a.error, 1);
        break;
      }
      __nanosleep(ns);
      if (ns < 256) ns <<= 1;  // short sleeps: an arrival is seen within a fraction of a microsecond
    }
  }
  __syncwarp();
  if (j == 0) *a.epoch = target;
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_peer_alloc(int64_t bytes, void** ptr, unsigned char* handle) {
  if (bytes <= 0 || ptr == nullptr || handle == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_LAUNCH;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return RFM_ERR_LAUNCH;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return RFM_OK;
}

extern "C" int rfm_peer_open(const unsigned char* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_LAUNCH;
  }
  *ptr = p;
  return RFM_OK;
}

extern "C" int rfm_peer_close(void* ptr) {
  if (ptr == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_LAUNCH;
  }
  return RFM_OK;
}

extern "C" int rfm_peer_free(void* ptr) {
  if (ptr == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  if (cudaFree(ptr) != cudaSuccess) {
    cudaGetLastError();
    return RFM_ERR_LAUNCH;
  }
  return RFM_OK;
}

extern "C" int rfm_peer_sync(const rfm_peer_sync_args* args, void* stream) {
  if (args == nullptr || args->world < 1 || args->world > RFM_MAX_PUSH || args->rank < 0 ||
      args->rank >= args->world || args->spin_limit < 1 || args->flags == nullptr || args->epoch == nullptr ||
      args->error == nullptr) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  for (int j = 0; j < args->world; ++j) {
    if (args->arrive[j] == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  }
  rfm::peer_sync_kernel<<<1, 32, 0, rfm::as_stream(stream)>>>(*args);
  return rfm::launch_status();
}
