// Peer memory (CUDA IPC) and the small kernels that frame a gathered step:
// klab_step_begin bumps the step epoch, klab_wait_flags waits (bounded) until
// every rank has raised its flag for a slot. Used by the column-sharded chain,
// whose projections push their outputs to the peers (stream_gemv.cuh Gather).
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "klab_kernels.h"

namespace klab {
namespace {

__global__ void step_begin_kernel(unsigned* epoch) {
  grid_dependency_wait();
  *epoch += 1u;
  grid_launch_dependents();
}

__global__ void wait_flags_kernel(const unsigned* flags, int slot, int npeers, const unsigned* epoch, int* status) {
  grid_dependency_wait();
  if (threadIdx.x < npeers) {
    const unsigned target = *epoch;
    if (!wait_flag_geq(flags + slot * npeers + threadIdx.x, target)) record_status(status, kStatusFlagTimeout);
  }
  __syncthreads();
  grid_launch_dependents();
}

}  // namespace
}  // namespace klab

extern "C" {

KLAB_API int klab_ipc_malloc(size_t bytes, void** ptr, void* handle64) {
  if (!ptr || !handle64 || bytes == 0) return KLAB_E_INVALID;
  cudaError_t err = cudaMalloc(ptr, bytes);
  if (err != cudaSuccess) return err;
  err = cudaMemset(*ptr, 0, bytes);
  if (err == cudaSuccess) {
    cudaIpcMemHandle_t h;
    err = cudaIpcGetMemHandle(&h, *ptr);
    if (err == cudaSuccess) std::memcpy(handle64, &h, sizeof(h));
  }
  if (err != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
  }
  return err;
}

KLAB_API int klab_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return KLAB_E_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

KLAB_API int klab_ipc_close(void* ptr) {
  if (!ptr) return KLAB_E_INVALID;
  return cudaIpcCloseMemHandle(ptr);
}

KLAB_API int klab_ipc_free(void* ptr) {
  if (!ptr) return KLAB_E_INVALID;
  return cudaFree(ptr);
}

KLAB_API int klab_step_begin(unsigned* epoch, void* stream) {
  if (!epoch) return KLAB_E_INVALID;
  klab::step_begin_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(epoch);
  return cudaGetLastError();
}

KLAB_API int klab_wait_flags(const unsigned* flags, int slot, int npeers, const unsigned* epoch, void* stream) {
  if (!flags || !epoch || slot < 0 || npeers <= 0 || npeers > 32) return KLAB_E_INVALID;
  klab::wait_flags_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, slot, npeers, epoch,
                                                                           klab::device_status_address());
  return cudaGetLastError();
}

}  // extern "C"
