// Allocation-free BF16 projection: klab_raw_linear_noalloc.
//
// Some callers cannot allocate device memory for the split-K workspace: code
// that runs where no allocator is available (a bare ctypes/C caller without a
// framework allocator, a plugin inside a host application that owns all device
// memory, a fixed-footprint serving process that must not grow after start-up).
// For them this entry point takes the split-K scratch from a fixed array inside
// the library instead of from the caller. It launches the same projection kernel
// as klab_raw_linear through klab_gemv, so its results are bit-identical.
//
// The scratch is a file-scope __device__ array of kScratchBytes (4 MiB). Every
// GPU that loads the library holds it until the process exits. In host code the
// array's name is only a host-side stand-in for the symbol, so its device
// address is obtained once per device with cudaGetSymbolAddress (with that
// device current) and cached. That set-up happens on the first call on each
// device: make that first call before any CUDA graph capture. The cached address
// belongs to the device's primary context: after cudaDeviceReset on a device, its
// cached address is stale, so use this entry point only in processes that do not
// reset their devices.
//
// All calls share the array and it keeps the last call's contents. The first
// 64 KiB hold the split-K completion tickets, which must start at zero: every
// call that splits clears that whole 64 KiB region with cudaMemsetAsync on its
// stream before the launch (a memset, not an allocation). Calls whose kernels can overlap on
// the GPU (different streams, or different host threads) race on the array and
// must be serialized by the caller. Shapes whose split-K scratch exceeds the
// array are rejected with KLAB_E_SCRATCH before any device work.
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/klab_b200.h"

namespace {

constexpr size_t kScratchBytes = 4u << 20;  // stated maximum: 4 MiB per device
constexpr size_t kTicketBytes = 64u << 10;  // the zero-initialised ticket region
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of the scratch array for the current device (set up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return KLAB_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_address[dev]) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess) return err;
    if (!ptr) return KLAB_E_DEVICE;
    g_scratch_address[dev] = ptr;
  }
  *out = g_scratch_address[dev];
  return 0;
}

}  // namespace

extern "C" KLAB_API int klab_raw_linear_noalloc(const void* x, const void* w, void* out, int out_dtype, int m, int n,
                                                int k, void* stream) {
  if (!x || !w || !out || m <= 0 || n <= 0 || k <= 0) return KLAB_E_INVALID;
  const size_t need = klab_gemv_workspace_bytes(KLAB_W_BF16, m, n, k);
  if (need > kScratchBytes) return KLAB_E_SCRATCH;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  if (need > 0) {
    cudaError_t err = cudaMemsetAsync(scratch, 0, kTicketBytes, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return err;
  }
  return klab_gemv(KLAB_W_BF16, KLAB_DT_BF16, x, k, w, nullptr, nullptr, out, n, out_dtype, m, n, k,
                   need > 0 ? scratch : nullptr, need > 0 ? kScratchBytes : 0, stream);
}
