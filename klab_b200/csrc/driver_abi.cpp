// The reference's C ABI over the CUDA driver API (native/driver.cpp:46-90):
// lab_load_ptx / lab_get_kernel / lab_launch / lab_unload / lab_error_string,
// with the same signatures, error codes (-1000 driver missing, -1001 no current
// context, -1002 null argument or zero dimension; positive CUresult passthrough)
// and ownership rules (callers own buffers, contexts, streams and the
// synchronization before unloading). libcuda is opened once with dlopen, so the
// library links no driver stub. Extensions: lab_launch_ex (dynamic shared
// memory, programmatic dependent launch) and lab_load_file.
#include <cuda.h>
#include <dlfcn.h>

#include <cstdio>
#include <mutex>
#include <vector>

#include "../../include/klab_b200.h"

namespace {

struct Driver {
  decltype(&cuInit) init = nullptr;
  decltype(&cuCtxGetCurrent) ctx_current = nullptr;
  decltype(&cuModuleLoadData) module_load = nullptr;
  decltype(&cuModuleGetFunction) module_function = nullptr;
  decltype(&cuModuleUnload) module_unload = nullptr;
  decltype(&cuLaunchKernel) launch = nullptr;
  decltype(&cuLaunchKernelEx) launch_ex = nullptr;
  decltype(&cuFuncSetAttribute) func_attribute = nullptr;
  decltype(&cuGetErrorString) error_string = nullptr;
  bool ready = false;
};

template <typename F>
void symbol(void* handle, F& fn, const char* name) {
  fn = reinterpret_cast<F>(dlsym(handle, name));
}

Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    // The handle stays open for the process lifetime.
    void* handle = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!handle) return;
    symbol(handle, d.init, "cuInit");
    symbol(handle, d.ctx_current, "cuCtxGetCurrent");
    symbol(handle, d.module_load, "cuModuleLoadData");
    symbol(handle, d.module_function, "cuModuleGetFunction");
    symbol(handle, d.module_unload, "cuModuleUnload");
    symbol(handle, d.launch, "cuLaunchKernel");
    symbol(handle, d.launch_ex, "cuLaunchKernelEx");
    symbol(handle, d.func_attribute, "cuFuncSetAttribute");
    symbol(handle, d.error_string, "cuGetErrorString");
    d.ready = d.init && d.ctx_current && d.module_load && d.module_function && d.module_unload && d.launch &&
              d.error_string;
  });
  return d;
}

int load_image(const void* image, void** out) {
  Driver& d = driver();
  if (!d.ready) return KLAB_E_DRIVER;
  int status = d.init(0);
  if (status) return status;
  CUcontext context = nullptr;
  status = d.ctx_current(&context);
  if (status) return status;
  if (!context) return KLAB_E_NO_CONTEXT;
  return d.module_load(reinterpret_cast<CUmodule*>(out), image);
}

}  // namespace

extern "C" {

int lab_load_ptx(const char* image, void** module_out) {
  if (!image || !module_out) return KLAB_E_INVALID;
  return load_image(image, module_out);
}

int lab_load_file(const char* path, void** module_out) {
  if (!path || !module_out) return KLAB_E_INVALID;
  FILE* file = std::fopen(path, "rb");
  if (!file) return KLAB_E_INVALID;
  std::vector<char> bytes;
  char buffer[1 << 16];
  size_t got;
  while ((got = std::fread(buffer, 1, sizeof(buffer), file)) > 0) bytes.insert(bytes.end(), buffer, buffer + got);
  std::fclose(file);
  if (bytes.empty()) return KLAB_E_INVALID;
  bytes.push_back('\0');  // PTX text must be NUL-terminated; binary images ignore it.
  return load_image(bytes.data(), module_out);
}

int lab_get_kernel(void* module, const char* name, void** fn_out) {
  if (!module || !name || !fn_out) return KLAB_E_INVALID;
  Driver& d = driver();
  if (!d.ready) return KLAB_E_DRIVER;
  return d.module_function(reinterpret_cast<CUfunction*>(fn_out), static_cast<CUmodule>(module), name);
}

int lab_launch(void* fn, unsigned grid_x, unsigned grid_y, unsigned block_x, void* stream, void** args) {
  if (!fn || !args || !grid_x || !grid_y || !block_x) return KLAB_E_INVALID;
  Driver& d = driver();
  if (!d.ready) return KLAB_E_DRIVER;
  return d.launch(static_cast<CUfunction>(fn), grid_x, grid_y, 1, block_x, 1, 1, 0, static_cast<CUstream>(stream),
                  args, nullptr);
}

int lab_launch_ex(void* fn, unsigned grid_x, unsigned grid_y, unsigned block_x, unsigned smem_bytes,
                  unsigned flags, void* stream, void** args) {
  if (!fn || !args || !grid_x || !grid_y || !block_x) return KLAB_E_INVALID;
  Driver& d = driver();
  if (!d.ready || !d.launch_ex || !d.func_attribute) return KLAB_E_DRIVER;
  CUfunction f = static_cast<CUfunction>(fn);
  if (smem_bytes > 48 * 1024) {
    int status = d.func_attribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, static_cast<int>(smem_bytes));
    if (status) return status;
  }
  CUlaunchAttribute attr[1] = {};
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg = {};
  cfg.gridDimX = grid_x;
  cfg.gridDimY = grid_y;
  cfg.gridDimZ = 1;
  cfg.blockDimX = block_x;
  cfg.blockDimY = 1;
  cfg.blockDimZ = 1;
  cfg.sharedMemBytes = smem_bytes;
  cfg.hStream = static_cast<CUstream>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = (flags & 1u) ? 1 : 0;
  return d.launch_ex(&cfg, f, args, nullptr);
}

int lab_unload(void* module) {
  if (!module) return KLAB_E_INVALID;
  Driver& d = driver();
  if (!d.ready) return KLAB_E_DRIVER;
  return d.module_unload(static_cast<CUmodule>(module));
}

const char* lab_error_string(int code) {
  switch (code) {
    case KLAB_E_DRIVER: return "Cannot load CUDA driver or required symbols";
    case KLAB_E_NO_CONTEXT: return "No current CUDA context; initialize PyTorch CUDA first";
    case KLAB_E_INVALID: return "Invalid null argument or launch dimensions";
    default: {
      if (code < 0) return klab_error_string(code);
      Driver& d = driver();
      const char* message = nullptr;
      if (d.ready && d.error_string(static_cast<CUresult>(code), &message) == CUDA_SUCCESS && message)
        return message;
      return "Unknown CUDA error";
    }
  }
}

}  // extern "C"
