// Kernels from a committed sm_100a cubin, loaded through the CUDA driver API: the counterpart of the reference
// engine's embedded code objects (kernels/embed.go:7-10) loaded by its own driver (internal/kfd/kernel.go:58,
// LoadCodeObject). lfm3a_load_cubin loads the image into the current device's primary context; from then on every
// library launch on that device (launch_pdl) resolves its kernel in the loaded module by the kernel's mangled name
// (cudaFuncGetName) and launches it with cuLaunchKernelEx, with the same programmatic-serialisation attribute.
// The driver entry points come from cudaGetDriverEntryPoint, so the library does not link libcuda itself (it
// still loads on a host without a driver). The module's own device globals (the error word, the wait limit) are
// found by name, so lfm3a_sync and lfm3a_set_wait_limit reach them as well as the library's.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"

namespace lfm3a {

struct DriverApi {
  CUresult (*module_load_data)(CUmodule*, const void*) = nullptr;
  CUresult (*module_unload)(CUmodule) = nullptr;
  CUresult (*module_get_function)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*module_get_global)(CUdeviceptr*, size_t*, CUmodule, const char*) = nullptr;
  CUresult (*launch_kernel_ex)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
  CUresult (*func_set_attribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*func_get_attribute)(int*, CUfunction_attribute, CUfunction) = nullptr;
  bool ok = false;
};

// One loaded module per device.
struct ModuleSlot {
  std::mutex mu;
  CUmodule mod = nullptr;
  std::unordered_map<const void*, CUfunction> fns;
  CUdeviceptr error_word = 0, wait_limit = 0;
  std::atomic<long long> launches{0};
};

constexpr int kMaxDevices = 64;
inline ModuleSlot g_modules[kMaxDevices];
inline std::atomic<int> g_modules_loaded{0};     // any device with a module (a fast path for the common case)
inline thread_local CUresult g_module_result = CUDA_SUCCESS;   // the last module launch's result on this thread
inline thread_local std::string g_module_what;

inline const DriverApi& driver_api() {
  static DriverApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name, void** fn) {
      cudaDriverEntryPointQueryResult q;
      return cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) == cudaSuccess &&
             q == cudaDriverEntryPointSuccess && *fn != nullptr;
    };
    bool ok = get("cuModuleLoadData", reinterpret_cast<void**>(&api.module_load_data));
    ok = get("cuModuleUnload", reinterpret_cast<void**>(&api.module_unload)) && ok;
    ok = get("cuModuleGetFunction", reinterpret_cast<void**>(&api.module_get_function)) && ok;
    ok = get("cuModuleGetGlobal", reinterpret_cast<void**>(&api.module_get_global)) && ok;
    ok = get("cuLaunchKernelEx", reinterpret_cast<void**>(&api.launch_kernel_ex)) && ok;
    ok = get("cuFuncSetAttribute", reinterpret_cast<void**>(&api.func_set_attribute)) && ok;
    ok = get("cuFuncGetAttribute", reinterpret_cast<void**>(&api.func_get_attribute)) && ok;
    api.ok = ok;
    if (!ok) cudaGetLastError();
  });
  return api;
}

inline ModuleSlot* current_module() {
  if (g_modules_loaded.load(std::memory_order_acquire) == 0) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  ModuleSlot& m = g_modules[dev];
  return m.mod ? &m : nullptr;
}

// The module's function for a kernel of this library (by its mangled name), with the dynamic shared-memory limit
// raised to the device's opt-in maximum and the whole unified L1 / shared storage preferred as shared memory, as
// the library sets them on its own kernels.
inline CUfunction module_function(ModuleSlot& m, const void* kernel) {
  std::lock_guard<std::mutex> lock(m.mu);
  auto it = m.fns.find(kernel);
  if (it != m.fns.end()) return it->second;
  const DriverApi& api = driver_api();
  const char* name = nullptr;
  if (cudaFuncGetName(&name, kernel) != cudaSuccess || !name) {
    cudaGetLastError();
    g_module_what = "cudaFuncGetName";
    return nullptr;
  }
  CUfunction f = nullptr;
  CUresult r = api.module_get_function(&f, m.mod, name);
  if (r != CUDA_SUCCESS) {
    g_module_result = r;
    g_module_what = std::string("cuModuleGetFunction(") + name + ")";
    return nullptr;
  }
  int static_smem = 0, optin = 0, dev = 0;
  api.func_get_attribute(&static_smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, f);
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  api.func_set_attribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, optin - static_smem);
  api.func_set_attribute(f, CU_FUNC_ATTRIBUTE_PREFERRED_SHARED_MEMORY_CARVEOUT, 100);
  m.fns.emplace(kernel, f);
  return f;
}

bool module_launch(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** params) {
  ModuleSlot* m = current_module();
  if (!m) return false;
  CUfunction f = module_function(*m, kernel);
  if (!f) {
    if (g_module_result == CUDA_SUCCESS) g_module_result = CUDA_ERROR_NOT_FOUND;
    return true;
  }
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg = {};
  cfg.gridDimX = grid.x;
  cfg.gridDimY = grid.y;
  cfg.gridDimZ = grid.z;
  cfg.blockDimX = block.x;
  cfg.blockDimY = block.y;
  cfg.blockDimZ = block.z;
  cfg.sharedMemBytes = (unsigned)smem;
  cfg.hStream = reinterpret_cast<CUstream>(st);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const CUresult r = driver_api().launch_kernel_ex(&cfg, f, params, nullptr);
  if (r != CUDA_SUCCESS) {
    g_module_result = r;
    g_module_what = "cuLaunchKernelEx";
  } else {
    m->launches.fetch_add(1, std::memory_order_relaxed);
  }
  return true;
}

}  // namespace lfm3a
