// LD_PRELOAD interposer: exported overrides of the driver entry points that
// allocate memory, load code, or exchange IPC handles, plus dlsym and
// cuGetProcAddress so cudart's entry-point lookups return the overrides.
//
// Parity: reference csrc/hook.cpp:1828-3081 (22 overrides), 2149-2244
// (cuGetProcAddress routing), 2806-2856 (dlsym). IPC (2864-3080) is in ipc.cpp.
//
// Known limitation, same as any dlsym interposer: dlsym(RTLD_NEXT, ...) calls
// made by other libraries are answered relative to this library.
#include <dlfcn.h>
#include <string.h>

#include <string>
#include <unordered_map>

#include "hook_internal.h"

// The header maps cuGetProcAddress onto the _v2 export; we export both.
#undef cuGetProcAddress

using namespace fbh;

extern "C" {
// Forward declarations of our overrides (defined below / in ipc.cpp).
CUresult cuMemAlloc_v2(CUdeviceptr* dptr, size_t bytesize);
CUresult cuMemFree_v2(CUdeviceptr dptr);
CUresult cuMemAllocPitch_v2(CUdeviceptr* dptr, size_t* pPitch, size_t WidthInBytes, size_t Height,
                            unsigned int ElementSizeBytes);
CUresult cuMemAddressReserve(CUdeviceptr* ptr, size_t size, size_t alignment, CUdeviceptr addr,
                             unsigned long long flags);
CUresult cuMemAddressFree(CUdeviceptr ptr, size_t size);
CUresult cuLibraryLoadData(CUlibrary* library, const void* code, CUjit_option* jitOptions,
                           void** jitOptionsValues, unsigned int numJitOptions,
                           CUlibraryOption* libraryOptions, void** libraryOptionValues,
                           unsigned int numLibraryOptions);
CUresult cuLibraryLoadFromFile(CUlibrary* library, const char* fileName, CUjit_option* jitOptions,
                               void** jitOptionsValues, unsigned int numJitOptions,
                               CUlibraryOption* libraryOptions, void** libraryOptionValues,
                               unsigned int numLibraryOptions);
CUresult cuModuleLoadData(CUmodule* module, const void* image);
CUresult cuModuleLoadDataEx(CUmodule* module, const void* image, unsigned int numOptions,
                            CUjit_option* options, void** optionValues);
CUresult cuModuleLoadFatBinary(CUmodule* module, const void* fatCubin);
CUresult cuModuleLoad(CUmodule* module, const char* fname);
CUresult cuIpcGetMemHandle(CUipcMemHandle* pHandle, CUdeviceptr dptr);
CUresult cuIpcOpenMemHandle_v2(CUdeviceptr* pdptr, CUipcMemHandle handle, unsigned int Flags);
CUresult cuIpcCloseMemHandle(CUdeviceptr dptr);
CUresult cuGetProcAddress_v2(const char* symbol, void** pfn, int cudaVersion, cuuint64_t flags,
                             CUdriverProcAddressQueryResult* symbolStatus);
CUresult cuGetProcAddress(const char* symbol, void** pfn, int cudaVersion, cuuint64_t flags);
void* dlsym(void* handle, const char* symbol);
}

namespace {

// Base name (as cudart asks cuGetProcAddress) -> our override.
const std::unordered_map<std::string, void*>& base_overrides() {
  static const std::unordered_map<std::string, void*> m = {
      {"cuMemAlloc", reinterpret_cast<void*>(&cuMemAlloc_v2)},
      {"cuMemFree", reinterpret_cast<void*>(&cuMemFree_v2)},
      {"cuMemAllocPitch", reinterpret_cast<void*>(&cuMemAllocPitch_v2)},
      {"cuMemAddressReserve", reinterpret_cast<void*>(&cuMemAddressReserve)},
      {"cuMemAddressFree", reinterpret_cast<void*>(&cuMemAddressFree)},
      {"cuLibraryLoadData", reinterpret_cast<void*>(&cuLibraryLoadData)},
      {"cuLibraryLoadFromFile", reinterpret_cast<void*>(&cuLibraryLoadFromFile)},
      {"cuModuleLoadData", reinterpret_cast<void*>(&cuModuleLoadData)},
      {"cuModuleLoadDataEx", reinterpret_cast<void*>(&cuModuleLoadDataEx)},
      {"cuModuleLoadFatBinary", reinterpret_cast<void*>(&cuModuleLoadFatBinary)},
      {"cuModuleLoad", reinterpret_cast<void*>(&cuModuleLoad)},
      {"cuIpcGetMemHandle", reinterpret_cast<void*>(&cuIpcGetMemHandle)},
      {"cuIpcOpenMemHandle", reinterpret_cast<void*>(&cuIpcOpenMemHandle_v2)},
      {"cuIpcCloseMemHandle", reinterpret_cast<void*>(&cuIpcCloseMemHandle)},
      {"cuGetProcAddress", reinterpret_cast<void*>(&cuGetProcAddress_v2)},
  };
  return m;
}

// Exported (versioned) symbol name -> our override, for dlsym.
const std::unordered_map<std::string, void*>& symbol_overrides() {
  static const std::unordered_map<std::string, void*> m = {
      {"cuMemAlloc_v2", reinterpret_cast<void*>(&cuMemAlloc_v2)},
      {"cuMemFree_v2", reinterpret_cast<void*>(&cuMemFree_v2)},
      {"cuMemAllocPitch_v2", reinterpret_cast<void*>(&cuMemAllocPitch_v2)},
      {"cuMemAddressReserve", reinterpret_cast<void*>(&cuMemAddressReserve)},
      {"cuMemAddressFree", reinterpret_cast<void*>(&cuMemAddressFree)},
      {"cuLibraryLoadData", reinterpret_cast<void*>(&cuLibraryLoadData)},
      {"cuLibraryLoadFromFile", reinterpret_cast<void*>(&cuLibraryLoadFromFile)},
      {"cuModuleLoadData", reinterpret_cast<void*>(&cuModuleLoadData)},
      {"cuModuleLoadDataEx", reinterpret_cast<void*>(&cuModuleLoadDataEx)},
      {"cuModuleLoadFatBinary", reinterpret_cast<void*>(&cuModuleLoadFatBinary)},
      {"cuModuleLoad", reinterpret_cast<void*>(&cuModuleLoad)},
      {"cuIpcGetMemHandle", reinterpret_cast<void*>(&cuIpcGetMemHandle)},
      {"cuIpcOpenMemHandle_v2", reinterpret_cast<void*>(&cuIpcOpenMemHandle_v2)},
      {"cuIpcOpenMemHandle", reinterpret_cast<void*>(&cuIpcOpenMemHandle_v2)},
      {"cuIpcCloseMemHandle", reinterpret_cast<void*>(&cuIpcCloseMemHandle)},
      {"cuGetProcAddress_v2", reinterpret_cast<void*>(&cuGetProcAddress_v2)},
      {"cuGetProcAddress", reinterpret_cast<void*>(&cuGetProcAddress)},
  };
  return m;
}

__attribute__((constructor)) void fb_hook_ctor() {
  // Preloaded iff our dlsym is the one the global scope resolves.
  void* global = reinterpret_cast<void*>(real_dlsym()(RTLD_DEFAULT, "dlsym"));
  g_preloaded = (global == reinterpret_cast<void*>(&dlsym));
}

}  // namespace

extern "C" {

int fb_hook_is_preloaded(void) { return g_preloaded ? 1 : 0; }

CUresult cuMemAlloc_v2(CUdeviceptr* dptr, size_t bytesize) {
  CUresult rc;
  if (region_try_alloc(bytesize, dptr, &rc)) return rc;
  return FB_CALL(cuMemAlloc, dptr, bytesize);
}

CUresult cuMemFree_v2(CUdeviceptr dptr) {
  CUresult rc;
  if (region_try_free(dptr, &rc)) return rc;
  return FB_CALL(cuMemFree, dptr);
}

// Pitched 2-D allocation inside the region. The pitch is chosen here, not by
// a throw-away driver allocation: the row width rounded up to the device's
// texture pitch alignment (at least 128 bytes), so a 2-D texture can be bound
// to the rows and SAVE and LOAD get the same pitch and the same address.
// Outside an active region the driver's own call runs.
CUresult cuMemAllocPitch_v2(CUdeviceptr* dptr, size_t* pPitch, size_t WidthInBytes, size_t Height,
                            unsigned int ElementSizeBytes) {
  if (!dptr || !pPitch || WidthInBytes == 0 || Height == 0 ||
      (ElementSizeBytes != 4 && ElementSizeBytes != 8 && ElementSizeBytes != 16))
    return CUDA_ERROR_INVALID_VALUE;
  if (region_active_for_current()) {
    size_t align = 128;
    CUdevice dev = 0;
    int attr = 0;
    if (FB_CALL(cuCtxGetDevice, &dev) == CUDA_SUCCESS &&
        FB_CALL(cuDeviceGetAttribute, &attr, CU_DEVICE_ATTRIBUTE_TEXTURE_PITCH_ALIGNMENT, dev) == CUDA_SUCCESS &&
        attr > static_cast<int>(align))
      align = static_cast<size_t>(attr);
    const size_t pitch = (WidthInBytes + align - 1) / align * align;
    CUresult rc;
    if (region_try_alloc(pitch * Height, dptr, &rc)) {
      if (rc == CUDA_SUCCESS) *pPitch = pitch;
      return rc;
    }
  }
  return FB_CALL(cuMemAllocPitch, dptr, pPitch, WidthInBytes, Height, ElementSizeBytes);
}

CUresult cuMemAddressReserve(CUdeviceptr* ptr, size_t size, size_t alignment, CUdeviceptr addr,
                             unsigned long long flags) {
  CUresult rc;
  if (region_try_reserve(ptr, size, alignment, addr, &rc)) return rc;
  return FB_CALL(cuMemAddressReserve, ptr, size, alignment, addr, flags);
}

CUresult cuMemAddressFree(CUdeviceptr ptr, size_t size) {
  CUresult rc;
  if (region_try_address_free(ptr, size, &rc)) return rc;
  return FB_CALL(cuMemAddressFree, ptr, size);
}

CUresult cuLibraryLoadData(CUlibrary* library, const void* code, CUjit_option* jitOptions,
                           void** jitOptionsValues, unsigned int numJitOptions,
                           CUlibraryOption* libraryOptions, void** libraryOptionValues,
                           unsigned int numLibraryOptions) {
  CUresult rc = FB_CALL(cuLibraryLoadData, library, code, jitOptions, jitOptionsValues,
                        numJitOptions, libraryOptions, libraryOptionValues, numLibraryOptions);
  if (rc == CUDA_SUCCESS && !registry_in_own_load())
    registry_on_library_loaded(*library, code, "cuLibraryLoadData",
                               capture_load_options(numJitOptions, jitOptions, jitOptionsValues, numLibraryOptions,
                                                    libraryOptions, libraryOptionValues));
  return rc;
}

CUresult cuLibraryLoadFromFile(CUlibrary* library, const char* fileName, CUjit_option* jitOptions,
                               void** jitOptionsValues, unsigned int numJitOptions,
                               CUlibraryOption* libraryOptions, void** libraryOptionValues,
                               unsigned int numLibraryOptions) {
  CUresult rc = FB_CALL(cuLibraryLoadFromFile, library, fileName, jitOptions, jitOptionsValues,
                        numJitOptions, libraryOptions, libraryOptionValues, numLibraryOptions);
  if (rc == CUDA_SUCCESS) registry_on_library_file_loaded(*library, fileName);
  return rc;
}

CUresult cuModuleLoadData(CUmodule* module, const void* image) {
  CUresult rc = FB_CALL(cuModuleLoadData, module, image);
  if (rc == CUDA_SUCCESS) registry_on_module_loaded(*module, image, "cuModuleLoadData", LoadOptions{});
  return rc;
}

CUresult cuModuleLoadDataEx(CUmodule* module, const void* image, unsigned int numOptions,
                            CUjit_option* options, void** optionValues) {
  CUresult rc = FB_CALL(cuModuleLoadDataEx, module, image, numOptions, options, optionValues);
  if (rc == CUDA_SUCCESS)
    registry_on_module_loaded(*module, image, "cuModuleLoadDataEx",
                              capture_load_options(numOptions, options, optionValues, 0, nullptr, nullptr));
  return rc;
}

CUresult cuModuleLoadFatBinary(CUmodule* module, const void* fatCubin) {
  CUresult rc = FB_CALL(cuModuleLoadFatBinary, module, fatCubin);
  if (rc == CUDA_SUCCESS) registry_on_module_loaded(*module, fatCubin, "cuModuleLoadFatBinary", LoadOptions{});
  return rc;
}

CUresult cuModuleLoad(CUmodule* module, const char* fname) {
  CUresult rc = FB_CALL(cuModuleLoad, module, fname);
  if (rc == CUDA_SUCCESS) registry_on_module_file_loaded(*module, fname);
  return rc;
}

CUresult cuGetProcAddress_v2(const char* symbol, void** pfn, int cudaVersion, cuuint64_t flags,
                             CUdriverProcAddressQueryResult* symbolStatus) {
  CUresult rc = FB_CALL(cuGetProcAddress_v2, symbol, pfn, cudaVersion, flags, symbolStatus);
  if (rc != CUDA_SUCCESS || !symbol || !pfn || !*pfn) return rc;
  const auto& m = base_overrides();
  auto it = m.find(symbol);
  if (it != m.end()) {
    // Only the versions we implement: modern cuMemAlloc/cuMemFree (_v2) and
    // cuIpcOpenMemHandle (_v2); older callers keep the driver's function.
    std::string s(symbol);
    if ((s == "cuMemAlloc" || s == "cuMemFree" || s == "cuMemAllocPitch") && cudaVersion < 3020) return rc;
    if (s == "cuIpcOpenMemHandle" && cudaVersion < 11000) return rc;
    if (s == "cuGetProcAddress" && cudaVersion < 12000)
      *pfn = reinterpret_cast<void*>(&cuGetProcAddress);
    else
      *pfn = it->second;
  }
  return rc;
}

CUresult cuGetProcAddress(const char* symbol, void** pfn, int cudaVersion, cuuint64_t flags) {
  return cuGetProcAddress_v2(symbol, pfn, cudaVersion, flags, nullptr);
}

void* dlsym(void* handle, const char* symbol) {
  RealDlsym real = real_dlsym();
  if (symbol && symbol[0] == 'c' && symbol[1] == 'u') {
    const auto& m = symbol_overrides();
    auto it = m.find(symbol);
    if (it != m.end()) {
      // Only redirect lookups that would have found the driver's symbol.
      void* orig = real(handle, symbol);
      if (orig) return it->second;
    }
  }
  return real(handle, symbol);
}

}  // extern "C"
