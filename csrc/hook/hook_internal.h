// Internal declarations shared by the translation units of libfoundry_hook.
#pragma once

#include <cstdint>
#include <utility>
#include <vector>

#include <cuda.h>

#include <cstdint>
#include <string>

#include "../common/fb_driver.h"
#include "../common/fb_hook_api.h"

namespace fbh {

using RealDlsym = void* (*)(void*, const char*);
RealDlsym real_dlsym();

fb_status drv_error(CUresult r, const char* what);
bool debug_enabled();

// Region internals used by the interposed entry points.
// Returns true and fills *out if the region for the current device served the
// request; false means "not handled, call the real driver".
bool region_try_alloc(size_t size, CUdeviceptr* out, CUresult* result);
// True when the current device has an enabled (not stopped) region.
bool region_active_for_current();
bool region_try_free(CUdeviceptr ptr, CUresult* result);
bool region_try_reserve(CUdeviceptr* ptr, size_t size, size_t alignment, CUdeviceptr addr,
                        CUresult* result);
bool region_try_address_free(CUdeviceptr ptr, size_t size, CUresult* result);
// Looks up the physical allocation backing ptr (for IPC export).
bool region_lookup_chunk(CUdeviceptr ptr, CUdeviceptr* base, size_t* size,
                         CUmemGenericAllocationHandle* handle);

// Registry hooks called after a successful real load by a foreign caller.
// Scalar load options of a foreign image (JIT options and library options
// whose value is passed by value); pointer and output options are not kept.
struct LoadOptions {
  std::vector<std::pair<int, uint64_t>> jit, lib;
};
LoadOptions capture_load_options(unsigned int num_jit, const CUjit_option* jit, void* const* jit_values,
                                 unsigned int num_lib, const CUlibraryOption* lib, void* const* lib_values);
void registry_on_library_loaded(CUlibrary lib, const void* code, const char* tag, const LoadOptions& opts);
void registry_on_module_loaded(CUmodule mod, const void* code, const char* tag, const LoadOptions& opts);
void registry_on_library_file_loaded(CUlibrary lib, const char* path);
void registry_on_module_file_loaded(CUmodule mod, const char* path);
bool registry_in_own_load();  // true while fb_registry_load_image runs on this thread

extern bool g_preloaded;
}  // namespace fbh
