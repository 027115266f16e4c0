// Function table of the CUDA driver API as seen by foundry_b200.
//
// Nothing in foundry_b200 links libcuda directly. The hook library resolves
// the *real* driver once (libcuda.so.1, or the library named by the
// FOUNDRY_CUDA_DRIVER environment variable, which is how the CPU-only mock
// driver is plugged in for tests) and every native component calls through
// this table. That keeps the interposer's own calls from re-entering its
// overrides and lets the whole stack run against the mock on a CPU box.
//
// Parity: the reference resolves 43 driver entry points into an indexed table
// (csrc/hook.cpp:40-130, 1732-1808). This table is our own list of what our
// components use; symbol names are the exported (versioned) ones.
#pragma once

#include <cuda.h>

#include <cstdint>

#define FB_STR2(x) #x
#define FB_STR(x) FB_STR2(x)

// X(header_name): header_name is the name as written in code; it may be a
// macro that cuda.h maps onto a versioned export (cuMemAlloc -> cuMemAlloc_v2),
// so FB_STR(header_name) yields the exported symbol to dlsym.
#define FB_DRIVER_FUNCS(X)                 \
  X(cuInit)                                \
  X(cuDriverGetVersion)                    \
  X(cuGetErrorString)                      \
  X(cuGetErrorName)                        \
  X(cuDeviceGet)                           \
  X(cuDeviceGetCount)                      \
  X(cuDeviceGetAttribute)                  \
  X(cuDevicePrimaryCtxRetain)              \
  X(cuCtxGetCurrent)                       \
  X(cuCtxSetCurrent)                       \
  X(cuCtxGetDevice)                        \
  X(cuCtxSynchronize)                      \
  X(cuMemAlloc)                            \
  X(cuMemFree)                             \
  X(cuMemAllocPitch)                       \
  X(cuMemGetInfo)                          \
  X(cuMemAddressReserve)                   \
  X(cuMemAddressFree)                      \
  X(cuMemCreate)                           \
  X(cuMemRelease)                          \
  X(cuMemMap)                              \
  X(cuMemUnmap)                            \
  X(cuMemSetAccess)                        \
  X(cuMemGetAllocationGranularity)         \
  X(cuMemExportToShareableHandle)          \
  X(cuMemImportFromShareableHandle)        \
  X(cuMemGetAddressRange)                  \
  X(cuMemcpyHtoD)                          \
  X(cuMemcpyDtoH)                          \
  X(cuMemsetD8)                            \
  X(cuMulticastCreate)                     \
  X(cuMulticastAddDevice)                  \
  X(cuMulticastBindMem)                    \
  X(cuMulticastUnbind)                     \
  X(cuMulticastGetGranularity)             \
  X(cuModuleLoadData)                      \
  X(cuModuleLoadDataEx)                    \
  X(cuModuleLoadFatBinary)                 \
  X(cuModuleLoad)                          \
  X(cuModuleUnload)                        \
  X(cuModuleGetFunction)                   \
  X(cuModuleGetGlobal)                     \
  X(cuModuleGetFunctionCount)              \
  X(cuModuleEnumerateFunctions)            \
  X(cuLibraryLoadData)                     \
  X(cuLibraryLoadFromFile)                 \
  X(cuLibraryUnload)                       \
  X(cuLibraryGetKernel)                    \
  X(cuLibraryGetKernelCount)               \
  X(cuLibraryEnumerateKernels)             \
  X(cuLibraryGetModule)                    \
  X(cuLibraryGetGlobal)                    \
  X(cuKernelGetFunction)                   \
  X(cuKernelGetName)                       \
  X(cuKernelGetLibrary)                    \
  X(cuKernelSetAttribute)                  \
  X(cuFuncGetName)                         \
  X(cuFuncGetModule)                       \
  X(cuFuncSetAttribute)                    \
  X(cuFuncGetAttribute)                    \
  X(cuFuncGetParamInfo)                    \
  X(cuLaunchKernelEx)                      \
  X(cuTensorMapEncodeTiled)                \
  X(cuStreamSynchronize)                   \
  X(cuStreamIsCapturing)                   \
  X(cuEventCreate)                         \
  X(cuEventDestroy)                        \
  X(cuGraphCreate)                         \
  X(cuGraphDestroy)                        \
  X(cuGraphGetNodes)                       \
  X(cuGraphGetEdges)                       \
  X(cuGraphGetEdges_v2)                    \
  X(cuGraphNodeGetType)                    \
  X(cuGraphKernelNodeGetParams)            \
  X(cuGraphKernelNodeGetAttribute)         \
  X(cuGraphKernelNodeSetAttribute)         \
  X(cuGraphMemsetNodeGetParams)            \
  X(cuGraphMemcpyNodeGetParams)            \
  X(cuGraphEventRecordNodeGetEvent)        \
  X(cuGraphEventWaitNodeGetEvent)          \
  X(cuGraphAddKernelNode)                  \
  X(cuGraphAddMemsetNode)                  \
  X(cuGraphAddMemcpyNode)                  \
  X(cuGraphAddEmptyNode)                   \
  X(cuGraphAddEventRecordNode)             \
  X(cuGraphAddEventWaitNode)               \
  X(cuGraphAddDependencies)                \
  X(cuGraphAddDependencies_v2)             \
  X(cuGraphInstantiate)                    \
  X(cuGraphExecDestroy)                    \
  X(cuGraphLaunch)                         \
  X(cuGraphExecKernelNodeSetParams)        \
  X(cuGraphExecMemsetNodeSetParams)        \
  X(cuGraphExecMemcpyNodeSetParams)        \
  X(cuGetProcAddress)                      \
  X(cuIpcGetMemHandle)                     \
  X(cuIpcOpenMemHandle)                    \
  X(cuIpcCloseMemHandle)                   \
  X(cuPointerGetAttribute)

struct FbDriver {
#define FB_DECL(name) decltype(&::name) name = nullptr;
  FB_DRIVER_FUNCS(FB_DECL)
#undef FB_DECL
  void* handle = nullptr;   // dlopen handle of the real driver
  bool loaded = false;      // the driver library was found
  bool is_mock = false;     // the mock driver (exports fbmock_is_mock)
};

#ifdef __cplusplus
extern "C" {
#endif
// Returns the process-wide table. Resolved lazily on first call; safe to call
// from any thread. Members are null if the driver (or a symbol) is missing.
const FbDriver* fb_driver(void);
// Name of the library that was (or will be) opened as the real driver.
const char* fb_driver_path(void);
#ifdef __cplusplus
}
#endif

// Call a driver function, returning CUDA_ERROR_NOT_INITIALIZED if the symbol
// is unavailable (CPU box without a driver, or an old driver).
#define FB_CALL(fn, ...) \
  (fb_driver()->fn ? fb_driver()->fn(__VA_ARGS__) : CUDA_ERROR_NOT_INITIALIZED)
