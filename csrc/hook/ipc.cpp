// CUDA IPC handles for region memory.
//
// cudaIpcGetMemHandle on memory that lives in a VMM region cannot use the
// driver's legacy IPC path (it only knows cuMemAlloc allocations). For region
// chunks the 64-byte handle instead carries {magic, exporter pid, POSIX fd of
// the physical allocation, original address, size, offset}; the importer
// duplicates the fd out of the exporter with pidfd_getfd (Linux >= 5.6) and
// maps the allocation at the exporter's address, so the pointer value is the
// same in both processes.
//
// Parity: reference csrc/hook.cpp:2864-3080. Difference by design: the
// reference passes the raw fd number, which is only meaningful inside the
// exporter's fd table (fork children); we transfer it with pidfd_getfd and fall
// back to the raw number only when that is unavailable.
#include <string.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <map>
#include <mutex>

#include "hook_internal.h"

using namespace fbh;

namespace {

constexpr uint32_t kMagic = 0x4D564246u;  // "FBVM"

#pragma pack(push, 1)
struct RegionIpcHandle {
  uint32_t magic;
  int32_t pid;
  int32_t fd;
  uint32_t _pad;
  uint64_t base;    // chunk base in the exporter
  uint64_t size;    // chunk size
  uint64_t offset;  // dptr - base
  uint8_t reserved[24];
};
#pragma pack(pop)
static_assert(sizeof(RegionIpcHandle) == CU_IPC_HANDLE_SIZE, "IPC handle must be 64 bytes");

struct Imported {
  uint64_t base;
  uint64_t size;
  CUmemGenericAllocationHandle handle;
  int refs;
};
std::mutex g_mu;
std::map<uint64_t, Imported> g_imported;  // base -> mapping

int dup_from_peer(int pid, int fd) {
#if defined(SYS_pidfd_open) && defined(SYS_pidfd_getfd)
  int pidfd = static_cast<int>(syscall(SYS_pidfd_open, pid, 0));
  if (pidfd >= 0) {
    int local = static_cast<int>(syscall(SYS_pidfd_getfd, pidfd, fd, 0));
    close(pidfd);
    if (local >= 0) return local;
  }
#endif
  return pid == getpid() ? dup(fd) : fd;
}

}  // namespace

extern "C" {

CUresult cuIpcGetMemHandle(CUipcMemHandle* pHandle, CUdeviceptr dptr) {
  CUdeviceptr base = 0;
  size_t size = 0;
  CUmemGenericAllocationHandle h = 0;
  if (!region_lookup_chunk(dptr, &base, &size, &h) || !h)
    return FB_CALL(cuIpcGetMemHandle, pHandle, dptr);
  int fd = -1;
  CUresult rc = FB_CALL(cuMemExportToShareableHandle, &fd, h,
                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (rc != CUDA_SUCCESS) return rc;
  RegionIpcHandle rh;
  memset(&rh, 0, sizeof(rh));
  rh.magic = kMagic;
  rh.pid = getpid();
  rh.fd = fd;
  rh.base = base;
  rh.size = size;
  rh.offset = dptr - base;
  memcpy(pHandle->reserved, &rh, sizeof(rh));
  return CUDA_SUCCESS;
}

CUresult cuIpcOpenMemHandle_v2(CUdeviceptr* pdptr, CUipcMemHandle handle, unsigned int Flags) {
  RegionIpcHandle rh;
  memcpy(&rh, handle.reserved, sizeof(rh));
  if (rh.magic != kMagic) return FB_CALL(cuIpcOpenMemHandle, pdptr, handle, Flags);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_imported.find(rh.base);
  if (it != g_imported.end()) {
    it->second.refs++;
    *pdptr = static_cast<CUdeviceptr>(rh.base + rh.offset);
    return CUDA_SUCCESS;
  }
  int fd = dup_from_peer(rh.pid, rh.fd);
  CUmemGenericAllocationHandle h = 0;
  CUresult rc = FB_CALL(cuMemImportFromShareableHandle, &h,
                        reinterpret_cast<void*>(static_cast<intptr_t>(fd)),
                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
  if (fd != rh.fd || rh.pid != getpid()) close(fd);
  if (rc != CUDA_SUCCESS) return rc;
  CUdeviceptr va = 0;
  rc = FB_CALL(cuMemAddressReserve, &va, rh.size, 0, static_cast<CUdeviceptr>(rh.base), 0);
  if (rc != CUDA_SUCCESS || va != rh.base) {
    if (rc == CUDA_SUCCESS) FB_CALL(cuMemAddressFree, va, rh.size);
    FB_CALL(cuMemRelease, h);
    return rc == CUDA_SUCCESS ? CUDA_ERROR_INVALID_VALUE : rc;
  }
  rc = FB_CALL(cuMemMap, va, rh.size, 0, h, 0);
  if (rc == CUDA_SUCCESS) {
    CUdevice dev = 0;
    FB_CALL(cuCtxGetDevice, &dev);
    CUmemAccessDesc d;
    memset(&d, 0, sizeof(d));
    d.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    d.location.id = dev;
    d.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    rc = FB_CALL(cuMemSetAccess, va, rh.size, &d, 1);
    if (rc != CUDA_SUCCESS) FB_CALL(cuMemUnmap, va, rh.size);
  }
  if (rc != CUDA_SUCCESS) {
    FB_CALL(cuMemAddressFree, va, rh.size);
    FB_CALL(cuMemRelease, h);
    return rc;
  }
  g_imported[rh.base] = Imported{rh.base, rh.size, h, 1};
  *pdptr = static_cast<CUdeviceptr>(rh.base + rh.offset);
  return CUDA_SUCCESS;
}

CUresult cuIpcCloseMemHandle(CUdeviceptr dptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto it = g_imported.begin(); it != g_imported.end(); ++it) {
    Imported& im = it->second;
    if (dptr < im.base || dptr >= im.base + im.size) continue;
    if (--im.refs > 0) return CUDA_SUCCESS;
    FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(im.base), im.size);
    FB_CALL(cuMemAddressFree, static_cast<CUdeviceptr>(im.base), im.size);
    FB_CALL(cuMemRelease, im.handle);
    g_imported.erase(it);
    return CUDA_SUCCESS;
  }
  return FB_CALL(cuIpcCloseMemHandle, dptr);
}

}  // extern "C"
