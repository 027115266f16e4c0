// libfoundry_mockcuda.so: a CPU-only stand-in for the subset of the CUDA
// driver API that foundry_b200's native layers use. Tests point
// FOUNDRY_CUDA_DRIVER at this library so the region, registry, graph
// analysis, archive writer/reader and restore engine run end to end on a box
// without a GPU.
//
// Model:
//  * "device memory" is host memory. cuMemAddressReserve reserves address
//    space with mmap(PROT_NONE) at the requested address; cuMemCreate makes a
//    memfd; cuMemMap maps it MAP_SHARED|MAP_FIXED; cuMemSetAccess mprotects.
//    Addresses therefore behave exactly like VMM addresses (fixed, shareable).
//  * a code image is a blob that starts with the header
//        "FBMOCK\n" { "<entry>:<param sizes comma separated>\n" | "@<global>:<bytes>\n" }* "\n"
//    followed by arbitrary payload bytes (tests append 1 MB of random data).
//  * graphs are node lists with edges; launching a graph (or a kernel) runs
//    the built-in host implementation of the entry point when it has one
//    (fbmock_axpy_f32, fbmock_fill_u32, fbmock_scale_add_f32), else does
//    nothing. Kernel params are deep-copied with their declared sizes.
// The mock is intentionally strict: unknown handles return
// CUDA_ERROR_INVALID_HANDLE, so host-side bugs surface as statuses.
// It has no counterpart in the reference, whose tests use no fakes.
#include <cuda.h>
#include <dlfcn.h>
#include <string.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#undef cuGetProcAddress

namespace {

std::recursive_mutex g_mu;
constexpr size_t kGran = 2ull << 20;

struct MockCtx {
  int device;
};
MockCtx g_ctx0{0};
thread_local CUcontext t_current = nullptr;
bool g_inited = false;

struct PhysAlloc {
  int fd;
  size_t size;
  int refs;
};
std::map<uint64_t, std::unique_ptr<PhysAlloc>> g_phys;  // handle id -> allocation
uint64_t g_next_handle = 1;
std::map<uint64_t, size_t> g_reservations;  // base -> size
std::map<uint64_t, std::pair<uint64_t, size_t>> g_mappings;  // va -> (handle, size)
std::map<uint64_t, size_t> g_plain_allocs;  // cuMemAlloc blocks

struct MockFunc;
struct MockLib {
  std::vector<std::unique_ptr<MockFunc>> funcs;
  std::map<std::string, std::vector<uint8_t>> globals;  // "@name:size" lines: zeroed host storage
  int module_tag;  // address used as the CUmodule of this library
};
struct MockFunc {
  std::string name;
  std::vector<size_t> param_sizes;
  MockLib* lib;
  int attrs[16];
};
std::set<MockLib*> g_libs;
std::set<MockFunc*> g_funcs;
// Options of every image load, in order: "<loader> <key>=<value> ..." (tests
// check that a LOAD replays the options of the original load).
std::vector<std::string> g_load_log;

enum NodeKind { KERNEL, MEMSET, MEMCPY, EMPTY, EV_RECORD, EV_WAIT };
struct MockNode {
  NodeKind kind;
  MockFunc* fn = nullptr;
  CUDA_KERNEL_NODE_PARAMS kp{};
  std::vector<std::vector<uint8_t>> params;
  std::vector<void*> param_ptrs;
  CUDA_MEMSET_NODE_PARAMS ms{};
  CUDA_MEMCPY3D mc{};
  CUevent ev = nullptr;
  std::map<int, CUlaunchAttributeValue> attrs;
};
struct MockGraph {
  std::vector<std::unique_ptr<MockNode>> nodes;
  std::vector<std::pair<MockNode*, MockNode*>> edges;
  std::vector<CUgraphEdgeData> edge_data;  // parallel to edges
};
std::set<MockGraph*> g_graphs;
struct MockExec {
  std::unique_ptr<MockGraph> g;
  std::map<MockNode*, MockNode*> from_orig;  // original node -> exec copy
};
std::set<MockExec*> g_execs;
std::atomic<uint64_t> g_launches{0};

bool parse_image(const void* code, MockLib* lib) {
  const char* p = static_cast<const char*>(code);
  if (strncmp(p, "FBMOCK\n", 7) != 0) return false;
  p += 7;
  while (*p && *p != '\n') {
    const char* eol = strchr(p, '\n');
    if (!eol) return false;
    std::string line(p, eol);
    p = eol + 1;
    auto colon = line.find(':');
    if (!line.empty() && line[0] == '@') {
      const size_t n = colon == std::string::npos ? 8 : strtoull(line.c_str() + colon + 1, nullptr, 10);
      lib->globals[line.substr(1, colon == std::string::npos ? std::string::npos : colon - 1)].assign(n, 0);
      continue;
    }
    std::unique_ptr<MockFunc> f(new MockFunc());
    f->name = line.substr(0, colon);
    memset(f->attrs, 0, sizeof(f->attrs));
    if (colon != std::string::npos) {
      std::string sizes = line.substr(colon + 1);
      size_t pos = 0;
      while (pos < sizes.size()) {
        size_t c = sizes.find(',', pos);
        if (c == std::string::npos) c = sizes.size();
        f->param_sizes.push_back(strtoull(sizes.substr(pos, c - pos).c_str(), nullptr, 10));
        pos = c + 1;
      }
    }
    f->lib = lib;
    g_funcs.insert(f.get());
    lib->funcs.push_back(std::move(f));
  }
  return true;
}

MockFunc* as_func(const void* h) {
  auto* f = static_cast<MockFunc*>(const_cast<void*>(h));
  return g_funcs.count(f) ? f : nullptr;
}

void copy_params(MockNode& n, MockFunc* f, void** kernelParams) {
  n.params.clear();
  n.param_ptrs.clear();
  for (size_t i = 0; i < f->param_sizes.size(); ++i) {
    const uint8_t* src = static_cast<const uint8_t*>(kernelParams[i]);
    n.params.emplace_back(src, src + f->param_sizes[i]);
  }
  for (auto& p : n.params) n.param_ptrs.push_back(p.data());
  n.kp.kernelParams = n.param_ptrs.data();
}

template <typename T>
T param_as(void** params, int i) {
  T v;
  memcpy(&v, params[i], sizeof(T));
  return v;
}

void run_kernel(MockFunc* f, void** params) {
  g_launches++;
  if (f->name == "fbmock_axpy_f32") {  // (float* y, const float* x, float a, uint32 n)
    float* y = param_as<float*>(params, 0);
    const float* x = param_as<const float*>(params, 1);
    float a = param_as<float>(params, 2);
    uint32_t n = param_as<uint32_t>(params, 3);
    for (uint32_t i = 0; i < n; ++i) y[i] += a * x[i];
  } else if (f->name == "fbmock_fill_u32") {  // (uint32* p, uint32 v, uint32 n)
    uint32_t* p = param_as<uint32_t*>(params, 0);
    uint32_t v = param_as<uint32_t>(params, 1);
    uint32_t n = param_as<uint32_t>(params, 2);
    for (uint32_t i = 0; i < n; ++i) p[i] = v;
  } else if (f->name == "fbmock_scale_add_f32") {  // (float* out, const float* a, const float* b, float s, uint32 n)
    float* out = param_as<float*>(params, 0);
    const float* a = param_as<const float*>(params, 1);
    const float* b = param_as<const float*>(params, 2);
    float s = param_as<float>(params, 3);
    uint32_t n = param_as<uint32_t>(params, 4);
    for (uint32_t i = 0; i < n; ++i) out[i] = a[i] * s + b[i];
  }
}

void run_node(MockNode& n) {
  switch (n.kind) {
    case KERNEL: run_kernel(n.fn, n.kp.kernelParams); break;
    case MEMSET: {
      for (size_t r = 0; r < std::max<size_t>(n.ms.height, 1); ++r) {
        uint8_t* row = reinterpret_cast<uint8_t*>(n.ms.dst + r * n.ms.pitch);
        for (size_t i = 0; i < n.ms.width; ++i)
          memcpy(row + i * n.ms.elementSize, &n.ms.value, n.ms.elementSize);
      }
      break;
    }
    case MEMCPY: {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(n.mc.srcDevice) + n.mc.srcXInBytes;
      uint8_t* dst = reinterpret_cast<uint8_t*>(n.mc.dstDevice) + n.mc.dstXInBytes;
      memcpy(dst, src, n.mc.WidthInBytes * std::max<size_t>(n.mc.Height, 1));
      break;
    }
    default: break;
  }
}

// Topological order of a graph (Kahn); node insertion order breaks ties.
std::vector<MockNode*> topo(MockGraph& g) {
  std::map<MockNode*, int> indeg;
  for (auto& n : g.nodes) indeg[n.get()] = 0;
  for (auto& e : g.edges) indeg[e.second]++;
  std::vector<MockNode*> out;
  std::vector<bool> done(g.nodes.size(), false);
  while (out.size() < g.nodes.size()) {
    bool progressed = false;
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      MockNode* n = g.nodes[i].get();
      if (done[i] || indeg[n] != 0) continue;
      done[i] = true;
      out.push_back(n);
      for (auto& e : g.edges)
        if (e.first == n) indeg[e.second]--;
      progressed = true;
    }
    if (!progressed) break;
  }
  return out;
}

}  // namespace

extern "C" {

int fbmock_is_mock(void) { return 1; }
unsigned long long fbmock_launch_count(void) { return g_launches.load(); }

CUresult cuInit(unsigned int) {
  g_inited = true;
  return CUDA_SUCCESS;
}
CUresult cuDriverGetVersion(int* v) {
  *v = 12090;
  return CUDA_SUCCESS;
}
CUresult cuGetErrorString(CUresult e, const char** s) {
  static thread_local std::string buf;
  buf = "mock error " + std::to_string(static_cast<int>(e));
  *s = buf.c_str();
  return CUDA_SUCCESS;
}
CUresult cuGetErrorName(CUresult e, const char** s) { return cuGetErrorString(e, s); }
CUresult cuDeviceGet(CUdevice* d, int ordinal) {
  if (ordinal != 0) return CUDA_ERROR_INVALID_DEVICE;
  *d = 0;
  return CUDA_SUCCESS;
}
CUresult cuDeviceGetCount(int* c) {
  *c = 1;
  return CUDA_SUCCESS;
}
CUresult cuDeviceGetAttribute(int* v, CUdevice_attribute a, CUdevice) {
  switch (a) {
    case CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT: *v = 148; break;
    case CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR: *v = 10; break;
    case CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR: *v = 0; break;
    case CU_DEVICE_ATTRIBUTE_TEXTURE_PITCH_ALIGNMENT: *v = 32; break;
    default: *v = 0;
  }
  return CUDA_SUCCESS;
}
CUresult cuDevicePrimaryCtxRetain(CUcontext* c, CUdevice) {
  *c = reinterpret_cast<CUcontext>(&g_ctx0);
  return CUDA_SUCCESS;
}
CUresult cuCtxGetCurrent(CUcontext* c) {
  *c = t_current;
  return CUDA_SUCCESS;
}
CUresult cuCtxSetCurrent(CUcontext c) {
  t_current = c;
  return CUDA_SUCCESS;
}
CUresult cuCtxGetDevice(CUdevice* d) {
  if (!t_current) return CUDA_ERROR_INVALID_CONTEXT;
  *d = 0;
  return CUDA_SUCCESS;
}
CUresult cuCtxSynchronize(void) { return CUDA_SUCCESS; }

// ---- memory ------------------------------------------------------------------
CUresult cuMemAlloc_v2(CUdeviceptr* p, size_t n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  void* m = mmap(nullptr, n ? n : 1, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (m == MAP_FAILED) return CUDA_ERROR_OUT_OF_MEMORY;
  *p = reinterpret_cast<CUdeviceptr>(m);
  g_plain_allocs[*p] = n ? n : 1;
  return CUDA_SUCCESS;
}
CUresult cuMemFree_v2(CUdeviceptr p) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_plain_allocs.find(p);
  if (it == g_plain_allocs.end()) return CUDA_ERROR_INVALID_VALUE;
  munmap(reinterpret_cast<void*>(p), it->second);
  g_plain_allocs.erase(it);
  return CUDA_SUCCESS;
}
CUresult cuMemAllocPitch_v2(CUdeviceptr* p, size_t* pitch, size_t w, size_t h, unsigned int) {
  *pitch = (w + 511) / 512 * 512;
  return cuMemAlloc_v2(p, *pitch * h);
}
CUresult cuMemGetInfo_v2(size_t* free_b, size_t* total) {
  *free_b = 64ull << 30;
  *total = 64ull << 30;
  return CUDA_SUCCESS;
}
CUresult cuMemGetAllocationGranularity(size_t* g, const CUmemAllocationProp*,
                                       CUmemAllocationGranularity_flags) {
  *g = kGran;
  return CUDA_SUCCESS;
}
CUresult cuMemAddressReserve(CUdeviceptr* ptr, size_t size, size_t, CUdeviceptr addr,
                             unsigned long long) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int flags = MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE;
  if (addr) flags |= MAP_FIXED_NOREPLACE;
  void* m = mmap(reinterpret_cast<void*>(addr), size, PROT_NONE, flags, -1, 0);
  if (m == MAP_FAILED) {
    if (!addr) return CUDA_ERROR_OUT_OF_MEMORY;
    // Address in use: behave like the driver and pick another address.
    m = mmap(nullptr, size, PROT_NONE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    if (m == MAP_FAILED) return CUDA_ERROR_OUT_OF_MEMORY;
  }
  *ptr = reinterpret_cast<CUdeviceptr>(m);
  g_reservations[*ptr] = size;
  return CUDA_SUCCESS;
}
CUresult cuMemAddressFree(CUdeviceptr ptr, size_t size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_reservations.find(ptr);
  if (it == g_reservations.end() || it->second != size) return CUDA_ERROR_INVALID_VALUE;
  munmap(reinterpret_cast<void*>(ptr), size);
  g_reservations.erase(it);
  return CUDA_SUCCESS;
}
CUresult cuMemCreate(CUmemGenericAllocationHandle* h, size_t size, const CUmemAllocationProp*,
                     unsigned long long) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (size % kGran) return CUDA_ERROR_INVALID_VALUE;
  int fd = memfd_create("fbmock", 0);
  if (fd < 0 || ftruncate(fd, static_cast<off_t>(size)) != 0) return CUDA_ERROR_OUT_OF_MEMORY;
  uint64_t id = g_next_handle++;
  g_phys[id].reset(new PhysAlloc{fd, size, 1});
  *h = id;
  return CUDA_SUCCESS;
}
CUresult cuMemRelease(CUmemGenericAllocationHandle h) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_phys.find(h);
  if (it == g_phys.end()) return CUDA_ERROR_INVALID_VALUE;
  if (--it->second->refs == 0) {
    close(it->second->fd);
    g_phys.erase(it);
  }
  return CUDA_SUCCESS;
}
CUresult cuMemMap(CUdeviceptr ptr, size_t size, size_t offset, CUmemGenericAllocationHandle h,
                  unsigned long long) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_phys.find(h);
  if (it == g_phys.end() || offset + size > it->second->size) return CUDA_ERROR_INVALID_VALUE;
  // Must lie inside a reservation.
  bool inside = false;
  for (auto& r : g_reservations)
    if (ptr >= r.first && ptr + size <= r.first + r.second) inside = true;
  if (!inside) return CUDA_ERROR_INVALID_VALUE;
  for (auto& m : g_mappings)
    if (ptr < m.first + m.second.second && m.first < ptr + size) return CUDA_ERROR_ALREADY_MAPPED;
  void* m = mmap(reinterpret_cast<void*>(ptr), size, PROT_NONE, MAP_SHARED | MAP_FIXED,
                 it->second->fd, static_cast<off_t>(offset));
  if (m == MAP_FAILED) return CUDA_ERROR_OUT_OF_MEMORY;
  it->second->refs++;
  g_mappings[ptr] = {h, size};
  return CUDA_SUCCESS;
}
CUresult cuMemUnmap(CUdeviceptr ptr, size_t size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_mappings.find(ptr);
  if (it == g_mappings.end() || it->second.second != size) return CUDA_ERROR_INVALID_VALUE;
  mmap(reinterpret_cast<void*>(ptr), size, PROT_NONE,
       MAP_PRIVATE | MAP_ANONYMOUS | MAP_FIXED | MAP_NORESERVE, -1, 0);
  uint64_t h = it->second.first;
  g_mappings.erase(it);
  cuMemRelease(h);
  return CUDA_SUCCESS;
}
CUresult cuMemSetAccess(CUdeviceptr ptr, size_t size, const CUmemAccessDesc*, size_t) {
  return mprotect(reinterpret_cast<void*>(ptr), size, PROT_READ | PROT_WRITE) == 0
             ? CUDA_SUCCESS
             : CUDA_ERROR_INVALID_VALUE;
}
CUresult cuMemExportToShareableHandle(void* out, CUmemGenericAllocationHandle h,
                                      CUmemAllocationHandleType, unsigned long long) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_phys.find(h);
  if (it == g_phys.end()) return CUDA_ERROR_INVALID_VALUE;
  *static_cast<int*>(out) = dup(it->second->fd);
  return CUDA_SUCCESS;
}
CUresult cuMemImportFromShareableHandle(CUmemGenericAllocationHandle* h, void* os,
                                        CUmemAllocationHandleType) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int fd = dup(static_cast<int>(reinterpret_cast<intptr_t>(os)));
  off_t size = lseek(fd, 0, SEEK_END);
  uint64_t id = g_next_handle++;
  g_phys[id].reset(new PhysAlloc{fd, static_cast<size_t>(size), 1});
  *h = id;
  return CUDA_SUCCESS;
}
CUresult cuMemGetAddressRange_v2(CUdeviceptr* base, size_t* size, CUdeviceptr p) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  for (auto& m : g_mappings)
    if (p >= m.first && p < m.first + m.second.second) {
      if (base) *base = m.first;
      if (size) *size = m.second.second;
      return CUDA_SUCCESS;
    }
  return CUDA_ERROR_NOT_FOUND;
}
CUresult cuMemcpyHtoD_v2(CUdeviceptr dst, const void* src, size_t n) {
  memcpy(reinterpret_cast<void*>(dst), src, n);
  return CUDA_SUCCESS;
}
CUresult cuMemcpyDtoH_v2(void* dst, CUdeviceptr src, size_t n) {
  memcpy(dst, reinterpret_cast<void*>(src), n);
  return CUDA_SUCCESS;
}
CUresult cuMemsetD8_v2(CUdeviceptr dst, unsigned char v, size_t n) {
  memset(reinterpret_cast<void*>(dst), v, n);
  return CUDA_SUCCESS;
}
CUresult cuPointerGetAttribute(void*, CUpointer_attribute, CUdeviceptr) {
  return CUDA_ERROR_NOT_SUPPORTED;
}
CUresult cuMulticastCreate(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*) {
  return CUDA_ERROR_NOT_SUPPORTED;
}

// ---- code images ----------------------------------------------------------------
namespace {
void log_load(const char* loader, unsigned nj, CUjit_option* jk, void** jv, unsigned nl, CUlibraryOption* lk,
              void** lv) {
  std::string e = loader;
  for (unsigned i = 0; jk && jv && i < nj; ++i)
    e += " jit" + std::to_string(static_cast<int>(jk[i])) + "=" +
         std::to_string(static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(jv[i])));
  for (unsigned i = 0; lk && lv && i < nl; ++i)
    e += " lib" + std::to_string(static_cast<int>(lk[i])) + "=" +
         std::to_string(static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(lv[i])));
  g_load_log.push_back(e);
}
}  // namespace
CUresult load_image(CUlibrary* lib, const void* code) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  std::unique_ptr<MockLib> l(new MockLib());
  if (!parse_image(code, l.get())) return CUDA_ERROR_INVALID_IMAGE;
  *lib = reinterpret_cast<CUlibrary>(l.get());
  g_libs.insert(l.release());
  return CUDA_SUCCESS;
}
CUresult cuLibraryLoadData(CUlibrary* lib, const void* code, CUjit_option* jitOptions, void** jitOptionsValues,
                           unsigned int numJitOptions, CUlibraryOption* libraryOptions, void** libraryOptionValues,
                           unsigned int numLibraryOptions) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  log_load("cuLibraryLoadData", numJitOptions, jitOptions, jitOptionsValues, numLibraryOptions, libraryOptions,
           libraryOptionValues);
  return load_image(lib, code);
}
// Test hook: entry i of the load log (returns its length, or -1 past the end).
extern "C" int fbmock_load_log(int i, char* buf, int cap) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (i < 0 || static_cast<size_t>(i) >= g_load_log.size()) return -1;
  snprintf(buf, static_cast<size_t>(cap), "%s", g_load_log[static_cast<size_t>(i)].c_str());
  return static_cast<int>(g_load_log[static_cast<size_t>(i)].size());
}
CUresult cuLibraryLoadFromFile(CUlibrary*, const char*, CUjit_option*, void**, unsigned int,
                               CUlibraryOption*, void**, unsigned int) {
  return CUDA_ERROR_NOT_SUPPORTED;
}
CUresult cuLibraryUnload(CUlibrary lib) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* l = reinterpret_cast<MockLib*>(lib);
  if (!g_libs.count(l)) return CUDA_ERROR_INVALID_HANDLE;
  for (auto& f : l->funcs) g_funcs.erase(f.get());
  g_libs.erase(l);
  delete l;
  return CUDA_SUCCESS;
}
CUresult cuModuleLoadData(CUmodule* mod, const void* image) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  log_load("cuModuleLoadData", 0, nullptr, nullptr, 0, nullptr, nullptr);
  CUlibrary lib;
  CUresult rc = load_image(&lib, image);
  if (rc == CUDA_SUCCESS) *mod = reinterpret_cast<CUmodule>(lib);
  return rc;
}
CUresult cuModuleLoadDataEx(CUmodule* mod, const void* image, unsigned int n, CUjit_option* o, void** v) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  log_load("cuModuleLoadDataEx", n, o, v, 0, nullptr, nullptr);
  CUlibrary lib;
  CUresult rc = load_image(&lib, image);
  if (rc == CUDA_SUCCESS) *mod = reinterpret_cast<CUmodule>(lib);
  return rc;
}
CUresult cuModuleLoadFatBinary(CUmodule* mod, const void* image) { return cuModuleLoadData(mod, image); }
CUresult cuModuleLoad(CUmodule*, const char*) { return CUDA_ERROR_NOT_SUPPORTED; }
CUresult cuModuleUnload(CUmodule m) { return cuLibraryUnload(reinterpret_cast<CUlibrary>(m)); }
CUresult cuLibraryGetKernelCount(unsigned int* count, CUlibrary lib) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* l = reinterpret_cast<MockLib*>(lib);
  if (!g_libs.count(l)) return CUDA_ERROR_INVALID_HANDLE;
  *count = static_cast<unsigned>(l->funcs.size());
  return CUDA_SUCCESS;
}
CUresult cuLibraryEnumerateKernels(CUkernel* ks, unsigned int n, CUlibrary lib) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* l = reinterpret_cast<MockLib*>(lib);
  if (!g_libs.count(l)) return CUDA_ERROR_INVALID_HANDLE;
  for (unsigned i = 0; i < n && i < l->funcs.size(); ++i)
    ks[i] = reinterpret_cast<CUkernel>(l->funcs[i].get());
  return CUDA_SUCCESS;
}
CUresult cuModuleGetFunctionCount(unsigned int* count, CUmodule m) {
  return cuLibraryGetKernelCount(count, reinterpret_cast<CUlibrary>(m));
}
CUresult cuModuleEnumerateFunctions(CUfunction* fs, unsigned int n, CUmodule m) {
  return cuLibraryEnumerateKernels(reinterpret_cast<CUkernel*>(fs), n, reinterpret_cast<CUlibrary>(m));
}
CUresult cuLibraryGetKernel(CUkernel* k, CUlibrary lib, const char* name) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* l = reinterpret_cast<MockLib*>(lib);
  if (!g_libs.count(l)) return CUDA_ERROR_INVALID_HANDLE;
  for (auto& f : l->funcs)
    if (f->name == name) {
      *k = reinterpret_cast<CUkernel>(f.get());
      return CUDA_SUCCESS;
    }
  return CUDA_ERROR_NOT_FOUND;
}
CUresult cuModuleGetFunction(CUfunction* f, CUmodule m, const char* name) {
  return cuLibraryGetKernel(reinterpret_cast<CUkernel*>(f), reinterpret_cast<CUlibrary>(m), name);
}
CUresult cuLibraryGetModule(CUmodule* m, CUlibrary lib) {
  *m = reinterpret_cast<CUmodule>(lib);
  return CUDA_SUCCESS;
}
CUresult cuLibraryGetGlobal(CUdeviceptr* ptr, size_t* size, CUlibrary lib, const char* name) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* l = reinterpret_cast<MockLib*>(lib);
  if (!g_libs.count(l)) return CUDA_ERROR_INVALID_HANDLE;
  auto it = l->globals.find(name);
  if (it == l->globals.end()) return CUDA_ERROR_NOT_FOUND;
  if (ptr) *ptr = reinterpret_cast<CUdeviceptr>(it->second.data());
  if (size) *size = it->second.size();
  return CUDA_SUCCESS;
}
CUresult cuModuleGetGlobal_v2(CUdeviceptr* ptr, size_t* size, CUmodule m, const char* name) {
  return cuLibraryGetGlobal(ptr, size, reinterpret_cast<CUlibrary>(m), name);
}
CUresult cuKernelGetFunction(CUfunction* f, CUkernel k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!as_func(k)) return CUDA_ERROR_INVALID_HANDLE;
  *f = reinterpret_cast<CUfunction>(k);
  return CUDA_SUCCESS;
}
CUresult cuKernelGetName(const char** name, CUkernel k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(k);
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  *name = f->name.c_str();
  return CUDA_SUCCESS;
}
CUresult cuFuncGetName(const char** name, CUfunction fn) {
  return cuKernelGetName(name, reinterpret_cast<CUkernel>(fn));
}
CUresult cuKernelGetLibrary(CUlibrary* lib, CUkernel k) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(k);
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  *lib = reinterpret_cast<CUlibrary>(f->lib);
  return CUDA_SUCCESS;
}
CUresult cuFuncGetModule(CUmodule* m, CUfunction fn) {
  CUlibrary lib;
  CUresult rc = cuKernelGetLibrary(&lib, reinterpret_cast<CUkernel>(fn));
  if (rc == CUDA_SUCCESS) *m = reinterpret_cast<CUmodule>(lib);
  return rc;
}
CUresult cuFuncSetAttribute(CUfunction fn, CUfunction_attribute a, int v) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(fn);
  if (!f || a < 0 || a >= 16) return CUDA_ERROR_INVALID_HANDLE;
  f->attrs[a] = v;
  return CUDA_SUCCESS;
}
CUresult cuKernelSetAttribute(CUfunction_attribute a, int v, CUkernel k, CUdevice) {
  return cuFuncSetAttribute(reinterpret_cast<CUfunction>(k), a, v);
}
CUresult cuFuncGetAttribute(int* v, CUfunction_attribute a, CUfunction fn) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(fn);
  if (!f || a < 0 || a >= 16) return CUDA_ERROR_INVALID_HANDLE;
  *v = f->attrs[a];
  return CUDA_SUCCESS;
}
CUresult cuFuncGetParamInfo(CUfunction fn, size_t index, size_t* offset, size_t* size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(fn);
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  if (index >= f->param_sizes.size()) return CUDA_ERROR_INVALID_VALUE;
  size_t off = 0;
  for (size_t i = 0; i < index; ++i) off += f->param_sizes[i];
  if (offset) *offset = off;
  if (size) *size = f->param_sizes[index];
  return CUDA_SUCCESS;
}
CUresult cuLaunchKernelEx(const CUlaunchConfig*, CUfunction fn, void** params, void**) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(fn);
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  run_kernel(f, params);
  return CUDA_SUCCESS;
}
CUresult cuTensorMapEncodeTiled(CUtensorMap* map, CUtensorMapDataType dt, cuuint32_t rank,
                                void* addr, const cuuint64_t* dims, const cuuint64_t* strides,
                                const cuuint32_t* box, const cuuint32_t* estr,
                                CUtensorMapInterleave il, CUtensorMapSwizzle sw,
                                CUtensorMapL2promotion l2, CUtensorMapFloatOOBfill oob) {
  // Deterministic, content-only encoding (no process state), like the real one.
  memset(map, 0, sizeof(*map));
  uint64_t* w = reinterpret_cast<uint64_t*>(map);
  w[0] = reinterpret_cast<uint64_t>(addr);
  w[1] = (uint64_t(dt) << 32) | rank;
  for (cuuint32_t i = 0; i < rank && i < 4; ++i) w[2 + i] = dims[i] ^ (uint64_t(box[i]) << 48);
  if (rank > 1) w[6] = strides[0];
  w[7] = (uint64_t(il) << 24) | (uint64_t(sw) << 16) | (uint64_t(l2) << 8) | uint64_t(oob) |
         (uint64_t(estr[0]) << 32);
  return CUDA_SUCCESS;
}
CUresult cuStreamSynchronize(CUstream) { return CUDA_SUCCESS; }
CUresult cuStreamIsCapturing(CUstream, CUstreamCaptureStatus* s) {
  *s = CU_STREAM_CAPTURE_STATUS_NONE;
  return CUDA_SUCCESS;
}
CUresult cuEventCreate(CUevent* e, unsigned int) {
  *e = reinterpret_cast<CUevent>(new int(0));
  return CUDA_SUCCESS;
}
CUresult cuEventDestroy_v2(CUevent e) {
  delete reinterpret_cast<int*>(e);
  return CUDA_SUCCESS;
}

// ---- graphs -------------------------------------------------------------------
static MockGraph* as_graph(CUgraph g) {
  auto* mg = reinterpret_cast<MockGraph*>(g);
  return g_graphs.count(mg) ? mg : nullptr;
}
CUresult cuGraphCreate(CUgraph* g, unsigned int) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* mg = new MockGraph();
  g_graphs.insert(mg);
  *g = reinterpret_cast<CUgraph>(mg);
  return CUDA_SUCCESS;
}
CUresult cuGraphDestroy(CUgraph g) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockGraph* mg = as_graph(g);
  if (!mg) return CUDA_ERROR_INVALID_HANDLE;
  g_graphs.erase(mg);
  delete mg;
  return CUDA_SUCCESS;
}
static CUresult add_node(CUgraph g, const CUgraphNode* deps, size_t ndeps, MockNode* n,
                         CUgraphNode* out) {
  MockGraph* mg = as_graph(g);
  if (!mg) {
    delete n;
    return CUDA_ERROR_INVALID_HANDLE;
  }
  mg->nodes.emplace_back(n);
  for (size_t i = 0; i < ndeps; ++i) {
    mg->edges.emplace_back(reinterpret_cast<MockNode*>(deps[i]), n);
    CUgraphEdgeData e;
    memset(&e, 0, sizeof(e));
    mg->edge_data.push_back(e);
  }
  *out = reinterpret_cast<CUgraphNode>(n);
  return CUDA_SUCCESS;
}
CUresult cuGraphAddKernelNode_v2(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd,
                                 const CUDA_KERNEL_NODE_PARAMS* p) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockFunc* f = as_func(p->func ? static_cast<const void*>(p->func) : static_cast<const void*>(p->kern));
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  auto* n = new MockNode();
  n->kind = KERNEL;
  n->fn = f;
  n->kp = *p;
  n->kp.func = reinterpret_cast<CUfunction>(f);
  n->kp.extra = nullptr;
  copy_params(*n, f, p->kernelParams);
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddMemsetNode(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd,
                              const CUDA_MEMSET_NODE_PARAMS* p, CUcontext) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* n = new MockNode();
  n->kind = MEMSET;
  n->ms = *p;
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddMemcpyNode(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd,
                              const CUDA_MEMCPY3D* p, CUcontext) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* n = new MockNode();
  n->kind = MEMCPY;
  n->mc = *p;
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddEmptyNode(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* n = new MockNode();
  n->kind = EMPTY;
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddEventRecordNode(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd,
                                   CUevent e) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* n = new MockNode();
  n->kind = EV_RECORD;
  n->ev = e;
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddEventWaitNode(CUgraphNode* out, CUgraph g, const CUgraphNode* deps, size_t nd,
                                 CUevent e) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* n = new MockNode();
  n->kind = EV_WAIT;
  n->ev = e;
  return add_node(g, deps, nd, n, out);
}
CUresult cuGraphAddDependencies_v2(CUgraph g, const CUgraphNode* from, const CUgraphNode* to,
                                   const CUgraphEdgeData* data, size_t n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockGraph* mg = as_graph(g);
  if (!mg) return CUDA_ERROR_INVALID_HANDLE;
  for (size_t i = 0; i < n; ++i) {
    mg->edges.emplace_back(reinterpret_cast<MockNode*>(from[i]), reinterpret_cast<MockNode*>(to[i]));
    CUgraphEdgeData e;
    memset(&e, 0, sizeof(e));
    if (data) e = data[i];
    mg->edge_data.push_back(e);
  }
  return CUDA_SUCCESS;
}
CUresult cuGraphAddDependencies(CUgraph g, const CUgraphNode* from, const CUgraphNode* to,
                                size_t n) {
  return cuGraphAddDependencies_v2(g, from, to, nullptr, n);
}
CUresult cuGraphGetNodes(CUgraph g, CUgraphNode* nodes, size_t* n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockGraph* mg = as_graph(g);
  if (!mg) return CUDA_ERROR_INVALID_HANDLE;
  if (nodes)
    for (size_t i = 0; i < *n && i < mg->nodes.size(); ++i)
      nodes[i] = reinterpret_cast<CUgraphNode>(mg->nodes[i].get());
  *n = mg->nodes.size();
  return CUDA_SUCCESS;
}
CUresult cuGraphGetEdges_v2(CUgraph g, CUgraphNode* from, CUgraphNode* to, CUgraphEdgeData* data, size_t* n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockGraph* mg = as_graph(g);
  if (!mg) return CUDA_ERROR_INVALID_HANDLE;
  bool lossy = false;
  if (from && to)
    for (size_t i = 0; i < *n && i < mg->edges.size(); ++i) {
      from[i] = reinterpret_cast<CUgraphNode>(mg->edges[i].first);
      to[i] = reinterpret_cast<CUgraphNode>(mg->edges[i].second);
      const CUgraphEdgeData& e = mg->edge_data[i];
      if (data)
        data[i] = e;
      else if (e.from_port || e.to_port || e.type)
        lossy = true;
    }
  *n = mg->edges.size();
  // Like the driver: a query without edge data cannot describe such edges.
  return lossy ? CUDA_ERROR_LOSSY_QUERY : CUDA_SUCCESS;
}
CUresult cuGraphGetEdges(CUgraph g, CUgraphNode* from, CUgraphNode* to, size_t* n) {
  return cuGraphGetEdges_v2(g, from, to, nullptr, n);
}
CUresult cuGraphNodeGetType(CUgraphNode node, CUgraphNodeType* t) {
  auto* n = reinterpret_cast<MockNode*>(node);
  switch (n->kind) {
    case KERNEL: *t = CU_GRAPH_NODE_TYPE_KERNEL; break;
    case MEMSET: *t = CU_GRAPH_NODE_TYPE_MEMSET; break;
    case MEMCPY: *t = CU_GRAPH_NODE_TYPE_MEMCPY; break;
    case EMPTY: *t = CU_GRAPH_NODE_TYPE_EMPTY; break;
    case EV_RECORD: *t = CU_GRAPH_NODE_TYPE_EVENT_RECORD; break;
    case EV_WAIT: *t = CU_GRAPH_NODE_TYPE_WAIT_EVENT; break;
  }
  return CUDA_SUCCESS;
}
CUresult cuGraphKernelNodeGetParams_v2(CUgraphNode node, CUDA_KERNEL_NODE_PARAMS* p) {
  auto* n = reinterpret_cast<MockNode*>(node);
  if (n->kind != KERNEL) return CUDA_ERROR_INVALID_VALUE;
  *p = n->kp;
  return CUDA_SUCCESS;
}
CUresult cuGraphKernelNodeGetAttribute(CUgraphNode node, CUkernelNodeAttrID id,
                                       CUkernelNodeAttrValue* v) {
  auto* n = reinterpret_cast<MockNode*>(node);
  memset(v, 0, sizeof(*v));
  auto it = n->attrs.find(static_cast<int>(id));
  if (it != n->attrs.end()) *v = it->second;
  return CUDA_SUCCESS;
}
CUresult cuGraphKernelNodeSetAttribute(CUgraphNode node, CUkernelNodeAttrID id,
                                       const CUkernelNodeAttrValue* v) {
  auto* n = reinterpret_cast<MockNode*>(node);
  n->attrs[static_cast<int>(id)] = *v;
  return CUDA_SUCCESS;
}
CUresult cuGraphMemsetNodeGetParams(CUgraphNode node, CUDA_MEMSET_NODE_PARAMS* p) {
  *p = reinterpret_cast<MockNode*>(node)->ms;
  return CUDA_SUCCESS;
}
CUresult cuGraphMemcpyNodeGetParams(CUgraphNode node, CUDA_MEMCPY3D* p) {
  *p = reinterpret_cast<MockNode*>(node)->mc;
  return CUDA_SUCCESS;
}
CUresult cuGraphEventRecordNodeGetEvent(CUgraphNode node, CUevent* e) {
  *e = reinterpret_cast<MockNode*>(node)->ev;
  return CUDA_SUCCESS;
}
CUresult cuGraphEventWaitNodeGetEvent(CUgraphNode node, CUevent* e) {
  *e = reinterpret_cast<MockNode*>(node)->ev;
  return CUDA_SUCCESS;
}
CUresult cuGraphInstantiateWithFlags(CUgraphExec* out, CUgraph g, unsigned long long) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  MockGraph* mg = as_graph(g);
  if (!mg) return CUDA_ERROR_INVALID_HANDLE;
  auto* ex = new MockExec();
  ex->g.reset(new MockGraph());
  for (auto& n : mg->nodes) {
    auto* c = new MockNode(*n);
    if (c->kind == KERNEL) {
      c->param_ptrs.clear();
      for (auto& p : c->params) c->param_ptrs.push_back(p.data());
      c->kp.kernelParams = c->param_ptrs.data();
    }
    ex->g->nodes.emplace_back(c);
    ex->from_orig[n.get()] = c;
  }
  for (auto& e : mg->edges) ex->g->edges.emplace_back(ex->from_orig[e.first], ex->from_orig[e.second]);
  ex->g->edge_data = mg->edge_data;
  g_execs.insert(ex);
  *out = reinterpret_cast<CUgraphExec>(ex);
  return CUDA_SUCCESS;
}
CUresult cuGraphExecDestroy(CUgraphExec e) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* ex = reinterpret_cast<MockExec*>(e);
  if (!g_execs.count(ex)) return CUDA_ERROR_INVALID_HANDLE;
  g_execs.erase(ex);
  delete ex;
  return CUDA_SUCCESS;
}
CUresult cuGraphLaunch(CUgraphExec e, CUstream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* ex = reinterpret_cast<MockExec*>(e);
  if (!g_execs.count(ex)) return CUDA_ERROR_INVALID_HANDLE;
  for (MockNode* n : topo(*ex->g)) run_node(*n);
  return CUDA_SUCCESS;
}
CUresult cuGraphExecKernelNodeSetParams_v2(CUgraphExec e, CUgraphNode node,
                                           const CUDA_KERNEL_NODE_PARAMS* p) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* ex = reinterpret_cast<MockExec*>(e);
  if (!g_execs.count(ex)) return CUDA_ERROR_INVALID_HANDLE;
  auto it = ex->from_orig.find(reinterpret_cast<MockNode*>(node));
  if (it == ex->from_orig.end() || it->second->kind != KERNEL) return CUDA_ERROR_INVALID_VALUE;
  MockFunc* f = as_func(p->func ? static_cast<const void*>(p->func) : static_cast<const void*>(p->kern));
  if (!f) return CUDA_ERROR_INVALID_HANDLE;
  MockNode* c = it->second;
  c->fn = f;
  c->kp = *p;
  c->kp.func = reinterpret_cast<CUfunction>(f);
  copy_params(*c, f, p->kernelParams);
  return CUDA_SUCCESS;
}
CUresult cuGraphExecMemsetNodeSetParams(CUgraphExec e, CUgraphNode node,
                                        const CUDA_MEMSET_NODE_PARAMS* p, CUcontext) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* ex = reinterpret_cast<MockExec*>(e);
  auto it = ex->from_orig.find(reinterpret_cast<MockNode*>(node));
  if (it == ex->from_orig.end()) return CUDA_ERROR_INVALID_VALUE;
  it->second->ms = *p;
  return CUDA_SUCCESS;
}
CUresult cuGraphExecMemcpyNodeSetParams(CUgraphExec e, CUgraphNode node, const CUDA_MEMCPY3D* p,
                                        CUcontext) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto* ex = reinterpret_cast<MockExec*>(e);
  auto it = ex->from_orig.find(reinterpret_cast<MockNode*>(node));
  if (it == ex->from_orig.end()) return CUDA_ERROR_INVALID_VALUE;
  it->second->mc = *p;
  return CUDA_SUCCESS;
}
CUresult cuIpcGetMemHandle(CUipcMemHandle*, CUdeviceptr) { return CUDA_ERROR_NOT_SUPPORTED; }
CUresult cuIpcOpenMemHandle_v2(CUdeviceptr*, CUipcMemHandle, unsigned int) {
  return CUDA_ERROR_NOT_SUPPORTED;
}
CUresult cuIpcCloseMemHandle(CUdeviceptr) { return CUDA_ERROR_NOT_SUPPORTED; }

// Like the driver: a base name resolves to its newest versioned entry point of
// this library. Lookups use libc's dlsym on this library's own handle, so an
// interposer's dlsym override (which redirects driver symbols) is not involved.
CUresult cuGetProcAddress_v2(const char* symbol, void** pfn, int, cuuint64_t,
                             CUdriverProcAddressQueryResult* status) {
  using RealDlsym = void* (*)(void*, const char*);
  static RealDlsym real = reinterpret_cast<RealDlsym>(dlvsym(RTLD_DEFAULT, "dlsym", "GLIBC_2.2.5"));
  // The address of an internal object names this library; an exported
  // function's address may resolve to an interposer's definition of it.
  static const int anchor = 0;
  static void* self = [] {
    Dl_info info;
    dladdr(&anchor, &info);
    return dlopen(info.dli_fname, RTLD_NOW | RTLD_NOLOAD);
  }();
  *pfn = nullptr;
  if (real && self && symbol) {
    for (const char* suffix : {"_v3", "_v2", ""}) {
      *pfn = real(self, (std::string(symbol) + suffix).c_str());
      if (*pfn) break;
    }
  }
  if (status) *status = *pfn ? CU_GET_PROC_ADDRESS_SUCCESS : CU_GET_PROC_ADDRESS_SYMBOL_NOT_FOUND;
  return *pfn ? CUDA_SUCCESS : CUDA_ERROR_NOT_FOUND;
}

}  // extern "C"
