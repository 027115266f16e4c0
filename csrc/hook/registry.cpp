// Module registry: which code images are loaded, under which content hash,
// and which entry points they export. Graph persistence stores kernel nodes as
// (image hash, entry name) and resolves them back to functions on LOAD.
//
// Two kinds of image:
//  * own images: cubins built by this repository, loaded through
//    fb_registry_load_image with their exact bytes and size. They are hashed
//    (CRC-64/XZ over the bytes) and stored in fatbin_image_packed.img.
//  * foreign images: loaded by other code (e.g. cudart inside torch) through
//    the interposed cuLibraryLoadData / cuModuleLoadData*. Their bytes are
//    never read or copied: the image is identified by the shared object that
//    contains it (dladdr) and the offset of the image pointer from that
//    object's load base, and re-loaded on LOAD by handing the driver the same
//    pointer in the new process. Images not backed by a loaded object (heap
//    buffers) cannot be identified; graphs using them fail at SAVE.
//
// Parity: reference csrc/hook.cpp:558-727 (dump_fatbin_and_info), 1059-1182
// (entry-point enumeration), 1589-1700 (pack format), 3514-3572 (queries),
// 3687-4183 (load_cuda_modules_and_libraries). The pack files keep the
// reference's layout ([u64 hash][u64 size][bytes] records; text blocks of
// hash / loader,options / count / names / ---) so archives look alike.
#include <dlfcn.h>
#include <fcntl.h>
#include <link.h>
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "../common/fb_crc64.h"
#include "hook_internal.h"

namespace fbh {
namespace {

struct Image {
  uint64_t hash = 0;
  std::string loader = "cuLibraryLoadData";  // base function name of the load
  bool own = false;
  bool used = false;
  bool byname = false;          // foreign kernel found by entry name among loaded images
  bool nvshmem = false;         // device code reads NVSHMEM's device state (needs module init)
  std::vector<uint8_t> bytes;   // own images only
  std::string src_file;         // foreign: shared object path
  uint64_t src_offset = 0;      // foreign: image pointer - object load base
  CUlibrary lib = nullptr;
  CUmodule mod = nullptr;
  LoadOptions options;          // foreign: scalar JIT / library options of the original load
  std::vector<std::string> names;
  std::unordered_map<std::string, CUkernel> kernels;
  std::unordered_map<std::string, CUfunction> functions;  // module-loaded images
};

struct FnKey {
  uint64_t hash;
  std::string name;
};

// binary_flags bits of the pack's text blocks (same meanings as the
// reference's pack, csrc/hook.cpp:157-162): bit 0 would mark an image that
// still needs a device link (never written here), bit 1 an image that needs
// NVSHMEM module initialisation.
constexpr unsigned kFlagNeedsNvshmem = 1u << 1;

// Device symbols of NVSHMEM's device-side runtime: an image that defines or
// references one needs nvshmemx_cumodule_init / nvshmemx_culibrary_init
// before its kernels run (the probe set of reference csrc/hook.cpp:993-1012).
const char* const kNvshmemSymbols[] = {
    "nvshmemi_device_state_d", "nvshmemi_team_pool_d", "nvshmemi_team_same_mype_node_pool_d",
    "nvshmemi_mype_d",         "nvshmemi_npes_d",      "nvshmemi_node_mype_d",
    "nvshmemi_node_npes_d",    "nvshmemi_heap_base_d",
};

std::recursive_mutex g_mu;
std::map<uint64_t, std::unique_ptr<Image>> g_images;
// LOAD: reloaded images that need NVSHMEM initialisation, flushed by
// fb_registry_init_nvshmem once the NVSHMEM runtime is up.
std::vector<uint64_t> g_nvshmem_pending;
std::unordered_map<CUlibrary, uint64_t> g_lib_to_hash;
std::unordered_map<CUmodule, uint64_t> g_mod_to_hash;
std::unordered_map<CUfunction, FnKey> g_fn_to_key;
std::unordered_map<CUkernel, FnKey> g_kernel_to_key;
bool g_skip_processing = false;
std::string g_pack_on_exit;
thread_local int t_own_load_depth = 0;

// Every foreign library/module handle loaded in this process, identified or
// not: "byname" kernels are looked up among these. Images handed to the driver
// from heap memory (e.g. fatbins a library decompressed at run time) cannot be
// tied to a file without reading their bytes, which this project never does;
// their kernels are persisted by name and found again in the LOAD process,
// where the same library loads the same images during its own initialisation.
struct ForeignHandle {
  CUlibrary lib;
  CUmodule mod;
};
std::vector<ForeignHandle> g_foreign;

uint64_t byname_hash(const std::string& name) {
  std::string key = "byname:" + name;
  return fb::crc64(key.data(), key.size());
}

bool module_is_foreign(CUmodule mod) {
  const FbDriver* d = fb_driver();
  for (const auto& f : g_foreign) {
    if (f.mod == mod) return true;
    CUmodule m = nullptr;
    if (f.lib && d->cuLibraryGetModule && d->cuLibraryGetModule(&m, f.lib) == CUDA_SUCCESS && m == mod)
      return true;
  }
  return false;
}

CUfunction find_foreign_by_name(const char* name) {
  const FbDriver* d = fb_driver();
  for (const auto& f : g_foreign) {
    if (f.lib) {
      CUkernel k = nullptr;
      CUfunction fn = nullptr;
      if (d->cuLibraryGetKernel(&k, f.lib, name) == CUDA_SUCCESS && k &&
          d->cuKernelGetFunction(&fn, k) == CUDA_SUCCESS)
        return fn;
    } else if (f.mod) {
      CUfunction fn = nullptr;
      if (d->cuModuleGetFunction(&fn, f.mod, name) == CUDA_SUCCESS && fn) return fn;
    }
  }
  return nullptr;
}

void enumerate_library(Image& img) {
  const FbDriver* d = fb_driver();
  unsigned int count = 0;
  if (!d->cuLibraryGetKernelCount || d->cuLibraryGetKernelCount(&count, img.lib) != CUDA_SUCCESS)
    return;
  std::vector<CUkernel> ks(count);
  if (count && d->cuLibraryEnumerateKernels(ks.data(), count, img.lib) != CUDA_SUCCESS) return;
  img.names.clear();
  for (CUkernel k : ks) {
    const char* name = nullptr;
    if (d->cuKernelGetName(&name, k) != CUDA_SUCCESS || !name) continue;
    img.names.emplace_back(name);
    img.kernels[name] = k;
    g_kernel_to_key[k] = FnKey{img.hash, name};
  }
  CUmodule mod = nullptr;
  if (d->cuLibraryGetModule && d->cuLibraryGetModule(&mod, img.lib) == CUDA_SUCCESS && mod)
    g_mod_to_hash[mod] = img.hash;
}

void enumerate_module(Image& img) {
  const FbDriver* d = fb_driver();
  unsigned int count = 0;
  if (!d->cuModuleGetFunctionCount || d->cuModuleGetFunctionCount(&count, img.mod) != CUDA_SUCCESS)
    return;
  std::vector<CUfunction> fs(count);
  if (count && d->cuModuleEnumerateFunctions(fs.data(), count, img.mod) != CUDA_SUCCESS) return;
  img.names.clear();
  for (CUfunction f : fs) {
    const char* name = nullptr;
    if (d->cuFuncGetName(&name, f) != CUDA_SUCCESS || !name) continue;
    img.names.emplace_back(name);
    img.functions[name] = f;
    g_fn_to_key[f] = FnKey{img.hash, name};
  }
  g_mod_to_hash[img.mod] = img.hash;
}

// Driver-API probe (no byte of the image is read): does the image carry one
// of NVSHMEM's device symbols?
bool probe_nvshmem(const Image& img) {
  const FbDriver* d = fb_driver();
  for (const char* sym : kNvshmemSymbols) {
    CUdeviceptr p = 0;
    size_t sz = 0;
    if (img.lib && d->cuLibraryGetGlobal && d->cuLibraryGetGlobal(&p, &sz, img.lib, sym) == CUDA_SUCCESS)
      return true;
    if (!img.lib && img.mod && d->cuModuleGetGlobal && d->cuModuleGetGlobal(&p, &sz, img.mod, sym) == CUDA_SUCCESS)
      return true;
  }
  return false;
}

// Identify a foreign image pointer by the loaded object that contains it.
bool identify_foreign(const void* code, std::string* file, uint64_t* offset) {
  Dl_info info;
  if (!code || dladdr(code, &info) == 0 || !info.dli_fname || !info.dli_fbase) return false;
  char resolved[PATH_MAX];
  const char* path = realpath(info.dli_fname, resolved) ? resolved : info.dli_fname;
  *file = path;
  *offset = reinterpret_cast<uint64_t>(code) - reinterpret_cast<uint64_t>(info.dli_fbase);
  return true;
}

uint64_t foreign_hash(const std::string& file, uint64_t offset) {
  struct stat st;
  uint64_t fsize = (stat(file.c_str(), &st) == 0) ? static_cast<uint64_t>(st.st_size) : 0;
  std::string key = "file:" + file + "@" + std::to_string(offset) + "#" + std::to_string(fsize);
  return fb::crc64(key.data(), key.size());
}

// Load base of a shared object in this process (loading it if needed).
const uint8_t* object_base(const std::string& file) {
  void* h = dlopen(file.c_str(), RTLD_NOLOAD | RTLD_LAZY);
  if (!h) h = dlopen(file.c_str(), RTLD_LAZY | RTLD_LOCAL);
  if (!h) return nullptr;
  struct link_map* lm = nullptr;
  if (dlinfo(h, RTLD_DI_LINKMAP, &lm) != 0 || !lm) return nullptr;
  return reinterpret_cast<const uint8_t*>(lm->l_addr);
}

Image* register_foreign(const void* code, const char* tag) {
  std::string file;
  uint64_t off = 0;
  if (!identify_foreign(code, &file, &off)) return nullptr;
  uint64_t h = foreign_hash(file, off);
  auto& slot = g_images[h];
  if (!slot) {
    slot.reset(new Image());
    slot->hash = h;
    slot->src_file = file;
    slot->src_offset = off;
  }
  slot->loader = tag;
  return slot.get();
}

std::string hex16(uint64_t v) {
  char buf[24];
  snprintf(buf, sizeof(buf), "%016llx", static_cast<unsigned long long>(v));
  return buf;
}

void pack_at_exit() {
  if (!g_pack_on_exit.empty()) fb_registry_pack(g_pack_on_exit.c_str());
}

bool jit_option_is_scalar(int o) {
  switch (o) {
    case CU_JIT_MAX_REGISTERS:
    case CU_JIT_THREADS_PER_BLOCK:
    case CU_JIT_OPTIMIZATION_LEVEL:
    case CU_JIT_TARGET_FROM_CUCONTEXT:
    case CU_JIT_TARGET:
    case CU_JIT_FALLBACK_STRATEGY:
    case CU_JIT_GENERATE_DEBUG_INFO:
    case CU_JIT_LOG_VERBOSE:
    case CU_JIT_GENERATE_LINE_INFO:
    case CU_JIT_CACHE_MODE:
    case CU_JIT_POSITION_INDEPENDENT_CODE:
    case CU_JIT_MIN_CTA_PER_SM:
    case CU_JIT_MAX_THREADS_PER_BLOCK:
    case CU_JIT_OVERRIDE_DIRECTIVE_VALUES:
      return true;
    default:
      return false;  // log buffers, wall time, symbol tables: pointers or outputs
  }
}

void append_options(std::ostream& txt, const LoadOptions& o) {
  for (const auto& kv : o.jit) txt << ",jit" << kv.first << "=" << kv.second;
  for (const auto& kv : o.lib) txt << ",libopt" << kv.first << "=" << kv.second;
}

LoadOptions options_from(const std::map<std::string, std::string>& opts) {
  LoadOptions o;
  for (const auto& kv : opts) {
    if (kv.first.rfind("jit", 0) == 0 && kv.first.size() > 3 && isdigit(static_cast<unsigned char>(kv.first[3])))
      o.jit.emplace_back(atoi(kv.first.c_str() + 3), strtoull(kv.second.c_str(), nullptr, 10));
    else if (kv.first.rfind("libopt", 0) == 0 && kv.first.size() > 6)
      o.lib.emplace_back(atoi(kv.first.c_str() + 6), strtoull(kv.second.c_str(), nullptr, 10));
  }
  return o;
}

}  // namespace

LoadOptions capture_load_options(unsigned int num_jit, const CUjit_option* jit, void* const* jit_values,
                                 unsigned int num_lib, const CUlibraryOption* lib, void* const* lib_values) {
  LoadOptions o;
  for (unsigned i = 0; jit && jit_values && i < num_jit; ++i)
    if (jit_option_is_scalar(jit[i]))
      o.jit.emplace_back(static_cast<int>(jit[i]), static_cast<uint64_t>(reinterpret_cast<uintptr_t>(jit_values[i])));
  for (unsigned i = 0; lib && lib_values && i < num_lib; ++i)
    if (lib[i] == CU_LIBRARY_BINARY_IS_PRESERVED)
      o.lib.emplace_back(static_cast<int>(lib[i]), static_cast<uint64_t>(reinterpret_cast<uintptr_t>(lib_values[i])));
  return o;
}

bool registry_in_own_load() { return t_own_load_depth > 0; }

void registry_on_library_loaded(CUlibrary lib, const void* code, const char* tag, const LoadOptions& opts) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (t_own_load_depth > 0) return;
  g_foreign.push_back(ForeignHandle{lib, nullptr});
  if (g_skip_processing) return;
  Image* img = register_foreign(code, tag);
  if (!img) return;
  img->options = opts;
  img->lib = lib;
  g_lib_to_hash[lib] = img->hash;
  enumerate_library(*img);
  img->nvshmem = probe_nvshmem(*img);
}

void registry_on_module_loaded(CUmodule mod, const void* code, const char* tag, const LoadOptions& opts) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (t_own_load_depth > 0) return;
  g_foreign.push_back(ForeignHandle{nullptr, mod});
  if (g_skip_processing) return;
  Image* img = register_foreign(code, tag);
  if (!img) return;
  img->options = opts;
  img->mod = mod;
  enumerate_module(*img);
  img->nvshmem = probe_nvshmem(*img);
}

void registry_on_library_file_loaded(CUlibrary lib, const char* path) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (g_skip_processing || !path) return;
  char resolved[PATH_MAX];
  std::string file = realpath(path, resolved) ? resolved : path;
  uint64_t h = foreign_hash(file, UINT64_MAX);
  auto& slot = g_images[h];
  if (!slot) slot.reset(new Image());
  slot->hash = h;
  slot->src_file = file;
  slot->src_offset = UINT64_MAX;  // whole file
  slot->loader = "cuLibraryLoadFromFile";
  slot->lib = lib;
  g_lib_to_hash[lib] = h;
  enumerate_library(*slot);
  slot->nvshmem = probe_nvshmem(*slot);
}

void registry_on_module_file_loaded(CUmodule mod, const char* path) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (g_skip_processing || !path) return;
  char resolved[PATH_MAX];
  std::string file = realpath(path, resolved) ? resolved : path;
  uint64_t h = foreign_hash(file, UINT64_MAX);
  auto& slot = g_images[h];
  if (!slot) slot.reset(new Image());
  slot->hash = h;
  slot->src_file = file;
  slot->src_offset = UINT64_MAX;
  slot->loader = "cuModuleLoad";
  slot->mod = mod;
  enumerate_module(*slot);
  slot->nvshmem = probe_nvshmem(*slot);
}

}  // namespace fbh

using namespace fbh;

extern "C" {

fb_status fb_registry_load_image(const void* data, size_t size, const char* tag,
                                 CUlibrary* out_lib, uint64_t* out_hash) {
  if (!data || size == 0) {
    fb_set_error(FB_ERR_INVALID, "load_image: empty image");
    return FB_ERR_INVALID;
  }
  const uint64_t h = fb::crc64(data, size);
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto& slot = g_images[h];
  if (slot && slot->lib) {
    if (out_lib) *out_lib = slot->lib;
    if (out_hash) *out_hash = h;
    return FB_OK;
  }
  if (!slot) slot.reset(new Image());
  Image& img = *slot;
  img.hash = h;
  img.own = true;
  img.loader = "cuLibraryLoadData";
  img.bytes.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + size);
  (void)tag;
  const FbDriver* d = fb_driver();
  if (!d->cuLibraryLoadData) {
    fb_set_error(FB_ERR_DRIVER, "CUDA driver not available (%s)", fb_driver_path());
    return FB_ERR_DRIVER;
  }
  ++t_own_load_depth;
  CUresult rc = d->cuLibraryLoadData(&img.lib, img.bytes.data(), nullptr, nullptr, 0, nullptr,
                                     nullptr, 0);
  --t_own_load_depth;
  if (rc != CUDA_SUCCESS) return drv_error(rc, "cuLibraryLoadData(own image)");
  g_lib_to_hash[img.lib] = h;
  enumerate_library(img);
  img.nvshmem = probe_nvshmem(img);
  if (out_lib) *out_lib = img.lib;
  if (out_hash) *out_hash = h;
  return FB_OK;
}

fb_status fb_registry_adopt_module(CUmodule mod, const void* data, size_t size, uint64_t* out_hash) {
  if (!mod || !data || size == 0) {
    fb_set_error(FB_ERR_INVALID, "adopt_module: null module or empty image");
    return FB_ERR_INVALID;
  }
  const uint64_t h = fb::crc64(data, size);
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto& slot = g_images[h];
  if (!slot) {
    slot.reset(new Image());
    slot->hash = h;
    slot->own = true;
    slot->loader = "cuLibraryLoadData";
    slot->bytes.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + size);
  }
  Image& img = *slot;
  if (!img.own) {
    fb_set_error(FB_ERR_INVALID, "adopt_module: image %016llx is registered as foreign", (unsigned long long)h);
    return FB_ERR_INVALID;
  }
  // The same bytes may be loaded as several modules (e.g. one per context);
  // every module's functions map to the one image.
  CUmodule keep = img.mod;
  img.mod = mod;
  enumerate_module(img);
  img.nvshmem = img.nvshmem || probe_nvshmem(img);
  if (keep && keep != mod) img.mod = keep;
  if (out_hash) *out_hash = h;
  return FB_OK;
}

fb_status fb_registry_library(uint64_t hash, CUlibrary* out_lib) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_images.find(hash);
  if (it == g_images.end() || !it->second->lib) {
    fb_set_error(FB_ERR_NOT_FOUND, "no loaded library with hash %016llx", (unsigned long long)hash);
    return FB_ERR_NOT_FOUND;
  }
  *out_lib = it->second->lib;
  return FB_OK;
}

fb_status fb_registry_function(uint64_t hash, const char* name, CUfunction* out_fn,
                               CUkernel* out_kernel) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_images.find(hash);
  if (it == g_images.end()) {
    fb_set_error(FB_ERR_NOT_FOUND, "image %016llx is not loaded (missing from the archive?)",
                 (unsigned long long)hash);
    return FB_ERR_NOT_FOUND;
  }
  Image& img = *it->second;
  const FbDriver* d = fb_driver();
  if (img.byname) {
    auto fit = img.functions.find(name);
    CUfunction f = fit != img.functions.end() ? fit->second : find_foreign_by_name(name);
    if (!f) {
      fb_set_error(FB_ERR_NOT_FOUND,
                   "kernel '%s' (persisted by name) is not exported by any library loaded in this process; "
                   "initialise the library that owns it (e.g. run one warm-up call) before loading graphs",
                   name);
      return FB_ERR_NOT_FOUND;
    }
    img.functions[name] = f;
    g_fn_to_key[f] = FnKey{hash, name};
    if (out_fn) *out_fn = f;
    if (out_kernel) *out_kernel = nullptr;
    return FB_OK;
  }
  if (img.lib) {
    auto kit = img.kernels.find(name);
    CUkernel k = nullptr;
    if (kit != img.kernels.end()) {
      k = kit->second;
    } else {
      CUresult rc = d->cuLibraryGetKernel(&k, img.lib, name);
      if (rc != CUDA_SUCCESS) {
        fb_set_error(FB_ERR_NOT_FOUND, "entry point '%s' not found in image %016llx", name,
                     (unsigned long long)hash);
        return FB_ERR_NOT_FOUND;
      }
      img.kernels[name] = k;
      g_kernel_to_key[k] = FnKey{hash, name};
    }
    CUfunction f = nullptr;
    CUresult rc = d->cuKernelGetFunction(&f, k);
    if (rc != CUDA_SUCCESS) return drv_error(rc, "cuKernelGetFunction");
    g_fn_to_key[f] = FnKey{hash, name};
    if (out_fn) *out_fn = f;
    if (out_kernel) *out_kernel = k;
    return FB_OK;
  }
  if (img.mod) {
    auto fit = img.functions.find(name);
    CUfunction f = nullptr;
    if (fit != img.functions.end()) {
      f = fit->second;
    } else if (d->cuModuleGetFunction(&f, img.mod, name) != CUDA_SUCCESS) {
      fb_set_error(FB_ERR_NOT_FOUND, "entry point '%s' not found in module %016llx", name,
                   (unsigned long long)hash);
      return FB_ERR_NOT_FOUND;
    }
    g_fn_to_key[f] = FnKey{hash, name};
    if (out_fn) *out_fn = f;
    if (out_kernel) *out_kernel = nullptr;
    return FB_OK;
  }
  fb_set_error(FB_ERR_NOT_FOUND, "image %016llx has no live handle", (unsigned long long)hash);
  return FB_ERR_NOT_FOUND;
}

fb_status fb_registry_identify(CUfunction fn, uint64_t* out_hash, char* name_buf, size_t cap) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  const FnKey* key = nullptr;
  auto it = g_fn_to_key.find(fn);
  if (it != g_fn_to_key.end()) key = &it->second;
  if (!key) {
    auto kit = g_kernel_to_key.find(reinterpret_cast<CUkernel>(fn));
    if (kit != g_kernel_to_key.end()) key = &kit->second;
  }
  FnKey tmp;
  if (!key) {
    // Fall back to the driver: owning module + name.
    const FbDriver* d = fb_driver();
    CUmodule mod = nullptr;
    const char* name = nullptr;
    if (d->cuFuncGetModule && d->cuFuncGetModule(&mod, fn) == CUDA_SUCCESS && mod &&
        d->cuFuncGetName && d->cuFuncGetName(&name, fn) == CUDA_SUCCESS && name) {
      auto mit = g_mod_to_hash.find(mod);
      if (mit != g_mod_to_hash.end()) {
        tmp = FnKey{mit->second, name};
        key = &tmp;
        g_fn_to_key[fn] = tmp;
      } else if (module_is_foreign(mod)) {
        // Loaded by another library from memory we cannot tie to a file:
        // persist by entry name (see ForeignHandle).
        const uint64_t h = byname_hash(name);
        auto& slot = g_images[h];
        if (!slot) {
          slot.reset(new Image());
          slot->hash = h;
          slot->byname = true;
          slot->loader = "byname";
          slot->names = {name};
        }
        slot->functions[name] = fn;
        tmp = FnKey{h, name};
        key = &tmp;
        g_fn_to_key[fn] = tmp;
      }
    }
    if (!key) {
      const char* n = nullptr;
      if (d->cuFuncGetName) d->cuFuncGetName(&n, fn);
      fb_set_error(FB_ERR_UNSUPPORTED,
                   "kernel '%s' comes from a module the registry did not see load; it cannot be "
                   "persisted (load the hook with LD_PRELOAD, or use kernels built in-tree)",
                   n ? n : "?");
      return FB_ERR_UNSUPPORTED;
    }
  }
  if (out_hash) *out_hash = key->hash;
  if (name_buf && cap) {
    snprintf(name_buf, cap, "%s", key->name.c_str());
  }
  return FB_OK;
}

fb_status fb_registry_mark_used(uint64_t hash) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  auto it = g_images.find(hash);
  if (it == g_images.end()) {
    fb_set_error(FB_ERR_NOT_FOUND, "mark_used: unknown image %016llx", (unsigned long long)hash);
    return FB_ERR_NOT_FOUND;
  }
  it->second->used = true;
  return FB_OK;
}

fb_status fb_registry_pack(const char* folder) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  std::string dir(folder);
  mkdir(dir.c_str(), 0755);
  std::ofstream img(dir + "/fatbin_image_packed.img", std::ios::binary | std::ios::trunc);
  std::ofstream txt(dir + "/fatbin_entrypoint_packed.txt", std::ios::trunc);
  if (!img || !txt) {
    fb_set_error(FB_ERR_IO, "cannot write pack files in %s", folder);
    return FB_ERR_IO;
  }
  for (auto& kv : g_images) {
    const Image& im = *kv.second;
    if (!im.used) continue;
    const unsigned flags = im.nvshmem ? kFlagNeedsNvshmem : 0u;
    txt << hex16(im.hash) << "\n" << im.loader;
    if (im.byname) {
      txt << ",binary_flags=" << flags << "\n" << im.names.size() << "\n";
      for (const auto& n : im.names) txt << n << "\n";
      txt << "---\n";
      continue;
    }
    if (im.own) {
      const uint64_t h = im.hash, n = im.bytes.size();
      img.write(reinterpret_cast<const char*>(&h), 8);
      img.write(reinterpret_cast<const char*>(&n), 8);
      img.write(reinterpret_cast<const char*>(im.bytes.data()), static_cast<std::streamsize>(n));
    } else {
      // Foreign image: identified, not copied; its load options replayed on LOAD.
      append_options(txt, im.options);
      txt << ",source=" << im.src_file << ",source_offset=" << im.src_offset;
    }
    txt << ",binary_flags=" << flags << "\n" << im.names.size() << "\n";
    for (const auto& n : im.names) txt << n << "\n";
    txt << "---\n";
  }
  img.flush();
  txt.flush();
  if (!img || !txt) {
    fb_set_error(FB_ERR_IO, "short write of pack files in %s", folder);
    return FB_ERR_IO;
  }
  return FB_OK;
}

fb_status fb_registry_load_archive(const char* folder) {
  std::string dir(folder);
  std::ifstream txt(dir + "/fatbin_entrypoint_packed.txt");
  if (!txt) {
    fb_set_error(FB_ERR_NOT_FOUND, "missing %s/fatbin_entrypoint_packed.txt", folder);
    return FB_ERR_NOT_FOUND;
  }
  // Read all own images from the .img into memory (hash -> bytes).
  std::map<uint64_t, std::vector<uint8_t>> blobs;
  {
    std::ifstream img(dir + "/fatbin_image_packed.img", std::ios::binary);
    if (img) {
      for (;;) {
        uint64_t h = 0, n = 0;
        if (!img.read(reinterpret_cast<char*>(&h), 8)) break;
        if (!img.read(reinterpret_cast<char*>(&n), 8)) {
          fb_set_error(FB_ERR_IO, "truncated image record header in %s", folder);
          return FB_ERR_IO;
        }
        if (n > (1ull << 34)) {
          fb_set_error(FB_ERR_IO, "corrupt image size %llu", (unsigned long long)n);
          return FB_ERR_IO;
        }
        std::vector<uint8_t> b(n);
        if (n && !img.read(reinterpret_cast<char*>(b.data()), static_cast<std::streamsize>(n))) {
          fb_set_error(FB_ERR_IO, "truncated image %016llx in %s", (unsigned long long)h, folder);
          return FB_ERR_IO;
        }
        if (fb::crc64(b.data(), b.size()) != h) {
          fb_set_error(FB_ERR_IO, "image %016llx fails its CRC-64 check (corrupt archive)",
                       (unsigned long long)h);
          return FB_ERR_IO;
        }
        blobs[h] = std::move(b);
      }
    }
  }
  std::string line;
  const FbDriver* d = fb_driver();
  while (std::getline(txt, line)) {
    if (line.empty()) continue;
    uint64_t h = strtoull(line.c_str(), nullptr, 16);
    std::string spec;
    if (!std::getline(txt, spec)) {
      fb_set_error(FB_ERR_IO, "truncated entry-point list");
      return FB_ERR_IO;
    }
    std::string count_s;
    std::getline(txt, count_s);
    size_t count = strtoull(count_s.c_str(), nullptr, 10);
    std::vector<std::string> names(count);
    for (size_t i = 0; i < count; ++i) std::getline(txt, names[i]);
    std::string sep;
    std::getline(txt, sep);
    if (sep != "---") {
      fb_set_error(FB_ERR_IO, "malformed entry-point list for %016llx", (unsigned long long)h);
      return FB_ERR_IO;
    }
    // spec: loader[,key=value]*
    std::map<std::string, std::string> opts;
    std::string loader;
    {
      std::stringstream ss(spec);
      std::string tok;
      bool first = true;
      while (std::getline(ss, tok, ',')) {
        if (first) {
          loader = tok;
          first = false;
          continue;
        }
        auto eq = tok.find('=');
        if (eq != std::string::npos) opts[tok.substr(0, eq)] = tok.substr(eq + 1);
      }
    }
    std::lock_guard<std::recursive_mutex> lk(g_mu);
    auto& slot = g_images[h];
    if (slot && (slot->lib || slot->mod || slot->byname)) continue;  // already known in this process
    if (!slot) slot.reset(new Image());
    Image& im = *slot;
    im.hash = h;
    im.loader = loader;
    im.used = true;
    if (loader == "byname") {
      // Resolved lazily (fb_registry_function) among the images this process loads.
      im.byname = true;
      im.names = names;
      continue;
    }
    CUresult rc = CUDA_SUCCESS;
    if (opts.count("source")) {
      im.src_file = opts["source"];
      im.src_offset = strtoull(opts["source_offset"].c_str(), nullptr, 10);
      if (im.src_offset == UINT64_MAX) {
        rc = loader == "cuModuleLoad"
                 ? d->cuModuleLoad(&im.mod, im.src_file.c_str())
                 : d->cuLibraryLoadFromFile(&im.lib, im.src_file.c_str(), nullptr, nullptr, 0,
                                            nullptr, nullptr, 0);
      } else {
        const uint8_t* base = object_base(im.src_file);
        if (!base) {
          fb_set_error(FB_ERR_NOT_FOUND, "cannot map %s for image %016llx", im.src_file.c_str(),
                       (unsigned long long)h);
          return FB_ERR_NOT_FOUND;
        }
        const void* code = base + im.src_offset;
        im.options = options_from(opts);
        std::vector<CUjit_option> jk;
        std::vector<void*> jv;
        for (const auto& kv : im.options.jit) {
          jk.push_back(static_cast<CUjit_option>(kv.first));
          jv.push_back(reinterpret_cast<void*>(static_cast<uintptr_t>(kv.second)));
        }
        std::vector<CUlibraryOption> lk2;
        std::vector<void*> lv;
        for (const auto& kv : im.options.lib) {
          lk2.push_back(static_cast<CUlibraryOption>(kv.first));
          lv.push_back(reinterpret_cast<void*>(static_cast<uintptr_t>(kv.second)));
        }
        const unsigned nj = static_cast<unsigned>(jk.size()), nl = static_cast<unsigned>(lk2.size());
        if (loader == "cuModuleLoadDataEx")
          rc = d->cuModuleLoadDataEx(&im.mod, code, nj, nj ? jk.data() : nullptr, nj ? jv.data() : nullptr);
        else if (loader.rfind("cuModule", 0) == 0)
          rc = d->cuModuleLoadData(&im.mod, code);
        else
          rc = d->cuLibraryLoadData(&im.lib, code, nj ? jk.data() : nullptr, nj ? jv.data() : nullptr, nj,
                                    nl ? lk2.data() : nullptr, nl ? lv.data() : nullptr, nl);
      }
    } else {
      auto bit = blobs.find(h);
      if (bit == blobs.end()) {
        fb_set_error(FB_ERR_IO, "image %016llx listed but missing from the .img pack",
                     (unsigned long long)h);
        return FB_ERR_IO;
      }
      im.own = true;
      im.bytes = std::move(bit->second);
      ++t_own_load_depth;
      rc = d->cuLibraryLoadData(&im.lib, im.bytes.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
      --t_own_load_depth;
    }
    if (rc != CUDA_SUCCESS) return drv_error(rc, "reloading archived image");
    if (im.lib) {
      g_lib_to_hash[im.lib] = h;
      enumerate_library(im);
    } else {
      enumerate_module(im);
    }
    if (im.names.size() != count) {
      fb_set_error(FB_ERR_IO, "image %016llx exports %zu entry points, archive lists %zu",
                   (unsigned long long)h, im.names.size(), count);
      return FB_ERR_IO;
    }
    const unsigned flags = static_cast<unsigned>(strtoul(opts["binary_flags"].c_str(), nullptr, 10));
    im.nvshmem = (flags & kFlagNeedsNvshmem) != 0 || probe_nvshmem(im);
    if (im.nvshmem) g_nvshmem_pending.push_back(h);
  }
  return FB_OK;
}

int fb_registry_init_nvshmem(char* err, size_t err_cap) {
  using ModuleInit = int (*)(CUmodule);
  using LibraryInit = int (*)(CUlibrary);
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (g_nvshmem_pending.empty()) return 0;
  // The NVSHMEM host library is whatever the process loaded (preloaded, or
  // linked by an extension such as DeepEP); it is looked up, never loaded here.
  auto mod_init = reinterpret_cast<ModuleInit>(real_dlsym()(RTLD_DEFAULT, "nvshmemx_cumodule_init"));
  auto lib_init = reinterpret_cast<LibraryInit>(real_dlsym()(RTLD_DEFAULT, "nvshmemx_culibrary_init"));
  if (!mod_init && !lib_init) {
    snprintf(err, err_cap, "%zu loaded image(s) need NVSHMEM, but no NVSHMEM host library is loaded",
             g_nvshmem_pending.size());
    return -1;
  }
  int done = 0;
  std::vector<uint64_t> left;
  for (uint64_t h : g_nvshmem_pending) {
    auto it = g_images.find(h);
    if (it == g_images.end()) continue;
    const Image& im = *it->second;
    int rc = -1;
    if (im.lib && lib_init) {
      rc = lib_init(im.lib);
    } else if (mod_init) {
      CUmodule m = im.mod;
      if (!m && im.lib && fb_driver()->cuLibraryGetModule) fb_driver()->cuLibraryGetModule(&m, im.lib);
      if (m) rc = mod_init(m);
    }
    if (rc != 0) {
      left.push_back(h);
      snprintf(err, err_cap, "NVSHMEM initialisation of image %016llx failed (%d)", (unsigned long long)h, rc);
      continue;
    }
    ++done;
  }
  const bool failed = !left.empty();
  g_nvshmem_pending.swap(left);
  return failed ? -1 : done;
}

void fb_registry_set_skip_processing(int enabled) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_skip_processing = enabled != 0;
}

void fb_registry_set_pack_on_exit(const char* folder_or_null) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  static bool registered = false;
  g_pack_on_exit = folder_or_null ? folder_or_null : "";
  if (!registered && !g_pack_on_exit.empty()) {
    atexit(pack_at_exit);
    registered = true;
  }
}

size_t fb_registry_count(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return g_images.size();
}

}  // extern "C"
