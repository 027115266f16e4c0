// Deterministic VMM allocation region and the allocation event log.
//
// One virtual span [base, base+size) is reserved with cuMemAddressReserve at a
// caller-chosen address. Every allocation routed here is placed at
// align_up(cursor, granularity) and the cursor only moves forward, so the same
// sequence of allocation sizes yields byte-identical device addresses in every
// process (SAVE and LOAD). Chunks are backed by cuMemCreate + cuMemMap with
// shareable handles so peers can map them at the same address.
//
// Parity: reference csrc/hook.cpp:201-275 (state), 2246-2441 (cuMemAlloc_v2),
// 2626-2681 (cuMemFree_v2), 2705-2804 (reserve carving), 3088-3348 (region
// API), 3350-3492 (event record/replay). Differences by design:
//  * state is process-global, one region per device ordinal (the reference
//    keeps it thread_local, so allocations from other threads escape);
//  * freeing a chunk unmaps and releases the physical memory but never calls
//    cuMemAddressFree on a sub-range of the reserved span;
//  * every check returns a status; nothing aborts.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../common/fb_json.h"
#include "hook_internal.h"

namespace fbh {
namespace {

constexpr uint64_t kDefaultGranularity = 2ull << 20;
constexpr size_t kCarveLimit = 2ull << 30;  // reservations below this are carved from the cursor

struct Chunk {
  uint64_t ptr;
  uint64_t size;
  CUmemGenericAllocationHandle handle;
  bool owns_handle;  // false for sub-allocations of the preallocated window
};

struct Region {
  int device = -1;
  uint64_t base = 0;
  uint64_t size = 0;
  uint64_t cursor = 0;          // offset from base of the next free byte
  uint64_t granularity = kDefaultGranularity;
  bool active = false;          // span reserved
  bool stopped = false;         // temporarily bypassed (stop/resume)
  bool reserved_by_us = false;
  // preallocated window [prealloc_off, prealloc_off + prealloc_size)
  uint64_t prealloc_off = 0;
  uint64_t prealloc_size = 0;
  CUmemGenericAllocationHandle prealloc_handle = 0;
  std::map<uint64_t, Chunk> chunks;          // ptr -> chunk
  std::map<uint64_t, uint64_t> carved;       // carved reservations ptr -> size
};

struct Event {
  enum Kind { Alloc, Free, Reserve } kind;
  uint64_t ptr;
  uint64_t size;
  uint64_t alignment;
};

std::recursive_mutex g_mu;
std::map<int, Region> g_regions;
int g_handle_types = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
std::vector<int> g_peers;
uint64_t g_fallbacks = 0;
uint64_t g_intercepted = 0;

bool g_recording = false;
uint64_t g_record_start = 0;
std::vector<Event> g_events;

int current_device() {
  CUdevice dev = -1;
  if (FB_CALL(cuCtxGetDevice, &dev) != CUDA_SUCCESS) return -1;
  return static_cast<int>(dev);
}

Region* region_for_current(bool require_enabled) {
  int dev = current_device();
  auto it = g_regions.find(dev);
  if (it == g_regions.end() || !it->second.active) return nullptr;
  if (require_enabled && it->second.stopped) return nullptr;
  return &it->second;
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

CUmemAllocationProp make_prop(int device) {
  CUmemAllocationProp prop;
  memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = static_cast<CUmemAllocationHandleType>(g_handle_types);
  return prop;
}

CUresult set_access(uint64_t ptr, uint64_t size, int device) {
  std::vector<CUmemAccessDesc> descs;
  CUmemAccessDesc d;
  memset(&d, 0, sizeof(d));
  d.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  d.location.id = device;
  d.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  descs.push_back(d);
  for (int p : g_peers) {
    if (p == device) continue;
    d.location.id = p;
    descs.push_back(d);
  }
  return FB_CALL(cuMemSetAccess, static_cast<CUdeviceptr>(ptr), size, descs.data(), descs.size());
}

// Map a fresh physical chunk at ptr. On failure nothing stays mapped.
CUresult map_chunk(Region& r, uint64_t ptr, uint64_t size, CUmemGenericAllocationHandle* out) {
  CUmemAllocationProp prop = make_prop(r.device);
  CUmemGenericAllocationHandle h = 0;
  CUresult rc = FB_CALL(cuMemCreate, &h, size, &prop, 0);
  if (rc != CUDA_SUCCESS) return rc;
  rc = FB_CALL(cuMemMap, static_cast<CUdeviceptr>(ptr), size, 0, h, 0);
  if (rc != CUDA_SUCCESS) {
    FB_CALL(cuMemRelease, h);
    return rc;
  }
  rc = set_access(ptr, size, r.device);
  if (rc != CUDA_SUCCESS) {
    FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(ptr), size);
    FB_CALL(cuMemRelease, h);
    return rc;
  }
  *out = h;
  return CUDA_SUCCESS;
}

void record(Event::Kind k, uint64_t ptr, uint64_t size, uint64_t alignment) {
  if (!g_recording) return;
  g_events.push_back(Event{k, ptr, size, alignment});
}

// Core allocation path shared by the interposed cuMemAlloc and fb_region_alloc.
CUresult region_alloc_locked(Region& r, uint64_t size, uint64_t* out) {
  if (size == 0) size = 1;
  const uint64_t g = r.granularity;
  uint64_t off = align_up(r.cursor, g);
  const uint64_t asize = align_up(size, g);
  // An allocation that would straddle the end of the preallocated window
  // starts after it instead (the window's tail stays unused): it must not
  // overlap memory that is already mapped.
  if (r.prealloc_size && off < r.prealloc_off + r.prealloc_size &&
      off + asize > r.prealloc_off + r.prealloc_size)
    off = r.prealloc_off + r.prealloc_size;
  if (off + asize > r.size) return CUDA_ERROR_OUT_OF_MEMORY;
  const uint64_t ptr = r.base + off;
  const bool in_prealloc = r.prealloc_size != 0 && off >= r.prealloc_off &&
                           off + asize <= r.prealloc_off + r.prealloc_size;
  if (in_prealloc) {
    r.chunks[ptr] = Chunk{ptr, asize, 0, false};
  } else {
    CUmemGenericAllocationHandle h = 0;
    CUresult rc = map_chunk(r, ptr, asize, &h);
    if (rc != CUDA_SUCCESS) return rc;
    r.chunks[ptr] = Chunk{ptr, asize, h, true};
  }
  r.cursor = off + asize;
  record(Event::Alloc, ptr, size, 0);
  *out = ptr;
  return CUDA_SUCCESS;
}

CUresult region_free_locked(Region& r, uint64_t ptr, bool* handled) {
  auto it = r.chunks.find(ptr);
  if (it == r.chunks.end()) {
    *handled = false;
    return CUDA_SUCCESS;
  }
  *handled = true;
  Chunk c = it->second;
  r.chunks.erase(it);
  record(Event::Free, ptr, 0, 0);
  if (!c.owns_handle) return CUDA_SUCCESS;  // inside the preallocated window
  CUresult rc = FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(c.ptr), c.size);
  if (rc != CUDA_SUCCESS) return rc;
  return FB_CALL(cuMemRelease, c.handle);
}

}  // namespace

bool g_preloaded = false;

bool region_active_for_current() {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return region_for_current(true) != nullptr;
}

bool region_try_alloc(size_t size, CUdeviceptr* out, CUresult* result) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(true);
  if (!r) return false;
  uint64_t p = 0;
  CUresult rc = region_alloc_locked(*r, size, &p);
  if (rc != CUDA_SUCCESS) {
    // Parity with the reference (hook.cpp:2364-2385): fall back to a plain
    // allocation rather than failing the caller, but count it so determinism
    // checks can flag the run.
    ++g_fallbacks;
    if (debug_enabled())
      fprintf(stderr, "[foundry hook] region alloc of %zu bytes failed (%d); falling back\n",
              size, static_cast<int>(rc));
    return false;
  }
  ++g_intercepted;
  *out = static_cast<CUdeviceptr>(p);
  *result = CUDA_SUCCESS;
  return true;
}

bool region_try_free(CUdeviceptr ptr, CUresult* result) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  for (auto& kv : g_regions) {
    Region& r = kv.second;
    if (!r.active || ptr < r.base || ptr >= r.base + r.size) continue;
    bool handled = false;
    CUresult rc = region_free_locked(r, ptr, &handled);
    if (!handled) {
      *result = CUDA_SUCCESS;  // carved/foreign mapping inside the span: not ours to free
      return true;
    }
    *result = rc;
    return true;
  }
  return false;
}

bool region_try_reserve(CUdeviceptr* ptr, size_t size, size_t alignment, CUdeviceptr addr,
                        CUresult* result) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(true);
  if (!r || addr != 0) return false;
  if (size < kCarveLimit) {
    const uint64_t a = std::max<uint64_t>(r->granularity, alignment ? alignment : 1);
    const uint64_t off = align_up(r->cursor, a);
    const uint64_t asize = align_up(size, r->granularity);
    if (off + asize > r->size) return false;
    *ptr = static_cast<CUdeviceptr>(r->base + off);
    r->cursor = off + asize;
    r->carved[r->base + off] = asize;
    record(Event::Reserve, r->base + off, size, alignment);
    *result = CUDA_SUCCESS;
    return true;
  }
  // Large reservations (symmetric heaps, expandable segments) get a hint just
  // past the span so they do not collide with it (reference hook.cpp:2745-2772).
  CUdeviceptr hint = static_cast<CUdeviceptr>(r->base + r->size);
  *result = fb_driver()->cuMemAddressReserve(ptr, size, alignment, hint, 0);
  return true;
}

bool region_try_address_free(CUdeviceptr ptr, size_t size, CUresult* result) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  for (auto& kv : g_regions) {
    Region& r = kv.second;
    auto it = r.carved.find(ptr);
    if (it == r.carved.end()) continue;
    (void)size;
    r.carved.erase(it);  // the VA stays part of the span; the cursor does not rewind
    *result = CUDA_SUCCESS;
    return true;
  }
  return false;
}

bool region_lookup_chunk(CUdeviceptr ptr, CUdeviceptr* base, size_t* size,
                         CUmemGenericAllocationHandle* handle) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  for (auto& kv : g_regions) {
    Region& r = kv.second;
    if (r.chunks.empty()) continue;
    auto it = r.chunks.upper_bound(ptr);
    if (it == r.chunks.begin()) continue;
    --it;
    if (ptr >= it->second.ptr && ptr < it->second.ptr + it->second.size) {
      *base = it->second.ptr;
      *size = it->second.size;
      *handle = it->second.owns_handle ? it->second.handle : r.prealloc_handle;
      return true;
    }
  }
  return false;
}

}  // namespace fbh

using namespace fbh;

extern "C" {

fb_status fb_region_set(uint64_t base, uint64_t size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  const FbDriver* d = fb_driver();
  if (!d->cuMemAddressReserve) {
    fb_set_error(FB_ERR_DRIVER, "CUDA driver not available (%s)", fb_driver_path());
    return FB_ERR_DRIVER;
  }
  int dev = current_device();
  if (dev < 0) {
    // No current context yet: make the primary context of device 0 current,
    // like cudaSetDevice(0) + cudaFree(0) would.
    CUresult rc = d->cuInit(0);
    if (rc != CUDA_SUCCESS) return drv_error(rc, "cuInit");
    CUcontext ctx = nullptr;
    rc = d->cuDevicePrimaryCtxRetain(&ctx, 0);
    if (rc != CUDA_SUCCESS) return drv_error(rc, "cuDevicePrimaryCtxRetain");
    d->cuCtxSetCurrent(ctx);
    dev = 0;
  }
  Region& r = g_regions[dev];
  if (r.active) {
    if (r.base == base && r.size == size) {
      r.stopped = false;
      return FB_OK;
    }
    fb_set_error(FB_ERR_INVALID, "a region [0x%llx, +%llu) is already set on device %d",
                 (unsigned long long)r.base, (unsigned long long)r.size, dev);
    return FB_ERR_INVALID;
  }
  CUmemAllocationProp prop = make_prop(dev);
  size_t gran = 0;
  if (d->cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) !=
          CUDA_SUCCESS ||
      gran == 0)
    gran = kDefaultGranularity;
  gran = std::max<size_t>(gran, kDefaultGranularity);
  if (base % gran != 0 || size % gran != 0) {
    fb_set_error(FB_ERR_INVALID, "region base/size must be multiples of %zu bytes", gran);
    return FB_ERR_INVALID;
  }
  CUdeviceptr got = 0;
  CUresult rc = d->cuMemAddressReserve(&got, size, gran, static_cast<CUdeviceptr>(base), 0);
  if (rc != CUDA_SUCCESS) return drv_error(rc, "cuMemAddressReserve(region)");
  if (got != base) {
    d->cuMemAddressFree(got, size);
    fb_set_error(FB_ERR_ADDRESS,
                 "driver placed the region at 0x%llx instead of 0x%llx (address range in use?)",
                 (unsigned long long)got, (unsigned long long)base);
    return FB_ERR_ADDRESS;
  }
  r = Region();
  r.device = dev;
  r.base = base;
  r.size = size;
  r.granularity = gran;
  r.active = true;
  r.reserved_by_us = true;
  return FB_OK;
}

fb_status fb_region_stop(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (r) r->stopped = true;
  return FB_OK;
}

fb_status fb_region_resume(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (!r) {
    fb_set_error(FB_ERR_INVALID, "no region was set on the current device");
    return FB_ERR_INVALID;
  }
  r->stopped = false;
  return FB_OK;
}

fb_status fb_region_release(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  int dev = current_device();
  auto it = g_regions.find(dev);
  if (it == g_regions.end() || !it->second.active) return FB_OK;
  Region& r = it->second;
  for (auto& kv : r.chunks) {
    if (!kv.second.owns_handle) continue;
    FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(kv.second.ptr), kv.second.size);
    FB_CALL(cuMemRelease, kv.second.handle);
  }
  r.chunks.clear();
  if (r.prealloc_size) {
    FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(r.base + r.prealloc_off), r.prealloc_size);
    FB_CALL(cuMemRelease, r.prealloc_handle);
  }
  if (r.reserved_by_us) FB_CALL(cuMemAddressFree, static_cast<CUdeviceptr>(r.base), r.size);
  g_regions.erase(it);
  return FB_OK;
}

fb_status fb_region_preallocate(uint64_t size) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (!r) {
    fb_set_error(FB_ERR_INVALID, "preallocate_region: no region on the current device");
    return FB_ERR_INVALID;
  }
  if (r->prealloc_size) {
    fb_set_error(FB_ERR_INVALID, "preallocate_region: a window is already mapped");
    return FB_ERR_INVALID;
  }
  const uint64_t off = align_up(r->cursor, r->granularity);
  const uint64_t asize = align_up(size, r->granularity);
  if (off + asize > r->size) {
    fb_set_error(FB_ERR_INVALID, "preallocate_region: %llu bytes do not fit the region",
                 (unsigned long long)asize);
    return FB_ERR_INVALID;
  }
  CUmemGenericAllocationHandle h = 0;
  CUresult rc = map_chunk(*r, r->base + off, asize, &h);
  if (rc != CUDA_SUCCESS) return drv_error(rc, "preallocate_region map");
  r->prealloc_off = off;
  r->prealloc_size = asize;
  r->prealloc_handle = h;
  return FB_OK;
}

fb_status fb_region_free_prealloc(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (!r || !r->prealloc_size) return FB_OK;
  // Sub-allocations inside the window lose their backing; drop them.
  for (auto it = r->chunks.begin(); it != r->chunks.end();) {
    if (!it->second.owns_handle) it = r->chunks.erase(it);
    else ++it;
  }
  FB_CALL(cuMemUnmap, static_cast<CUdeviceptr>(r->base + r->prealloc_off), r->prealloc_size);
  FB_CALL(cuMemRelease, r->prealloc_handle);
  r->prealloc_off = r->prealloc_size = 0;
  r->prealloc_handle = 0;
  return FB_OK;
}

uint64_t fb_region_get_offset(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  return r ? r->cursor : 0;
}

fb_status fb_region_set_offset(uint64_t offset) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (!r) {
    fb_set_error(FB_ERR_INVALID, "set_current_alloc_offset: no region on the current device");
    return FB_ERR_INVALID;
  }
  if (offset < r->cursor) {
    fb_set_error(FB_ERR_ADDRESS,
                 "set_current_alloc_offset: offset %llu is behind the cursor %llu (forward only)",
                 (unsigned long long)offset, (unsigned long long)r->cursor);
    return FB_ERR_ADDRESS;
  }
  if (offset > r->size) {
    fb_set_error(FB_ERR_INVALID, "set_current_alloc_offset: offset beyond the region");
    return FB_ERR_INVALID;
  }
  r->cursor = offset;
  return FB_OK;
}

uint64_t fb_region_base(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  return r ? r->base : 0;
}

uint64_t fb_region_size(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  return r ? r->size : 0;
}

int fb_region_active(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return region_for_current(true) != nullptr;
}

uint64_t fb_region_granularity(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  return r ? r->granularity : kDefaultGranularity;
}

uint64_t fb_region_fallback_count(void) { return g_fallbacks; }
uint64_t fb_hook_intercepted_allocs(void) { return g_intercepted; }

fb_status fb_region_alloc(uint64_t size, uint64_t* out_ptr) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  if (!r) {
    fb_set_error(FB_ERR_INVALID, "region_alloc: no region on the current device");
    return FB_ERR_INVALID;
  }
  CUresult rc = region_alloc_locked(*r, size, out_ptr);
  if (rc != CUDA_SUCCESS) return drv_error(rc, "region_alloc");
  return FB_OK;
}

fb_status fb_region_free(uint64_t ptr) {
  CUresult rc = CUDA_SUCCESS;
  if (!region_try_free(static_cast<CUdeviceptr>(ptr), &rc)) {
    fb_set_error(FB_ERR_INVALID, "region_free: 0x%llx is not in a region", (unsigned long long)ptr);
    return FB_ERR_INVALID;
  }
  return rc == CUDA_SUCCESS ? FB_OK : drv_error(rc, "region_free");
}

void fb_region_set_handle_types(int types) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_handle_types = types;
}

int fb_region_get_handle_types(void) { return g_handle_types; }

void fb_region_set_peer_access(const int* devices, int n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_peers.assign(devices, devices + n);
}

// ---- event log -------------------------------------------------------------

fb_status fb_events_start(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Region* r = region_for_current(false);
  g_events.clear();
  g_recording = true;
  g_record_start = r ? r->base + r->cursor : 0;
  return FB_OK;
}

fb_status fb_events_end(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_recording = false;
  return FB_OK;
}

void fb_events_clear(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  g_events.clear();
  g_record_start = 0;
}

size_t fb_events_to_json(char* buf, size_t cap) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  namespace J = fb::json;
  J::Array evs;
  for (const Event& e : g_events) {
    J::Object o;
    switch (e.kind) {
      case Event::Alloc:
        o["type"] = "alloc";
        o["size"] = static_cast<unsigned long long>(e.size);
        o["ptr"] = static_cast<unsigned long long>(e.ptr);
        break;
      case Event::Free:
        o["type"] = "free";
        o["ptr"] = static_cast<unsigned long long>(e.ptr);
        break;
      case Event::Reserve:
        o["type"] = "reserve";
        o["size"] = static_cast<unsigned long long>(e.size);
        o["ptr"] = static_cast<unsigned long long>(e.ptr);
        o["alignment"] = static_cast<unsigned long long>(e.alignment);
        break;
    }
    evs.push_back(J::Value(std::move(o)));
  }
  J::Object root;
  root["start_base_addr"] = static_cast<unsigned long long>(g_record_start);
  root["events"] = J::Value(std::move(evs));
  std::string s = J::Value(std::move(root)).dump();
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return s.size();
}

fb_status fb_events_replay_json(const char* text, size_t len) {
  namespace J = fb::json;
  J::Value root;
  try {
    root = J::parse(text, len);
  } catch (const std::exception& e) {
    fb_set_error(FB_ERR_IO, "allocator events: %s", e.what());
    return FB_ERR_IO;
  }
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  const auto& obj = root.as_object();
  const auto* evs = obj.find("events");
  if (!evs || evs->as_array().empty()) return FB_OK;
  Region* r = region_for_current(false);
  if (!r) {
    fb_set_error(FB_ERR_INVALID, "allocator events present but no region is set");
    return FB_ERR_INVALID;
  }
  const uint64_t start = obj.at("start_base_addr").as_u64();
  if (start != 0) {
    if (start < r->base || start > r->base + r->size) {
      fb_set_error(FB_ERR_ADDRESS, "recorded start 0x%llx lies outside the region",
                   (unsigned long long)start);
      return FB_ERR_ADDRESS;
    }
    const uint64_t want = start - r->base;
    if (r->cursor > want) {
      fb_set_error(FB_ERR_ADDRESS,
                   "cursor drift: LOAD cursor %llu is already past the SAVE start %llu",
                   (unsigned long long)r->cursor, (unsigned long long)want);
      return FB_ERR_ADDRESS;
    }
    r->cursor = want;
  }
  for (const auto& ev : evs->as_array()) {
    const auto& e = ev.as_object();
    const std::string& type = e.at("type").as_string();
    const uint64_t ptr = e.at("ptr").as_u64();
    if (type == "alloc") {
      uint64_t got = 0;
      CUresult rc = region_alloc_locked(*r, e.at("size").as_u64(), &got);
      if (rc != CUDA_SUCCESS) return drv_error(rc, "replay alloc");
      if (got != ptr) {
        fb_set_error(FB_ERR_ADDRESS, "replayed alloc landed at 0x%llx, SAVE had 0x%llx",
                     (unsigned long long)got, (unsigned long long)ptr);
        return FB_ERR_ADDRESS;
      }
    } else if (type == "free") {
      bool handled = false;
      CUresult rc = region_free_locked(*r, ptr, &handled);
      if (rc != CUDA_SUCCESS) return drv_error(rc, "replay free");
    } else if (type == "reserve") {
      const uint64_t size = e.at("size").as_u64();
      const uint64_t alignment = e.contains("alignment") ? e.at("alignment").as_u64() : 0;
      const uint64_t a = std::max<uint64_t>(r->granularity, alignment ? alignment : 1);
      const uint64_t off = align_up(r->cursor, a);
      if (r->base + off != ptr) {
        fb_set_error(FB_ERR_ADDRESS, "replayed reserve at 0x%llx, SAVE had 0x%llx",
                     (unsigned long long)(r->base + off), (unsigned long long)ptr);
        return FB_ERR_ADDRESS;
      }
      r->cursor = off + align_up(size, r->granularity);
      r->carved[ptr] = align_up(size, r->granularity);
    } else {
      fb_set_error(FB_ERR_IO, "unknown allocator event type '%s'", type.c_str());
      return FB_ERR_IO;
    }
  }
  return FB_OK;
}

}  // extern "C"
