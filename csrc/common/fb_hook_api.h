// C API of libfoundry_hook.so: the deterministic VMM region, the allocation
// event log and the module registry. The pybind module links against this
// library; under LD_PRELOAD the same instance also interposes the driver.
//
// Every function returns an fb_status (0 = ok) instead of aborting; the last
// error message of the calling thread is available from fb_last_error().
//
// Parity map (reference csrc/hook.h:25-52 and csrc/hook.cpp):
//   fb_region_set            set_allocation_region        hook.cpp:3088-3142
//   fb_region_stop/resume    stop/resume_allocation_region hook.cpp:3144-3159
//   fb_region_preallocate    preallocate_region           hook.cpp:3161-3275
//   fb_region_free_prealloc  free_preallocated_region     hook.cpp:3277-3300
//   fb_region_get/set_offset get/set_current_alloc_offset hook.cpp:3302-3348
//   fb_events_*              start/end_hook_record, save/replay  hook.cpp:3350-3492
//   fb_registry_*            module capture, pack, load, query   hook.cpp:558-1182, 1589-1700, 3514-4183
#pragma once

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int fb_status;
enum {
  FB_OK = 0,
  FB_ERR_DRIVER = 1,        // a driver call failed (message has the CUresult)
  FB_ERR_INVALID = 2,       // bad argument / state
  FB_ERR_ADDRESS = 3,       // determinism violated (address mismatch, cursor drift)
  FB_ERR_NOT_FOUND = 4,     // missing module / entry point / file
  FB_ERR_IO = 5,            // file read/write failed or archive corrupt
  FB_ERR_UNSUPPORTED = 6,   // e.g. kernel from a module that cannot be persisted
};

const char* fb_last_error(void);
void fb_set_error(fb_status code, const char* fmt, ...);

// ---- region -------------------------------------------------------------
fb_status fb_region_set(uint64_t base, uint64_t size);
fb_status fb_region_stop(void);
fb_status fb_region_resume(void);
fb_status fb_region_release(void);                 // unmap everything and free the VA span
fb_status fb_region_preallocate(uint64_t size);    // map [cursor, cursor+size) in one chunk
fb_status fb_region_free_prealloc(void);
uint64_t fb_region_get_offset(void);
fb_status fb_region_set_offset(uint64_t offset);   // forward only
uint64_t fb_region_base(void);
uint64_t fb_region_size(void);
int fb_region_active(void);
uint64_t fb_region_granularity(void);
uint64_t fb_region_fallback_count(void);           // allocs that fell back to cuMemAlloc
// Allocate/free through the region (same code path as the interposed cuMemAlloc).
fb_status fb_region_alloc(uint64_t size, uint64_t* out_ptr);
fb_status fb_region_free(uint64_t ptr);
// Handle types requested by cuMemCreate for region chunks (CUmemAllocationHandleType bits).
void fb_region_set_handle_types(int types);
int fb_region_get_handle_types(void);
// Peer access: devices (besides the owner) given RW access to every new chunk.
void fb_region_set_peer_access(const int* devices, int n);

// ---- allocation event log ------------------------------------------------
fb_status fb_events_start(void);
fb_status fb_events_end(void);
void fb_events_clear(void);
// JSON text {"start_base_addr":..., "events":[...]} of the last recording.
// Returns the number of bytes needed (excluding NUL); writes at most cap bytes.
size_t fb_events_to_json(char* buf, size_t cap);
// Replays events: fast-forwards the cursor, re-issues allocs and checks addresses.
fb_status fb_events_replay_json(const char* json, size_t len);

// ---- module registry -----------------------------------------------------
// Loads an image whose bytes and size are known (our own cubins). The image is
// hashed (CRC-64/XZ), kept for packing, loaded with cuLibraryLoadData and its
// kernels enumerated. Loading the same bytes twice returns the same library.
fb_status fb_registry_load_image(const void* data, size_t size, const char* tag,
                                 CUlibrary* out_lib, uint64_t* out_hash);
// Adopts a module that another component loaded from bytes it compiled in
// this process (a JIT compiler such as Triton): data/size are exactly the
// image handed to cuModuleLoadData. The image is hashed and kept like an own
// image (packed by bytes, reloaded with cuLibraryLoadData on LOAD) and the
// module's functions resolve to it. The bytes are stored, never parsed.
fb_status fb_registry_adopt_module(CUmodule mod, const void* data, size_t size, uint64_t* out_hash);
// Look up the library handle of an image by hash (after load or archive load).
fb_status fb_registry_library(uint64_t hash, CUlibrary* out_lib);
// Resolve an entry point of a registered image to a function of the current context.
fb_status fb_registry_function(uint64_t hash, const char* name, CUfunction* out_fn,
                               CUkernel* out_kernel);
// Reverse lookup for graph analysis: which image and entry point is this function?
// Writes the name into name_buf (cap bytes). FB_ERR_NOT_FOUND if unknown.
fb_status fb_registry_identify(CUfunction fn, uint64_t* out_hash, char* name_buf, size_t cap);
fb_status fb_registry_mark_used(uint64_t hash);
fb_status fb_registry_pack(const char* folder);
fb_status fb_registry_load_archive(const char* folder);
void fb_registry_set_skip_processing(int enabled);
// Initialises, with the process's NVSHMEM host library, every image reloaded
// from an archive that needs NVSHMEM (flag bit 1 of the pack, or one of
// NVSHMEM's device symbols found by driver lookup). Returns the number of
// images initialised (0 when none is pending), or -1 with a message in err
// (nothing is retried automatically; pending images stay queued).
int fb_registry_init_nvshmem(char* err, size_t err_cap);
void fb_registry_set_pack_on_exit(const char* folder_or_null);
size_t fb_registry_count(void);

// ---- misc ----------------------------------------------------------------
int fb_hook_is_preloaded(void);   // 1 when the interposer is active (LD_PRELOAD)
uint64_t fb_hook_intercepted_allocs(void);

#ifdef __cplusplus
}
#endif
