// Split-KV decode attention with a static scratch buffer: an entry point that
// allocates no device memory.
//
// This entry point has no counterpart in the reference: foundry-org/foundry
// persists graphs and has no attention kernels of its own. It exists for
// callers that cannot allocate:
//   * code running inside an active deterministic allocation region
//     (foundry_b200.allocation_region). Every allocation there advances the
//     region cursor, so a scratch allocation made by a diagnostic or
//     inspection call would move every later buffer and break the
//     SAVE == LOAD address layout that restored graphs depend on;
//   * a process at its device-memory limit (an out-of-memory handler that
//     still needs one attention result), where any allocation fails;
//   * a plain C or C++ host that links only this library and has no caching
//     allocator (torch's or otherwise) to borrow scratch from.
//
// The kernels are the ones of csrc/kernels/attention.cu (same source,
// compiled into this library): fb_decode_attn_g{4,8} writes per-split fp32
// partials (o, m, l), fb_decode_attn_combine merges them. Where the cubin
// path takes its partials from a caller-owned workspace, this entry point
// takes them from g_scratch, a file-scope __device__ array of
// FB_NOALLOC_SCRATCH_BYTES (8,519,680 bytes: room for 16,384 partial rows of
// 128 + 2 floats). Requests needing more partial rows are rejected with an
// error message.
//
// Nothing in g_scratch must start at zero: the split kernel writes every
// (sequence, head, split) row it owns before the combine reads it - a split
// past a sequence's end writes m = -inf, l = 0 - so no clearing is needed.
//
// Setup: the first call in each CUDA context resolves g_scratch's device
// address with cudaGetSymbolAddress, raises the split kernels' dynamic
// shared-memory limit and loads the combine kernel; make that first call
// before any stream capture. The set-up is cached per context, keyed by the
// driver's context ID (cuCtxGetId), which is never reused within a process:
// a second context on the same device, a non-primary context or a context
// re-created after cudaDeviceReset gets its own set-up instead of a stale
// address from another context. Later calls in a context only launch.
//
// Concurrency: every call on a device uses the same g_scratch. Calls that
// overlap on the device (different streams, or different host threads with
// no ordering between their streams) race on it and corrupt each other's
// partials; calls on one stream are ordered and safe.
//
// Allocation: the entry point makes no cudaMalloc/cudaFree call and calls no
// library that allocates; its only CUDA calls are
// cudaGetDriverEntryPointByVersion, cuCtxGetCurrent, cuCtxGetId,
// cudaGetSymbolAddress, cudaFuncSetAttribute, cudaFuncGetAttributes, two
// kernel launches and cudaGetLastError.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../kernels/attention.cu"
#include "decode_attn_noalloc.h"

#define FB_NOALLOC_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kHeadDim = 128;
constexpr int kPage = 64;
constexpr long long kMaxPartialRows = FB_NOALLOC_MAX_PARTIAL_ROWS;  // (sequence, query head, split) rows
constexpr size_t FB_NOALLOC_SCRATCH_BYTES = kMaxPartialRows * (kHeadDim + 2) * sizeof(float);
static_assert(FB_NOALLOC_SCRATCH_BYTES == 8519680, "documented scratch size");
constexpr int kMaxContexts = 64;

// o partials first ([rows][128] fp32), then (m, l) pairs ([rows][2] fp32).
static __device__ __align__(256) float g_scratch[FB_NOALLOC_SCRATCH_BYTES / sizeof(float)];

// One entry per CUDA context that has called the entry point.
struct ContextSetup {
  unsigned long long ctx_id = 0;
  float* scratch = nullptr;
};
ContextSetup g_setup[kMaxContexts];
int g_setup_count = 0;
std::mutex g_setup_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

int decode_smem_bytes(int group) {
  return 2 * 2 * kPage * kHeadDim * 2 + (group * kPage * 2 + group + group * kHeadDim) * 4;
}

int fail(char* err, int err_len, int code, const char* fmt, long long a = 0, long long b = 0) {
  if (err && err_len > 0) snprintf(err, static_cast<size_t>(err_len), fmt, a, b);
  return code;
}

int fail_cuda(char* err, int err_len, const char* what, cudaError_t e) {
  if (err && err_len > 0) snprintf(err, static_cast<size_t>(err_len), "%s: %s", what, cudaGetErrorString(e));
  return 3;
}

int driver_entry(const char* name, void** fn, char* err, int err_len) {
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaGetDriverEntryPointByVersion", e);
  if (q != cudaDriverEntryPointSuccess || !*fn) {
    if (err && err_len > 0) snprintf(err, static_cast<size_t>(err_len), "driver entry point %s not found", name);
    return 3;
  }
  return 0;
}

// ID of the context current on this thread; a runtime call is made first when
// none is current, so that the runtime binds the device's primary context.
int current_context_id(unsigned long long* id, char* err, int err_len) {
  if (!g_ctx_get_current) {
    void* a = nullptr;
    void* b = nullptr;
    if (int rc = driver_entry("cuCtxGetCurrent", &a, err, err_len)) return rc;
    if (int rc = driver_entry("cuCtxGetId", &b, err, err_len)) return rc;
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(b);
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(a);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return fail(err, err_len, 3, "cuCtxGetCurrent failed");
  if (!ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);  // initialises the primary context
    if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaGetSymbolAddress(g_scratch)", e);
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx) return fail(err, err_len, 3, "no current CUDA context");
  }
  if (g_ctx_get_id(ctx, id) != CUDA_SUCCESS) return fail(err, err_len, 3, "cuCtxGetId failed");
  return 0;
}

// Once per context, with that context current.
int setup_context(float** scratch, char* err, int err_len) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  unsigned long long id = 0;
  if (int rc = current_context_id(&id, err, err_len)) return rc;
  for (int i = 0; i < g_setup_count; ++i) {
    if (g_setup[i].ctx_id == id) {
      *scratch = g_setup[i].scratch;
      return 0;
    }
  }
  if (g_setup_count == kMaxContexts)
    return fail(err, err_len, 2, "more than %lld CUDA contexts called this entry point", kMaxContexts);
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
  if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaGetSymbolAddress(g_scratch)", e);
  e = cudaFuncSetAttribute(fb_decode_attn_g4, cudaFuncAttributeMaxDynamicSharedMemorySize, decode_smem_bytes(4));
  if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaFuncSetAttribute(fb_decode_attn_g4)", e);
  e = cudaFuncSetAttribute(fb_decode_attn_g8, cudaFuncAttributeMaxDynamicSharedMemorySize, decode_smem_bytes(8));
  if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaFuncSetAttribute(fb_decode_attn_g8)", e);
  // Under lazy module loading the combine kernel would otherwise load on the
  // first call with splits > 1, which may come during a stream capture.
  cudaFuncAttributes attrs;
  e = cudaFuncGetAttributes(&attrs, fb_decode_attn_combine);
  if (e != cudaSuccess) return fail_cuda(err, err_len, "cudaFuncGetAttributes(fb_decode_attn_combine)", e);
  g_setup[g_setup_count].ctx_id = id;
  g_setup[g_setup_count].scratch = static_cast<float*>(p);
  ++g_setup_count;
  *scratch = static_cast<float*>(p);
  return 0;
}

}  // namespace

// Declared and documented in decode_attn_noalloc.h.
FB_NOALLOC_EXPORT int fb_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                  const int* block_tables, int max_blocks, const int* seq_lens,
                                                  void* out, int batch, int n_q, int n_kv, int splits,
                                                  int pages_per_split, float scale, void* stream, char* err,
                                                  int err_len) {
  if (batch <= 0 || n_kv <= 0 || n_q <= 0 || splits <= 0 || pages_per_split <= 0 || max_blocks <= 0)
    return fail(err, err_len, 2, "batch, n_q, n_kv, splits, pages_per_split and max_blocks must be positive");
  if (n_q % n_kv != 0 || (n_q / n_kv != 4 && n_q / n_kv != 8))
    return fail(err, err_len, 2, "GQA group n_q/n_kv = %lld/%lld is not 4 or 8", n_q, n_kv);
  if (static_cast<long long>(splits) * pages_per_split < max_blocks)
    return fail(err, err_len, 2, "splits * pages_per_split = %lld does not cover max_blocks = %lld",
                static_cast<long long>(splits) * pages_per_split, max_blocks);
  if (!q || !k_cache || !v_cache || !block_tables || !seq_lens || !out)
    return fail(err, err_len, 2, "null tensor pointer");
  const long long rows = static_cast<long long>(batch) * n_q * splits;
  if (splits > 1 && rows > kMaxPartialRows)
    return fail(err, err_len, 1,
                "batch * n_q * splits = %lld partial rows exceed the static scratch (%lld rows, 8,519,680 bytes)",
                rows, kMaxPartialRows);
  float* scratch = nullptr;
  if (int rc = setup_context(&scratch, err, err_len)) return rc;
  float* o_part = scratch;
  float* ml_part = scratch + kMaxPartialRows * kHeadDim;
  const int group = n_q / n_kv;
  const float scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaGetLastError();  // start from a clean launch-error state of this runtime
  cudaError_t e;
  const dim3 grid(splits, n_kv, batch);
  const auto* qb = static_cast<const bf16*>(q);
  const auto* kb = static_cast<const bf16*>(k_cache);
  const auto* vb = static_cast<const bf16*>(v_cache);
  auto* ob = static_cast<bf16*>(out);
  if (group == 4)
    fb_decode_attn_g4<<<grid, 128, decode_smem_bytes(4), st>>>(qb, kb, vb, block_tables, max_blocks, seq_lens, ob,
                                                               o_part, ml_part, n_kv, pages_per_split, scale_log2);
  else
    fb_decode_attn_g8<<<grid, 128, decode_smem_bytes(8), st>>>(qb, kb, vb, block_tables, max_blocks, seq_lens, ob,
                                                               o_part, ml_part, n_kv, pages_per_split, scale_log2);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(err, err_len, "decode attention launch", e);
  if (splits > 1) {
    fb_decode_attn_combine<<<dim3(batch, n_q), 128, 0, st>>>(o_part, ml_part, ob, n_q, splits);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(err, err_len, "decode attention combine launch", e);
  }
  return 0;
}
