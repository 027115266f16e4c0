// Real-driver resolution and thread-local error reporting for libfoundry_hook.
//
// Parity: reference csrc/hook.cpp:1709-1822 (get_real_dlsym, load_cuda_library,
// init_hook). Differences by design: the driver is resolved lazily (so tests
// can point FOUNDRY_CUDA_DRIVER at the CPU mock before first use), and failure
// to find it is an error status, never an abort.
#include <dlfcn.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>
#include <string>

#include "../common/fb_driver.h"
#include "../common/fb_hook_api.h"
#include "hook_internal.h"

namespace fbh {

RealDlsym real_dlsym() {
  static RealDlsym fn = [] {
    // dlsym itself may be interposed by this library; take glibc's by version.
    void* p = dlvsym(RTLD_NEXT, "dlsym", "GLIBC_2.34");
    if (!p) p = dlvsym(RTLD_NEXT, "dlsym", "GLIBC_2.2.5");
    return reinterpret_cast<RealDlsym>(p);
  }();
  return fn;
}

static FbDriver g_driver;
static std::once_flag g_driver_once;
static std::string g_driver_path;

static void load_driver() {
  const char* env = getenv("FOUNDRY_CUDA_DRIVER");
  g_driver_path = (env && *env) ? env : "libcuda.so.1";
  // RTLD_NODELETE: the driver must outlive every static destructor that may
  // still call into it at exit.
  void* h = dlopen(g_driver_path.c_str(), RTLD_NOW | RTLD_LOCAL | RTLD_NODELETE);
  if (!h) return;
  g_driver.handle = h;
  g_driver.loaded = true;
  RealDlsym sym = real_dlsym();
#define FB_RESOLVE(name) \
  g_driver.name = reinterpret_cast<decltype(g_driver.name)>(sym(h, FB_STR(name)));
  FB_DRIVER_FUNCS(FB_RESOLVE)
#undef FB_RESOLVE
  g_driver.is_mock = sym(h, "fbmock_is_mock") != nullptr;
}

thread_local std::string t_last_error;

}  // namespace fbh

extern "C" {

const FbDriver* fb_driver(void) {
  std::call_once(fbh::g_driver_once, fbh::load_driver);
  return &fbh::g_driver;
}

const char* fb_driver_path(void) {
  fb_driver();
  return fbh::g_driver_path.c_str();
}

const char* fb_last_error(void) { return fbh::t_last_error.c_str(); }

void fb_set_error(fb_status code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  fbh::t_last_error = std::string("[foundry status ") + std::to_string(code) + "] " + buf;
  if (getenv("FOUNDRY_HOOK_DEBUG")) fprintf(stderr, "%s\n", fbh::t_last_error.c_str());
}

}  // extern "C"

namespace fbh {

fb_status drv_error(CUresult r, const char* what) {
  const char* name = nullptr;
  if (fb_driver()->cuGetErrorName) fb_driver()->cuGetErrorName(r, &name);
  fb_set_error(FB_ERR_DRIVER, "%s failed: %s (%d)", what, name ? name : "?", static_cast<int>(r));
  return FB_ERR_DRIVER;
}

bool debug_enabled() {
  static const bool on = getenv("FOUNDRY_HOOK_DEBUG") != nullptr;
  return on;
}

}  // namespace fbh
