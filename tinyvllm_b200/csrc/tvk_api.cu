// tvk_api.cu -- library-wide C ABI pieces: version, thread-local last error,
// and the driver entry point for TMA tensor-map encoding.
#include <stdarg.h>
#include <stdlib.h>
#include <mutex>

#include "tvk_common.cuh"

namespace tvk {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("TVK_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

static thread_local WaitTest g_wait_test = {false, 0};

WaitTest take_wait_test() {
  const WaitTest w = g_wait_test;
  g_wait_test = WaitTest{false, 0};
  return w;
}

}  // namespace tvk

extern "C" int tvk_abi_version(void) { return 1; }

extern "C" int tvk_debug_arm_wait_timeout(long long limit_ns) {
  if (limit_ns < 100000 || limit_ns > (long long)tvk::kDefaultWaitNs) {
    tvk::set_error("wait limit %lld ns outside [1e5, 2e9]", limit_ns);
    return TVK_ERR_INVALID;
  }
  tvk::g_wait_test = tvk::WaitTest{true, (unsigned long long)limit_ns};
  return TVK_OK;
}

extern "C" const char* tvk_last_error(void) { return tvk::g_last_error; }
