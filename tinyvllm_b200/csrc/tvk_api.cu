// tvk_api.cu -- library-wide C ABI pieces: version, thread-local last error,
// and the driver entry point for TMA tensor-map encoding.
#include <stdarg.h>
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

}  // namespace tvk

extern "C" int tvk_abi_version(void) { return 1; }

extern "C" const char* tvk_last_error(void) { return tvk::g_last_error; }
