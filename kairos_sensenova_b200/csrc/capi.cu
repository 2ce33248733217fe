// capi.cu -- error reporting and version entry points of the kb200 C ABI.
#include <cstdarg>
#include <cstdio>
#include "kb200_internal.h"

namespace kb {
static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(KB200_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return KB200_OK;
}
}  // namespace kb

extern "C" int kb200_abi_version(void) { return 2; }
extern "C" const char* kb200_last_error(void) { return kb::g_err; }
