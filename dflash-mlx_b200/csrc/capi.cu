// C-ABI housekeeping: version, last-error message.
#include "common.cuh"

#include <string>

namespace dfl {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

}  // namespace dfl

extern "C" int dfl_abi_version(void) { return DFL_ABI_VERSION; }

extern "C" const char* dfl_last_error(void) { return dfl::g_last_error.c_str(); }
