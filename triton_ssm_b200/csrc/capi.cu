// Status reporting shared by every entry point.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace tssm {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return TSSM_ERR_CUDA;
  }
  g_last_error[0] = '\0';
  return TSSM_OK;
}

}  // namespace tssm

extern "C" int tssm_version(void) { return 100; }

extern "C" const char* tssm_status_string(int s) {
  switch (s) {
    case TSSM_OK: return "ok";
    case TSSM_ERR_INVALID: return "invalid argument";
    case TSSM_ERR_UNSUPPORTED: return "unsupported configuration";
    case TSSM_ERR_CUDA: return "CUDA error";
    case TSSM_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* tssm_last_error(void) { return tssm::g_last_error; }
