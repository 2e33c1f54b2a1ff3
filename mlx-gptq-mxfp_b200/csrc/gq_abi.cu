// Version, status strings and the per-thread last-error message.
#include <stdarg.h>
#include <stdio.h>

#include "gq_common.cuh"

namespace gq {

static thread_local char g_last_error[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s: %s", what, cudaGetErrorString(e));
    return GQ_ERR_CUDA;
  }
  return GQ_OK;
}

}  // namespace gq

extern "C" int gq_abi_version(void) { return GQ_ABI_VERSION; }

extern "C" const char* gq_status_string(int status) {
  switch (status) {
    case GQ_OK: return "ok";
    case GQ_ERR_ARG: return "invalid argument";
    case GQ_ERR_NOT_PD: return "Hessian not positive definite after damping escalation";
    case GQ_ERR_CUDA: return "CUDA error";
    case GQ_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* gq_last_error(void) { return gq::g_last_error; }
