// Version, status strings, the per-thread last-error message and the driver lookups.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "gq_common.cuh"

namespace gq {

EncodeTiledFn tensor_map_encoder() {
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

// ---------------------------------------------------------------------------
// Self-test of the bounded device-side waits: one CTA waits on an mbarrier
// phase that nothing will complete, through the same mbar_wait used by the
// tcgen05 pipelines, with a short limit. The wait must give up, raise the CTA's
// abort flag and record GQ_ERR_TIMEOUT; the kernel then returns normally.
// ---------------------------------------------------------------------------
namespace gq {
__global__ void wait_selftest_kernel(unsigned long long limit_ns, int32_t* status, int32_t* gave_up) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status, limit_ns);
    *gave_up = ok ? 0 : 1;
  }
}
}  // namespace gq

extern "C" int gq_selftest_wait_timeout(unsigned long long limit_ns, int32_t* status, int32_t* gave_up,
                                        void* stream) {
  GQ_REQUIRE(status && gave_up, "gq_selftest_wait_timeout: null pointer");
  GQ_REQUIRE(limit_ns > 0 && limit_ns <= gq::kWaitLimitNs, "gq_selftest_wait_timeout: limit must be in (0, 2 s]");
  gq::wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, status, gave_up);
  return gq::check_launch("wait_selftest_kernel");
}
