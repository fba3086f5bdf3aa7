// Status reporting shared by every entry point.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"
#include "tcgen05.cuh"

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

// Device status word written by kernels whose bounded waits give up (one per
// device: a __device__ variable lives in each device's copy of the module).
__device__ int g_device_status;

// Looked up on every call rather than cached per device number: a cached
// address could belong to another context than the caller's current one.
int* device_status_ptr() {
  int* p = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_device_status) != cudaSuccess) return nullptr;
  return p;
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      n < 1)
    return 1;
  return n;
}

// Self-test of the bounded-wait path: one thread waits on an mbarrier phase
// that nothing completes, with the same helper the pipelined kernels use; the
// wait gives up after `timeout_ns` and the code is stored in the status word.
__global__ void wait_timeout_selftest_kernel(uint64_t timeout_ns, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
    if (!sm100::mbar_wait(&bar, 0, nullptr, timeout_ns)) atomicExch(status, 9001);
  }
}

}  // namespace tssm

extern "C" int tssm_selftest_wait_timeout(int64_t timeout_ns, tssm_stream_t stream) {
  TSSM_REQUIRE(timeout_ns > 0 && timeout_ns <= 2000000000, "selftest_wait_timeout: timeout in (0, 2 s]");
  int* status = tssm::device_status_ptr();
  if (!status) {
    tssm::set_error("selftest_wait_timeout: device status word unavailable");
    return TSSM_ERR_CUDA;
  }
  tssm::wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)timeout_ns,
                                                                                          status);
  return tssm::check_launch("selftest_wait_timeout");
}

extern "C" int tssm_check_device_status(tssm_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return tssm::check_launch("check_device_status");
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tssm::g_device_status, sizeof(int)) != cudaSuccess)
    return tssm::check_launch("check_device_status");
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(tssm::g_device_status, &zero, sizeof(int));
    tssm::set_error("a kernel's bounded device-side wait gave up (code %d)", v);
    return TSSM_ERR_TIMEOUT;
  }
  return TSSM_OK;
}

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
