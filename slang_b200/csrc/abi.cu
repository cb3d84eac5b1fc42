// Host-side plumbing shared by every entry point: thread-local error text,
// the device error word that bounded waits write, and device queries.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace {
thread_local char g_err[512] = "";

// One word per device: kernels record SB_ERR_TIMEOUT here instead of hanging.
__device__ int g_device_error = 0;
}  // namespace

namespace sb {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SB_OK : cuda_fail(e, what);
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int* device_error_word() {
  // cudaGetSymbolAddress is per device; cache per device id.
  static int* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

}  // namespace sb

extern "C" {

const char* sb_version(void) { return "slang_b200 0.1 (sm_100a)"; }

const char* sb_last_error(void) { return g_err; }

int sb_device_status(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* word = sb::device_error_word();
  if (!word) return sb::fail(SB_ERR_CUDA, "cannot resolve the device error word");
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, word, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return sb::cuda_fail(e, "sb_device_status");
  if (host != 0) {
    int zero = 0;
    cudaMemcpyAsync(word, &zero, sizeof(int), cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return sb::fail(SB_ERR_TIMEOUT, "a device-side wait timed out (code %d)", host);
  }
  return SB_OK;
}

}  // extern "C"
