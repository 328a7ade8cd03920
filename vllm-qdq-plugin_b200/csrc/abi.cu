// Error plumbing and device-property cache shared by every C-ABI entry point.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace qdqb200 {

static thread_local char g_last_error[1024] = "no error";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(QDQ_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return QDQ_OK;
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// One status word per device, in this translation unit's device memory.  It
// stays zero unless a kernel's bounded wait gives up.
static __device__ int g_device_status = 0;

int* device_status_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("device_status_ptr: cudaGetDevice failed");
    return nullptr;
  }
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) {
      set_error("device_status_ptr: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

}  // namespace qdqb200

extern "C" int qdq_device_status(int* out, int clear) {
  using namespace qdqb200;
  if (out == nullptr) return fail(QDQ_ERR_INVALID_ARG, "qdq_device_status: null out");
  int* p = device_status_ptr();
  if (p == nullptr) return QDQ_ERR_CUDA;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(out, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "qdq_device_status: %s", cudaGetErrorString(e));
  return QDQ_OK;
}

extern "C" const char* qdq_last_error(void) { return qdqb200::g_last_error; }

extern "C" int qdq_abi_version(void) { return 100; }
