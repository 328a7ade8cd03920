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

}  // namespace qdqb200

extern "C" const char* qdq_last_error(void) { return qdqb200::g_last_error; }

extern "C" int qdq_abi_version(void) { return 100; }
