// Self-test of the failure path: a kernel waits on an mbarrier that nothing
// ever arrives at.  Its bounded wait must give up after `timeout_ns`, record
// QDQ_ERR_TIMEOUT in the device status word and let the kernel exit, leaving
// the CUDA context usable.  Nothing here faults, traps or hangs the GPU.
#include "sm100.cuh"

namespace qdqb200 {
namespace {

__global__ void stuck_wait_kernel(uint64_t timeout_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) sm100::mbar_wait(&bar, 0, status, 0x7E57, timeout_ns);
}

}  // namespace
}  // namespace qdqb200

using namespace qdqb200;

extern "C" int qdq_selftest_bounded_wait(int64_t timeout_ns, void* stream) {
  if (timeout_ns <= 0 || timeout_ns > 10000000000ll)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_selftest_bounded_wait: timeout_ns must be in (0, 1e10]");
  int* status = device_status_ptr();
  if (status == nullptr) return QDQ_ERR_CUDA;
  stuck_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(timeout_ns), status);
  return check_launch("qdq_selftest_bounded_wait");
}
