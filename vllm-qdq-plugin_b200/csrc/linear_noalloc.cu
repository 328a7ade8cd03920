// fp4_linear_mxf4_noalloc: the fused MXFP4 linear (activation quantisation +
// tcgen05 block-scaled GEMM) without any device allocation.
//
// fp4_linear_mxf4 quantises the activation into a caller-provided workspace.
// Some callers cannot allocate device memory at the point of the call: C or
// C++ hosts that embed this library without an allocator of their own, code
// running where a cudaMalloc would synchronise the device or is not permitted
// (for instance between the capture-setup steps of an engine that hands out
// no scratch), or callers whose memory pool is already fully reserved.  This
// variant uses a fixed scratch array that lives in this library's device
// memory instead.
//
// Limits and sharing:
//   - the scratch is kLinearScratchBytes (32 MiB) per GPU, held by every GPU
//     that loads the library until the process exits;
//   - fp4_linear_workspace_bytes(M, K) must not exceed it (for K = 4096 that is
//     M <= 14561 rows); larger calls are rejected with QDQ_ERR_INVALID_ARG;
//   - all calls on a device share the one array; two calls whose kernels can
//     overlap on the GPU (different streams without ordering) race on it;
//   - the array keeps the last call's contents and is never cleared.  Every
//     activation code and every scale byte of a real row (row < M) is written
//     earlier in the same call.  The GEMM also reads the tiled scale bytes of
//     the pad rows that complete the last 128-row block (M <= row < 128 *
//     ceil(M / 128)); this call does not write them, so they hold whatever an
//     earlier call left.  Those scales only multiply the pad rows' codes,
//     which the tensor map fills with zeros, and pad rows of the product are
//     never stored, so they cannot reach the output.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current); make that first call
// before any stream capture.  The per-device lookup is guarded by a mutex, so
// host threads may make their first calls concurrently.
#include <mutex>

#include "common.cuh"

namespace qdqb200 {
namespace {

constexpr int64_t kLinearScratchBytes = 32ll << 20;

__device__ __align__(256) uint8_t g_linear_scratch[kLinearScratchBytes];

uint8_t* linear_scratch_ptr() {
  static std::mutex lock;
  static uint8_t* cache[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("fp4_linear_mxf4_noalloc: cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> guard(lock);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess) {
      set_error("fp4_linear_mxf4_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    cache[dev] = static_cast<uint8_t*>(p);
  }
  return cache[dev];
}

}  // namespace
}  // namespace qdqb200

using namespace qdqb200;

extern "C" int64_t fp4_linear_noalloc_scratch_bytes(void) { return kLinearScratchBytes; }

extern "C" int fp4_linear_mxf4_noalloc(const void* a, int64_t lda, int dtype, const void* w_codes,
                                       const void* w_sf_tiled, const void* bias, void* c, int64_t M,
                                       int64_t N, int64_t K, int64_t ldw_bytes, int64_t ldc, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(QDQ_ERR_INVALID_ARG, "fp4_linear_mxf4_noalloc: negative shape");
  if (M == 0 || N == 0) return QDQ_OK;
  const int64_t need = fp4_linear_workspace_bytes(M, K);
  if (need > kLinearScratchBytes)
    return fail(QDQ_ERR_INVALID_ARG,
                "fp4_linear_mxf4_noalloc: an [%lld, %lld] activation needs %lld bytes of scratch, more than "
                "the %lld-byte static array; use fp4_linear_mxf4 with a workspace",
                (long long)M, (long long)K, (long long)need, (long long)kLinearScratchBytes);
  uint8_t* scratch = linear_scratch_ptr();
  if (scratch == nullptr) return QDQ_ERR_CUDA;
  return fp4_linear_mxf4(a, lda, dtype, w_codes, w_sf_tiled, bias, c, M, N, K, ldw_bytes, ldc, scratch,
                         kLinearScratchBytes, stream);
}
