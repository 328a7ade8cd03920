// Quant-dequant of a host-resident activation, streamed through the GPU in
// row blocks.  Block c goes host -> device on copy stream 0, through the QDQ
// kernel on the caller's stream, and device -> host on copy stream 1, with
// `depth` blocks in flight, so both PCIe directions and the kernel overlap.
// Scale groups never cross a row, so any row split gives the whole-tensor
// result bit for bit (NVFP4 takes its per-tensor global scale as an input).
//
// Ordering: the copy streams first wait for an event recorded on the
// caller's stream at entry, and the caller's stream waits for the last
// copy at exit, so every use of the staging buffer lies between those two
// points of the caller's stream.  Within the call, per staging slot s:
//   loaded[s]  recorded after block c's H2D     (the kernel waits for it)
//   done[s]    recorded after block c's kernel  (the D2H waits for it)
//   freed[s]   recorded after block c's D2H     (block c + depth's H2D waits)
// A wait binds to the record enqueued most recently before it, and each
// slot's records and waits are enqueued in block order, so one event per
// slot and role suffices.
#include <mutex>

#include "common.cuh"
#include "qdq_b200.h"

namespace qdqb200 {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxDepth = 8;

std::mutex g_stream_mutex;
cudaStream_t g_copy_streams[kMaxDevices][2] = {};

// The two copy streams of the current device, created on first use and kept
// for the life of the process.  Calls from several threads share them; each
// call's events keep its own blocks in order.
int copy_streams(cudaStream_t out[2]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(QDQ_ERR_CUDA, "qdq_host_stream: cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(g_stream_mutex);
  for (int i = 0; i < 2; ++i) {
    if (g_copy_streams[dev][i] == nullptr) {
      e = cudaStreamCreateWithFlags(&g_copy_streams[dev][i], cudaStreamNonBlocking);
      if (e != cudaSuccess) {
        g_copy_streams[dev][i] = nullptr;
        return fail(QDQ_ERR_CUDA, "qdq_host_stream: cudaStreamCreate: %s", cudaGetErrorString(e));
      }
    }
    out[i] = g_copy_streams[dev][i];
  }
  return QDQ_OK;
}

struct Events {
  cudaEvent_t ev[3 * kMaxDepth + 3] = {};  // loaded, done, freed per slot; entry; two tails
  int n = 0;
  ~Events() {
    // Destroying an event whose record has not completed is allowed: its
    // resources are released once the device reaches it.
    for (int i = 0; i < n; ++i) cudaEventDestroy(ev[i]);
  }
  cudaError_t create(int count) {
    for (; n < count; ++n) {
      cudaError_t e = cudaEventCreateWithFlags(&ev[n], cudaEventDisableTiming);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
};

int elt_bytes(int dtype) { return (dtype == QDQ_DTYPE_BF16 || dtype == QDQ_DTYPE_FP16) ? 2 : 0; }

cudaError_t copy_rows(void* dst, int64_t ld_dst, const void* src, int64_t ld_src, int64_t rows, int64_t row_bytes,
                      cudaMemcpyKind kind, cudaStream_t s) {
  if (ld_dst == row_bytes && ld_src == row_bytes) return cudaMemcpyAsync(dst, src, rows * row_bytes, kind, s);
  return cudaMemcpy2DAsync(dst, ld_dst, src, ld_src, row_bytes, rows, kind, s);
}

}  // namespace
}  // namespace qdqb200

extern "C" int64_t qdq_host_stream_staging_bytes(int64_t block_rows, int64_t K, int dtype, int depth) {
  using namespace qdqb200;
  const int eb = elt_bytes(dtype);
  if (block_rows <= 0 || K <= 0 || eb == 0 || depth < 1 || depth > kMaxDepth) return -1;
  return 2 * static_cast<int64_t>(depth) * block_rows * K * eb;
}

extern "C" int qdq_host_stream(int format, const void* x_host, void* y_host, const float* global_scale, int64_t M,
                               int64_t K, int64_t ldx, int64_t ldy, int dtype, void* staging,
                               int64_t staging_bytes, int64_t block_rows, void* stream) {
  using namespace qdqb200;
  const int eb = elt_bytes(dtype);
  if (eb == 0) return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: unknown dtype %d", dtype);
  if (format != QDQ_FORMAT_MXFP4 && format != QDQ_FORMAT_NVFP4 && format != QDQ_FORMAT_MXFP8)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: unknown format %d", format);
  if (M < 0 || K < 0 || ldx < K || ldy < K)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: bad shape M=%lld K=%lld ldx=%lld ldy=%lld",
                static_cast<long long>(M), static_cast<long long>(K), static_cast<long long>(ldx),
                static_cast<long long>(ldy));
  if (M == 0 || K == 0) return QDQ_OK;
  if (x_host == nullptr || y_host == nullptr || staging == nullptr)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: null x, y or staging");
  if (format == QDQ_FORMAT_NVFP4 && global_scale == nullptr)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: NVFP4 needs the device global scale");
  if (block_rows <= 0) return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: block_rows must be positive");
  block_rows = block_rows < M ? block_rows : M;
  const int64_t slot_bytes = 2 * block_rows * K * eb;  // input + output block
  const int64_t blocks = (M + block_rows - 1) / block_rows;
  int64_t depth = staging_bytes / slot_bytes;
  if (depth < 1)
    return fail(QDQ_ERR_INVALID_ARG, "qdq_host_stream: staging of %lld bytes holds no block of %lld rows",
                static_cast<long long>(staging_bytes), static_cast<long long>(block_rows));
  if (depth > kMaxDepth) depth = kMaxDepth;
  if (depth > blocks) depth = blocks;

  cudaStream_t compute = static_cast<cudaStream_t>(stream);
  cudaStream_t cs[2];
  int st = copy_streams(cs);
  if (st != QDQ_OK) return st;
  Events ev;
  cudaError_t e = ev.create(static_cast<int>(3 * depth + 3));
  if (e != cudaSuccess) return fail(QDQ_ERR_CUDA, "qdq_host_stream: cudaEventCreate: %s", cudaGetErrorString(e));
  cudaEvent_t* loaded = ev.ev;
  cudaEvent_t* done = ev.ev + depth;
  cudaEvent_t* freed = ev.ev + 2 * depth;
  cudaEvent_t entry = ev.ev[3 * depth];
  cudaEvent_t* tail = ev.ev + 3 * depth + 1;
  // On a failure after copies were enqueued, `stream` still waits for both
  // copy streams, so the caller may release the staging buffer in its order.
  auto abandon = [&](int status) {
    for (int i = 0; i < 2; ++i)
      if (cudaEventRecord(tail[i], cs[i]) == cudaSuccess) cudaStreamWaitEvent(compute, tail[i], 0);
    return status;
  };

#define QDQ_HS_CHECK(call)                                                                                      \
  do {                                                                                                          \
    cudaError_t err_ = (call);                                                                                  \
    if (err_ != cudaSuccess) return abandon(fail(QDQ_ERR_CUDA, "qdq_host_stream: %s", cudaGetErrorString(err_))); \
  } while (0)

  // the staging buffer belongs to the caller's stream order
  QDQ_HS_CHECK(cudaEventRecord(entry, compute));
  QDQ_HS_CHECK(cudaStreamWaitEvent(cs[0], entry, 0));
  QDQ_HS_CHECK(cudaStreamWaitEvent(cs[1], entry, 0));
  const int64_t row_bytes = K * eb;
  uint8_t* base = static_cast<uint8_t*>(staging);
  for (int64_t c = 0; c < blocks; ++c) {
    const int64_t r0 = c * block_rows;
    const int64_t rows = (M - r0) < block_rows ? (M - r0) : block_rows;
    const int s = static_cast<int>(c % depth);
    uint8_t* in = base + s * slot_bytes;
    uint8_t* out = in + block_rows * row_bytes;
    if (c >= depth) QDQ_HS_CHECK(cudaStreamWaitEvent(cs[0], freed[s], 0));  // block c - depth has left slot s
    QDQ_HS_CHECK(copy_rows(in, row_bytes, static_cast<const uint8_t*>(x_host) + r0 * ldx * eb, ldx * eb, rows,
                           row_bytes, cudaMemcpyHostToDevice, cs[0]));
    QDQ_HS_CHECK(cudaEventRecord(loaded[s], cs[0]));
    QDQ_HS_CHECK(cudaStreamWaitEvent(compute, loaded[s], 0));
    if (format == QDQ_FORMAT_MXFP4)
      st = qdq_mxfp4(in, out, nullptr, nullptr, rows, K, K, K, dtype, 32, compute);
    else if (format == QDQ_FORMAT_MXFP8)
      st = qdq_mxfp8(in, out, nullptr, nullptr, rows, K, K, K, dtype, 32, compute);
    else
      st = qdq_nvfp4(in, out, nullptr, nullptr, global_scale, rows, K, K, K, dtype, compute);
    if (st != QDQ_OK) return abandon(st);
    QDQ_HS_CHECK(cudaEventRecord(done[s], compute));
    QDQ_HS_CHECK(cudaStreamWaitEvent(cs[1], done[s], 0));
    QDQ_HS_CHECK(copy_rows(static_cast<uint8_t*>(y_host) + r0 * ldy * eb, ldy * eb, out, row_bytes, rows,
                           row_bytes, cudaMemcpyDeviceToHost, cs[1]));
    QDQ_HS_CHECK(cudaEventRecord(freed[s], cs[1]));
  }
  // the caller's stream resumes after the last block's D2H (which follows
  // every H2D and kernel of the call)
  QDQ_HS_CHECK(cudaStreamWaitEvent(compute, freed[(blocks - 1) % depth], 0));
#undef QDQ_HS_CHECK
  return QDQ_OK;
}
