/*
 * qdq_b200.h — C ABI of the B200 (sm_100a) block-scaled FP4 hot path.
 *
 * Every entry point:
 *   - takes plain device pointers, element counts/strides and a cudaStream_t
 *     passed as `void*` (NULL = legacy default stream);
 *   - is stream-ordered: it enqueues work and returns without a host sync;
 *   - returns QDQ_OK (0) or one of the qdq_status_t codes below; the text of
 *     the last failure on the calling thread is available from
 *     qdq_last_error();
 *   - never calls abort()/exit() and never allocates device memory unless the
 *     comment says so (scratch comes from the caller's `workspace`).
 *
 * dtype codes: QDQ_DTYPE_BF16 = 0, QDQ_DTYPE_FP16 = 1.
 * Strides (ldx, ldy, ...) are in ELEMENTS of the pointed-to type.
 */
#ifndef QDQ_B200_H_
#define QDQ_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  QDQ_OK = 0,
  QDQ_ERR_INVALID_ARG = 1,   /* bad shape / null pointer / unknown dtype      */
  QDQ_ERR_UNSUPPORTED = 2,   /* valid request this build does not implement   */
  QDQ_ERR_CUDA = 3,          /* a CUDA runtime call or launch failed          */
  QDQ_ERR_TIMEOUT = 4,       /* a bounded device-side wait gave up            */
  QDQ_ERR_ALIGNMENT = 5      /* pointer/stride alignment the kernel requires  */
} qdq_status_t;

enum { QDQ_DTYPE_BF16 = 0, QDQ_DTYPE_FP16 = 1 };

/* Human-readable text of the last non-zero status returned on this thread. */
const char* qdq_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int qdq_abi_version(void);

/*
 * MXFP4 activation quant-dequant: E2M1 elements, one E8M0 scale per 32
 * consecutive elements of a row.  Bit-exact with the reference
 *   vllm_qdq_plugin/qdq/mxfp4.py:98-156  (mxfp4_qdq, group_size=32)
 * including its amax rounding `(bits(amax) + 0x20) & 0xFF80` (bf16; fp16:
 * `+0x100 & 0xFC00`), scale = 2^(clamp(floor(log2 amax_r) + 125, 0, 254) - 127)
 * and round-to-nearest-even onto E2M1 with saturation at 6.
 *
 *   x      [M, K] bf16/fp16, row stride ldx   (input, not modified)
 *   y      [M, K] same dtype, row stride ldy  (output; may alias x iff ldx == ldy;
 *          may be NULL when `codes` is given, to emit only codes + scales)
 *   codes  optional [M, Kp/2] uint8, Kp = round_up(K, 32): packed E2M1 codes,
 *          element 2j in bits 0..3 and 2j+1 in bits 4..7 of byte j (NULL = skip)
 *   scales optional [M, Kp/32] uint8 E8M0 exponents (value 2^(s-127)) (NULL = skip)
 * group_size must be 32 (the only value the reference's callers use:
 * vllm_qdq_plugin/patch.py:57,142,149).
 */
int qdq_mxfp4(const void* x, void* y, void* codes, void* scales, int64_t M,
              int64_t K, int64_t ldx, int64_t ldy, int dtype, int group_size,
              void* stream);

/*
 * MXFP8 quant-dequant: E4M3 (float8_e4m3fn) elements, one E8M0 scale per 32
 * elements.  Replaces the reference's MXFP8 QDQ in front of float8_e4m3fn
 * Marlin GEMMs, vllm_qdq_plugin/qdq/mxfp8.py:73-125 (called at
 * vllm_qdq_plugin/patch.py:61-67 and :150-152), bit-exact: scale =
 * 2^(clamp(floor(log2 max(amax, FLT_MIN)) + 119, 0, 254) - 127), elements
 * rounded to nearest-even onto E4M3 with saturation at 448 and the
 * reference's subnormal clamp at 7 * 2^-9, zero quotients as +0.
 *
 *   x, y, ldx, ldy, dtype as qdq_mxfp4 (y may be NULL when `codes` is given)
 *   codes  optional [M, Kp] uint8 E4M3 bytes, Kp = round_up(K, 32), zero padded
 *   scales optional [M, Kp/32] uint8 E8M0 exponents (NULL = skip)
 * group_size must be 32 (patch.py:67, :152).
 */
int qdq_mxfp8(const void* x, void* y, void* codes, void* scales, int64_t M,
              int64_t K, int64_t ldx, int64_t ldy, int dtype, int group_size,
              void* stream);

/*
 * NVFP4 quant-dequant with a given per-tensor global scale: E2M1 elements,
 * one E4M3 scale per 16 elements, fp32 global scale `gs` read from device
 * memory (`global_scale`, 1 float).  Bit-exact with the CPU branch of
 *   vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py:
 *   ref_nvfp4_quant (:439-452) + ref_nvfp4_quant_dequant (:455-478)
 * (gs is vLLM's multiplier convention, 448*6/amax).  K % 16 == 0.
 *   codes  optional [M, K/2] uint8 packed E2M1 (same packing as qdq_mxfp4)
 *   scales optional [M, K/16] uint8 E4M3 block scales (NULL = skip)
 */
int qdq_nvfp4(const void* x, void* y, void* codes, void* scales,
              const float* global_scale, int64_t M, int64_t K, int64_t ldx,
              int64_t ldy, int dtype, void* stream);

/*
 * NVFP4 per-tensor global scale gs = 2688 / amax(|x|) in fp32 (2688 = 448*6),
 * written to `global_scale_out` (1 float, device).  `workspace` must point to
 * at least QDQ_AMAX_WORKSPACE_BYTES of device memory; it is cleared by this
 * call on `stream` before use.
 */
#define QDQ_AMAX_WORKSPACE_BYTES 16
int qdq_nvfp4_global_scale(const void* x, float* global_scale_out,
                           void* workspace, int64_t M, int64_t K, int64_t ldx,
                           int dtype, void* stream);

/*
 * Quant-dequant of an activation held in HOST memory, with the result written
 * to host memory.  Replaces the caller-side sequence "copy x to the GPU,
 * mxfp4_qdq / mxfp8_qdq / NVFP4 QDQ, copy the result back"
 * (vllm_qdq_plugin/qdq/mxfp4.py:98, qdq/mxfp8.py:73 and vLLM 0.22
 * nvfp4_emulation_utils.py:455 take device tensors).  The rows go through
 * the GPU in blocks of `block_rows`: H2D on an internal copy stream, the QDQ
 * kernel on `stream`, D2H on a second internal copy stream, with
 * staging_bytes / (2 * block_rows * K * elt) blocks in flight (at most 8),
 * so both PCIe directions and the kernel overlap.  Output is bit-identical to
 * the device entry points on the whole tensor (group size 32 for MXFP4 and
 * MXFP8, 16 for NVFP4, whose `global_scale` is a device float computed over
 * the whole tensor).
 *
 *   x_host, y_host  [M, K] bf16/fp16 with row strides ldx, ldy; pinned
 *                   (cudaHostAlloc / cudaHostRegister) for the copies to run
 *                   asynchronously
 *   staging         device buffer of at least
 *                   qdq_host_stream_staging_bytes(block_rows, K, dtype, 1)
 *                   bytes; with a 16-byte aligned base and block_rows * K * elt
 *                   a multiple of 16 every block takes the vectorised kernel
 *
 * Stream-ordered like every entry point: the copies start after the work
 * already on `stream`, and `stream` continues after the last copy, so the
 * caller synchronises `stream` before reading y_host and may release
 * `staging` in `stream`'s order.  The two copy streams are created per device
 * on first use and kept until exit.  Allocates no device memory.
 */
enum { QDQ_FORMAT_MXFP4 = 0, QDQ_FORMAT_NVFP4 = 1, QDQ_FORMAT_MXFP8 = 2 };
int qdq_host_stream(int format, const void* x_host, void* y_host,
                    const float* global_scale, int64_t M, int64_t K,
                    int64_t ldx, int64_t ldy, int dtype, void* staging,
                    int64_t staging_bytes, int64_t block_rows, void* stream);

/* Staging bytes for `depth` blocks of block_rows x K in flight; -1 if invalid. */
int64_t qdq_host_stream_staging_bytes(int64_t block_rows, int64_t K, int dtype,
                                      int depth);

/*
 * Device status word of the library on the current device: 0, or the first
 * failure a kernel recorded, as (qdq_status_t << 16) | site.  Kernels record
 * QDQ_ERR_TIMEOUT there when a bounded wait gives up (they then release their
 * tensor memory and exit instead of hanging).  Synchronises the device.
 * clear != 0 resets the word to 0.
 */
int qdq_device_status(int* out, int clear);

/*
 * Failure-path self-test (no counterpart in the reference): launches one CTA
 * that waits on an mbarrier nothing arrives at.  The bounded wait gives up
 * after timeout_ns (<= 1e10) and records (QDQ_ERR_TIMEOUT << 16) | 0x7E57 in
 * the status word read by qdq_device_status(); the context stays usable.
 */
int qdq_selftest_bounded_wait(int64_t timeout_ns, void* stream);

/* ---------------------------------------------------------------------------
 * Block-scaled FP4 GEMM (tcgen05 kind::mxf4) — replaces "MXFP4 QDQ of the
 * activation + Marlin bf16 x dequantised-FP4 GEMM" for MXFP4 Marlin layers:
 *   reference  vllm_qdq_plugin/patch.py:29-92 (_patch_marlin_gemm._patched)
 *              -> vllm/_custom_ops.py:1277 marlin_gemm
 *              (caller vllm/.../marlin_utils_fp4.py:149-202 apply_fp4_marlin_linear)
 * ------------------------------------------------------------------------- */

/*
 * Bytes of a scale-factor matrix in the tcgen05 tiled layout for `rows` rows
 * and K elements per row (E8M0, one scale per 32): rows padded to 128 and
 * scales per row padded to a multiple of 8, grouped into 512-byte chunks
 * (128 rows x 4 scales); chunk (rb, kc) starts at (rb * kchunks + kc) * 512
 * and holds the scale of (row r, scale k) at (r%32)*16 + ((r/32)%4)*4 + k%4.
 */
int64_t qdq_sf_tiled_bytes(int64_t rows, int64_t k);

/* Same for NVFP4's E4M3 scales, one per 16 elements: scales per row padded
 * to a multiple of 16 (one K-256 GEMM stage), same chunk layout. */
int64_t qdq_sf16_tiled_bytes(int64_t rows, int64_t k);

/* Row-major scales [rows, ceil(k/block)] (row stride ld bytes) -> tiled
 * layout above; padding bytes are written as 0.  block 32 (E8M0, sized by
 * qdq_sf_tiled_bytes) or 16 (E4M3, sized by qdq_sf16_tiled_bytes). */
int qdq_sf_tile(const void* sf, void* sf_tiled, int64_t rows, int64_t k, int64_t ld, int block,
                void* stream);

/*
 * C[M, N] (out_dtype bf16/fp16, row stride ldc elements) = A . W^T (+ bias[N], out_dtype),
 * fp32 accumulation.  A: E2M1 codes [M, K/2] (row stride lda_bytes), W: E2M1
 * codes [N, K/2] (row stride ldw_bytes), packed two per byte with element 2j
 * in the low nibble (the layout qdq_mxfp4 emits); a_sf_tiled / w_sf_tiled:
 * E8M0 scales in the tiled layout, 16-byte aligned.  K % 32 == 0; code
 * buffers and row strides 16-byte aligned (TMA).  bias may be NULL.
 */
int fp4_gemm_mxf4(const void* a_codes, const void* a_sf_tiled, const void* w_codes,
                  const void* w_sf_tiled, const void* bias, void* c, int64_t M, int64_t N,
                  int64_t K, int64_t lda_bytes, int64_t ldw_bytes, int64_t ldc, int out_dtype,
                  void* stream);

/*
 * NVFP4 GEMM: C = alpha * A . W^T (+ bias), fp32 accumulation, where A and W
 * are E2M1 codes as in fp4_gemm_mxf4 with one UE4M3 scale per 16 K elements
 * (tiled by qdq_sf_tile with block 16) and alpha = w_global_scale /
 * *a_global_scale.  Conventions are vLLM's NVFP4 ones: the activation
 * dequantises as code * s / gs_a (gs_a = 2688 / amax, the `global_scale` of
 * qdq_nvfp4; device pointer, read after the previous kernel on the stream
 * completes), the weight as code * s * gs_w (the layer's weight_global_scale,
 * passed by value).  Replaces, for NVFP4 Marlin layers:
 *   vllm/.../marlin_utils_fp4.py:149-202 apply_fp4_marlin_linear with a
 *   global_scale -> vllm/_custom_ops.py:1277 marlin_gemm.
 */
int fp4_gemm_nvf4(const void* a_codes, const void* a_sf_tiled, const float* a_global_scale,
                  const void* w_codes, const void* w_sf_tiled, float w_global_scale, const void* bias,
                  void* c, int64_t M, int64_t N, int64_t K, int64_t lda_bytes, int64_t ldw_bytes,
                  int64_t ldc, int out_dtype, void* stream);

/* Workspace bytes fp4_linear_nvf4 needs for an [M, K] activation. */
int64_t fp4_linear_nvf4_workspace_bytes(int64_t M, int64_t K);

/*
 * Fused linear for NVFP4 layers with NVFP4 activations (the build's
 * VLLM_QDQ_NVFP4_ACT=1 route): the activation's global scale (computed here
 * when a_global_scale is NULL, as nvfp4_qdq does), its NVFP4 codes and E4M3
 * scales (bit-identical to qdq_nvfp4's), then fp4_gemm_nvf4.  Equals
 * marlin_gemm(nvfp4_qdq(a), W_nvfp4) up to the bf16 rounding nvfp4_qdq
 * applies to each activation element and fp32 summation order.  workspace:
 * 256-byte aligned, fp4_linear_nvf4_workspace_bytes(M, K).  K % 32 == 0.
 * Same programmatic-dependent-launch stream order as fp4_linear_mxf4 for
 * M > 128.
 */
int fp4_linear_nvf4(const void* a, int64_t lda, int dtype, const float* a_global_scale,
                    const void* w_codes, const void* w_sf_tiled, float w_global_scale,
                    const void* bias, void* c, int64_t M, int64_t N, int64_t K, int64_t ldw_bytes,
                    int64_t ldc, void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes fp4_linear_mxf4 needs for an [M, K] activation. */
int64_t fp4_linear_workspace_bytes(int64_t M, int64_t K);

/*
 * Fused linear for MXFP4 layers: a [M, K] bf16/fp16 activation (row stride
 * lda elements) is quantised exactly as mxfp4_qdq does (qdq_mxfp4 codes +
 * scales, into `workspace`), then multiplied with the MXFP4 weight as in
 * fp4_gemm_mxf4; c and bias have the activation's dtype.  Output equals marlin_gemm(mxfp4_qdq(a), W) up to fp32
 * summation order.
 * Stream order: fp4_linear_mxf4 and fp4_gemm_mxf4 (M > 128) launch with
 * programmatic dependent launch.  Their kernels may start while the previous
 * kernel on the stream finishes and prefetch the weight (w_codes, w_sf_tiled)
 * before waiting for it; the activation, workspace, bias and output are
 * touched only after that kernel has completed.  The weight must therefore
 * not be written by the kernel launched just before the call (as in
 * inference, where weights are static).
 */
int fp4_linear_mxf4(const void* a, int64_t lda, int dtype, const void* w_codes,
                    const void* w_sf_tiled, const void* bias, void* c, int64_t M, int64_t N,
                    int64_t K, int64_t ldw_bytes, int64_t ldc, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Sage3 FP4 / FP8 attention — replaces the SAGE_ATTN backend's attention:
 *   reference  vllm_qdq_plugin/sage3_attn/impl.py:91-137 (_forward_sage3)
 *              -> sage3/api.py:89-387 (_run_attention: qk_smoothing,
 *              quantize_to_mxfp4, mxfp4_flash_attention / tiled_online_attention)
 * ------------------------------------------------------------------------- */

/* Workspace bytes sage3_fp4_attn needs (0 for an unsupported shape). */
int64_t sage3_attn_workspace_bytes(int64_t B, int64_t L, int64_t H, int64_t D);

/*
 * O = softmax(Q K^T * sm_scale) V with FP4 tensor-core MMAs (self-attention,
 * Q/K/V/O of the same [B, L, H, D] shape, D in {32, 64, 96, 128}, bf16 or fp16
 * (dtype QDQ_DTYPE_BF16 / QDQ_DTYPE_FP16; with fp16 the smoothing rounds to
 * fp16 and O is fp16, as the reference's torch ops on fp16 tensors); the
 * reference's hardware kernels take D in {64, 128}, mxfp4_hw_kernel.py:439).
 * Head dims below 128 are zero-extended to 128 inside the pre-pass, which
 * leaves every real quantisation group and every product unchanged.
 *   strides: 12 element strides, for q, k, v, o in turn: (batch, token, head);
 *            the head-dim stride must be 1.  NHD tensors [B, L, H, D] and HND
 *            tensors [B, H, L, D] are both expressed this way.
 *   quant_format: 0 = config "mxfp4_hw": MXFP4 (E2M1 + E8M0 per 32) with the
 *                reference hardware kernel's P handling (l = sum of unquantised P),
 *                mxfp4_hw_kernel.py:167-393;
 *            1 = config "nvfp4": NVFP4 (E2M1 + E4M3 per 16) with the reference's
 *                emulated-config P handling (P scaled by 448*6 before block
 *                scaling, l = sum of quantised P), p_quant_kernels.py:37-99 and
 *                attention_kernel.py:176-186;
 *            2 = config "mxfp4": the reference's emulated MXFP4 with the
 *                emulated-config P handling (p_quant_kernels.py:106-150).
 *                Q/K/V follow its quantize_qk / quantize_v steps (scale
 *                arithmetic in the input dtype, quantize.py:21-141) onto its
 *                9-level grid {0, .5, .75, 1, 1.5, 2, 3, 4, 6}, and so does
 *                P; 0.75 is no E2M1 value, so all of them are held as E4M3
 *                codes with E8M0 scales per 32 (kind::mxf8f6f4 MMAs);
 *            3 = config "mxfp8_hw": MXFP8 (E4M3 + E8M0 per 32) Q/K/V and P
 *                with the reference hardware kernel's P handling,
 *                mxfp8_hw_kernel.py:88-389 (kind::mxf8f6f4 MMAs);
 *            4 = "mxfp4_s1": as 2, P without the 448*6 prescale
 *                (p_quant_kernels.py:158-195);
 *            5 = "mxfp8_s1": the reference's emulated MXFP8 Q/K/V (its
 *                quantize_qk / quantize_v steps, E4M3 codes), emulated
 *                single-level MXFP8 P (p_quant_kernels.py:238-275);
 *            6 = "mixed_fp8qk_fp4pv": Q/K as 5, P/V as 4;
 *            7 = "mixed_fp4qk_fp8pv": Q/K as 4, P/V as 5;
 *            8 = "mixed_mxfp8qk_mxfp4pv_hw", 9 = "mixed_mxfp4qk_mxfp8pv_hw":
 *                the mixed hardware kernels (hardware P handling);
 *           10 = "mxfp4_s1_e4m3": E2M1 with an E4M3 scale per 32 for Q/K/V
 *                (quant_config.py:246-263) and single-level P with E4M3
 *                scales per 32, at least 2^-9 (p_quant_kernels.py:197-232).
 *   acc_mode: 0 = fp32, 1 = a reduced-precision PV accumulator of the
 *            reference (accepted; this kernel accumulates in fp32 either way).
 *   causal: non-zero for a causal mask (query i sees keys <= i).
 *   smoothing: bit 0 for the reference's qk_smoothing (K centring,
 *            per-128-token Q means and the delta_s correction); bit 1 for its
 *            v_smoothing (V centred over the sequence before quantisation,
 *            the mean added back to the output: the "_vs" / "_vsmooth" configs).
 *   workspace: >= sage3_attn_workspace_bytes() device bytes.
 * Keys beyond L are masked (the reference attends to its zero padding).
 */
int sage3_fp4_attn(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t L,
                   int64_t H, int64_t D, const int64_t* strides, float sm_scale,
                   int quant_format, int acc_mode, int causal, int smoothing, int dtype,
                   void* workspace, int64_t workspace_bytes, void* stream);

/*
 * fp4_linear_mxf4 for callers that cannot allocate device memory (no
 * counterpart in the reference: its QDQ and Marlin paths allocate through
 * torch).  Same arguments and result as fp4_linear_mxf4 minus the workspace:
 * the activation codes go to a static 32 MiB scratch array in the library's
 * device memory (fp4_linear_noalloc_scratch_bytes()), held by every GPU that
 * loads the library until exit.  Calls needing more scratch than that
 * (fp4_linear_workspace_bytes(M, K) > 32 MiB) fail with QDQ_ERR_INVALID_ARG.
 * All calls on a device share the array: calls that overlap on the GPU race.
 * The first call on a device looks up the array's address; make it before any
 * stream capture.  Allocates nothing (no cudaMalloc/cudaFree).
 */
int64_t fp4_linear_noalloc_scratch_bytes(void);
int fp4_linear_mxf4_noalloc(const void* a, int64_t lda, int dtype, const void* w_codes,
                            const void* w_sf_tiled, const void* bias, void* c, int64_t M, int64_t N,
                            int64_t K, int64_t ldw_bytes, int64_t ldc, void* stream);

/*
 * Grouped MXFP4 MoE GEMM.  Replaces "MXFP4 QDQ of the activation, then vLLM's
 * moe_wna16_marlin_gemm" for MXFP4 experts (reference:
 * vllm_qdq_plugin/patch.py:139-152 + vllm/_custom_ops.py:2469, as called from
 * vllm/model_executor/layers/fused_moe/experts/marlin_moe.py).  For every block
 * b < num_tokens_post_padded / moe_block_size whose expert e = expert_ids[b]
 * lies in [0, num_experts), and every slot s = sorted_token_ids[b *
 * moe_block_size + i] < size_m * top_k:
 *   C[s, :] = mxfp4_qdq(A[s / top_k, :]) . W_e^T   (x topk_weights[s] if mul_topk_weights)
 * with fp32 accumulation; rows of C no slot names are not written.
 *   a            [size_m, K] bf16/fp16 (dtype), row stride lda elements, 16-byte aligned rows
 *   w_codes      [num_experts, N, K/2] packed E2M1 (element 2j in the low nibble), contiguous
 *   w_sf_tiled   num_experts blocks of qdq_sf_tiled_bytes(N, K) bytes: each expert's E8M0
 *                scales in the tiled layout of qdq_sf_tile
 *   sorted_token_ids [num_sorted], expert_ids [num_sorted / moe_block_size],
 *   num_tokens_post_padded [1]: int32 device arrays (vLLM's moe_align_block_size output)
 *   topk_weights [size_m * top_k] fp32 (read only when mul_topk_weights)
 *   c            [size_m * top_k, N], dtype of a, row stride ldc
 *   workspace    device scratch of fp4_moe_workspace_bytes(num_sorted, moe_block_size, K)
 *                bytes, 256-byte aligned: the routed activation rows quantised once, in
 *                sorted order, and the table of same-expert block runs the GEMM walks
 * moe_block_size in [1, 64]; K % 32 == 0.
 */
int64_t fp4_moe_workspace_bytes(int64_t num_sorted, int moe_block_size, int64_t K);
int fp4_moe_mxf4(const void* a, int64_t lda, int dtype, const void* w_codes, const void* w_sf_tiled,
                 int64_t num_experts, const int32_t* sorted_token_ids, const int32_t* expert_ids,
                 const int32_t* num_tokens_post_padded, const float* topk_weights, int64_t num_sorted,
                 int moe_block_size, int top_k, int mul_topk_weights, void* c, int64_t ldc,
                 int64_t size_m, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                 void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* QDQ_B200_H_ */
