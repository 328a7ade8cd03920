// C-ABI entry of the Sage3 FP4 / FP8 attention (pre-pass + flash kernel).
#include "attn_common.cuh"

using namespace qdqb200;

// Head dims the kernels take: 128, and 32 / 64 / 96 zero-extended to 128.
static bool head_dim_ok(int64_t D) { return D == 32 || D == 64 || D == 96 || D == 128; }

extern "C" int64_t sage3_attn_workspace_bytes(int64_t B, int64_t L, int64_t H, int64_t D) {
  if (B <= 0 || L <= 0 || H <= 0 || !head_dim_ok(D)) return 0;
  return attn::carve(static_cast<int>(B), static_cast<int>(H), static_cast<int>(L), nullptr, nullptr);
}

extern "C" int sage3_fp4_attn(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t L,
                              int64_t H, int64_t D, const int64_t* strides, float sm_scale, int quant_format,
                              int acc_mode, int causal, int smoothing, int dtype, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  if (B < 0 || L < 0 || H < 0) return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: negative shape");
  if (B == 0 || L == 0 || H == 0) return QDQ_OK;
  if (!head_dim_ok(D))
    return fail(QDQ_ERR_UNSUPPORTED, "sage3_fp4_attn: head_dim %lld (this build supports 32, 64, 96 and 128)",
                (long long)D);
  if (dtype != QDQ_DTYPE_BF16 && dtype != QDQ_DTYPE_FP16)
    return fail(QDQ_ERR_UNSUPPORTED, "sage3_fp4_attn: inputs must be bf16 or fp16 (dtype %d)", dtype);
  // quant_format -> (Q/K format, P/V format, emulated P, P prescale); see include/qdq_b200.h
  struct Variant { int qk, pv, emu; float pre; };
  static const Variant kVariants[] = {
      {attn::F_MX4, attn::F_MX4, 0, 1.f},      // 0 mxfp4_hw
      {attn::F_NV4, attn::F_NV4, 1, 2688.f},   // 1 nvfp4
      {attn::F_G9, attn::F_G9, 1, 2688.f},     // 2 mxfp4 (= mxfp4_s1_2level)
      {attn::F_MX8, attn::F_MX8, 0, 1.f},      // 3 mxfp8_hw
      {attn::F_G9, attn::F_G9, 1, 1.f},        // 4 mxfp4_s1
      {attn::F_E8, attn::F_E8, 1, 1.f},        // 5 mxfp8_s1
      {attn::F_E8, attn::F_G9, 1, 1.f},        // 6 mixed_fp8qk_fp4pv
      {attn::F_G9, attn::F_E8, 1, 1.f},        // 7 mixed_fp4qk_fp8pv
      {attn::F_MX8, attn::F_MX4, 0, 1.f},      // 8 mixed_mxfp8qk_mxfp4pv_hw
      {attn::F_MX4, attn::F_MX8, 0, 1.f},      // 9 mixed_mxfp4qk_mxfp8pv_hw
      {attn::F_NV4B32, attn::F_NV4B32, 1, 1.f},  // 10 mxfp4_s1_e4m3
  };
  if (quant_format < 0 || quant_format > 10)
    return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: quant_format must be in [0, 10] (got %d)", quant_format);
  if (smoothing < 0 || smoothing > 3)
    return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: smoothing must be in [0, 3] (bit 0 QK, bit 1 V)");
  if (acc_mode < 0 || acc_mode > 1) return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: acc_mode must be 0 or 1");
  if (!q || !k || !v || !o || !strides) return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: null pointer");
  if (!(sm_scale > 0.f)) return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: sm_scale must be positive");
  if (L > (1 << 24) || B * H > (1 << 20)) return fail(QDQ_ERR_UNSUPPORTED, "sage3_fp4_attn: problem too large");
  for (int i = 0; i < 12; ++i)
    if (strides[i] % 8 != 0) return fail(QDQ_ERR_ALIGNMENT, "sage3_fp4_attn: strides must be multiples of 8 elements");
  const uintptr_t mis = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o);
  if (mis & 15) return fail(QDQ_ERR_ALIGNMENT, "sage3_fp4_attn: q/k/v/o must be 16-byte aligned");
  const int64_t need = sage3_attn_workspace_bytes(B, L, H, D);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(QDQ_ERR_INVALID_ARG, "sage3_fp4_attn: workspace smaller than sage3_attn_workspace_bytes()");
  attn::Problem p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.B = static_cast<int>(B);
  p.H = static_cast<int>(H);
  p.L = static_cast<int>(L);
  p.Lp = static_cast<int>((L + 127) / 128 * 128);
  p.D = static_cast<int>(D);
  p.f16 = dtype == QDQ_DTYPE_FP16 ? 1 : 0;
  p.q_sb = strides[0]; p.q_sn = strides[1]; p.q_sh = strides[2];
  p.k_sb = strides[3]; p.k_sn = strides[4]; p.k_sh = strides[5];
  p.v_sb = strides[6]; p.v_sn = strides[7]; p.v_sh = strides[8];
  p.o_sb = strides[9]; p.o_sn = strides[10]; p.o_sh = strides[11];
  p.sm_scale = sm_scale;
  p.causal = causal ? 1 : 0;
  const Variant& var = kVariants[quant_format];
  p.smoothing = smoothing & 1;
  p.vsmooth = (smoothing >> 1) & 1;
  p.qk_fmt = var.qk;
  p.pv_fmt = var.pv;
  p.emulated = var.emu;
  p.p_prescale = var.pre;
  attn::Workspace w;
  attn::carve(p.B, p.H, p.L, static_cast<uint8_t*>(workspace), &w);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = attn::launch_prepass(p, w, s)) return st;
  return attn::launch_flash(p, w, s);
}
