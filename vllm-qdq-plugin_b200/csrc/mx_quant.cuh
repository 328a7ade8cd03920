// MXFP4 group quantisation shared by the QDQ kernels and the fused decode
// GEMM: the reference's per-dtype exponent / scale rules
// (vllm_qdq_plugin/qdq/mxfp4.py:98-156) and the E2M1 codes of one 32-element
// group.  Everything here reproduces the reference bit for bit.
#pragma once

#include "common.cuh"

namespace qdqb200 {
namespace {

// ---------------------------------------------------------------------------
// per-dtype pieces
// ---------------------------------------------------------------------------
template <int kDtype>
struct Fmt;

template <>
struct Fmt<QDQ_DTYPE_BF16> {
  __device__ static float lo(uint32_t w) { return bf16lo(w); }
  __device__ static float hi(uint32_t w) { return bf16hi(w); }
  __device__ static float one(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
  __device__ static uint32_t pack(float a, float b) { return pack_bf16x2(a, b); }
  __device__ static uint16_t pack1(float a) { return static_cast<uint16_t>(pack_bf16x2(a, 0.f) & 0xFFFFu); }
  __device__ static float amax_value(uint32_t bits) { return __uint_as_float(bits << 16); }
  // E8M0 exponent of the group scale from the group's max |x| bit pattern:
  // round the mantissa up at 0.75 (`+0x20 & 0xFF80`, mxfp4.py:138-140), then
  // clamp(floor(log2) + 127 - 2, 0, 254) (mxfp4.py:142-145).  A rounded max of
  // zero, inf or NaN makes the reference's float->int32 cast of +-inf land on
  // the lower clamp, i.e. exponent 0.
  __device__ static int mx_exp(uint32_t amax_bits) {
    const uint32_t r = (amax_bits + 0x20u) & 0xFF80u;
    const int ef = static_cast<int>((r >> 7) & 0xFFu);
    return (ef == 0 || ef == 255) ? 0 : max(ef - 2, 0);
  }
  // 2^(e-127) as the reference holds it in bf16 (mxfp4.py:146): always exact.
  __device__ static float mx_scale(int e) {
    return e ? __uint_as_float(static_cast<uint32_t>(e) << 23) : __uint_as_float(0x00400000u);
  }
  static constexpr bool kScaleCanBeZero = false;
};

template <>
struct Fmt<QDQ_DTYPE_FP16> {
  __device__ static float lo(uint32_t w) { return f16lo(w); }
  __device__ static float hi(uint32_t w) { return f16hi(w); }
  __device__ static float one(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  __device__ static uint32_t pack(float a, float b) { return pack_f16x2(a, b); }
  __device__ static uint16_t pack1(float a) { return static_cast<uint16_t>(pack_f16x2(a, 0.f) & 0xFFFFu); }
  __device__ static float amax_value(uint32_t bits) { return __half2float(__ushort_as_half(static_cast<unsigned short>(bits))); }
  // fp16 variant of the same rule (`+0x100 & 0xFC00`, exponent bias 15).
  __device__ static int mx_exp(uint32_t amax_bits) {
    const uint32_t r = (amax_bits + 0x100u) & 0xFC00u;
    const int ef = static_cast<int>((r >> 10) & 0x1Fu);
    return (ef == 0 || ef == 31) ? 0 : ef + 110;
  }
  // In fp16, 2^(e-127) underflows to 0 for e == 0 and is exact otherwise
  // (e >= 111 for every finite non-tiny group).
  __device__ static float mx_scale(int e) {
    return e ? __uint_as_float(static_cast<uint32_t>(e) << 23) : 0.0f;
  }
  static constexpr bool kScaleCanBeZero = true;
};

// fp16 groups whose scale is 0: the reference divides by zero, turning x != 0
// into +-inf and +-0 into a NaN whose sign on x86 is negative; the E2M1
// simulation maps both to +-6 and the final multiply by the zero scale leaves
// a signed zero.  Result: copysign(0, x) for x != 0, -0 for x == +-0.
__device__ __forceinline__ uint16_t fp16_zero_scale_result(uint16_t xb) {
  return ((xb & 0x7FFFu) == 0) ? static_cast<uint16_t>(0x8000u) : static_cast<uint16_t>(xb & 0x8000u);
}
__device__ __forceinline__ uint32_t fp16_zero_scale_word(uint32_t w) {
  return static_cast<uint32_t>(fp16_zero_scale_result(static_cast<uint16_t>(w & 0xFFFFu))) |
         (static_cast<uint32_t>(fp16_zero_scale_result(static_cast<uint16_t>(w >> 16))) << 16);
}

// E2M1 byte holding two signed zeros with the signs of an fp16x2 word.
__device__ __forceinline__ uint32_t zero_codes_of(uint32_t w) {
  return ((w >> 12) & 0x8u) | ((w >> 24) & 0x80u);
}

__device__ __forceinline__ uint32_t absmax8(const uint4& v) {
  const uint32_t m = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                              __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return max(m & 0xFFFFu, m >> 16);
}

// MXFP4 codes of one 32-element group held as four 16-byte chunks (8
// elements each): returns the E8M0 exponent byte and writes the four code
// words (element 2j of a chunk in the low nibble of byte j).  These are the
// codes the QDQ kernel emits for the same group.
template <int kDtype>
__device__ __forceinline__ int mx_group_codes(const uint4 (&v)[4], uint32_t (&code)[4]) {
  using F = Fmt<kDtype>;
  const uint32_t amax = max(max(absmax8(v[0]), absmax8(v[1])), max(absmax8(v[2]), absmax8(v[3])));
  const int e = F::mx_exp(amax);
  const float inv = __uint_as_float(static_cast<uint32_t>(254 - e) << 23);  // 1/scale, exact
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    if (F::kScaleCanBeZero && e == 0) {
      uint32_t cw = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) cw |= zero_codes_of(fp16_zero_scale_word(w[j])) << (8 * j);
      code[c] = cw;
    } else {
      float sv[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = mul_f32x2(make_float2(F::lo(w[j]), F::hi(w[j])), make_float2(inv, inv));
        sv[2 * j] = t.x;
        sv[2 * j + 1] = t.y;
      }
      code[c] = cvt_e2m1x8(sv[0], sv[1], sv[2], sv[3], sv[4], sv[5], sv[6], sv[7]);
    }
  }
  return e;
}


// ---------------------------------------------------------------------------
// NVFP4 group math (nvfp4_emulation_utils.py:439-452 and :474-476)
// ---------------------------------------------------------------------------
constexpr float kRecip6 = 1.0f / 6.0f;  // fp32 value of vLLM's FLOAT4_E2M1_MAX_RECIPROCAL

struct NvGroup {
  float out_scale;  // 1 / (scale * (1/gs))  with vLLM's zero-safe reciprocal
  float deq;        // scale / gs
  uint32_t sbyte;   // E4M3 byte of the block scale
};

__device__ __forceinline__ float zero_safe_recip(float t) {
  // get_reciprocal(t) = 1 / (t + (t == 0) * 1e8)   (nvfp4_emulation_utils.py:415-418)
  return __fdiv_rn(1.0f, __fadd_rn(t, t == 0.0f ? 1e8f : 0.0f));
}

__device__ __forceinline__ NvGroup nv_group(float vec_max, float gs, float rgs) {
  float s = __fmul_rn(gs, __fmul_rn(vec_max, kRecip6));
  s = fminf(fmaxf(s, -448.0f), 448.0f);
  NvGroup g;
  g.sbyte = e4m3_byte(s);
  s = round_e4m3(s);
  g.out_scale = zero_safe_recip(__fmul_rn(s, rgs));
  g.deq = __fdiv_rn(s, gs);
  return g;
}

// Codes of two elements x*out_scale.  The reference clamps to +-6 and rounds
// to nearest-even (nvfp4_emulation_utils.py:450-451, :425-436): the
// satfinite E2M1 conversion does both.  cast_to_fp4 multiplies by
// torch.sign(), which is +0 for a -0 product (x == -0, or an underflow), so a
// zero product is encoded as +0.
__device__ __forceinline__ uint32_t nv_codes(float xa, float xb, float out_scale) {
  const float2 p = mul_f32x2(make_float2(xa, xb), make_float2(out_scale, out_scale));
  uint32_t byte = cvt_e2m1x2(p.x, p.y);
  if (p.x == 0.0f) byte &= 0xF7u;
  if (p.y == 0.0f) byte &= 0x7Fu;
  return byte;
}

// With out_scale >= 2^-16 no nonzero bf16 or fp16 input (smallest magnitude
// 2^-133, resp. 2^-24) has a product below the smallest fp32 subnormal
// 2^-149, so the only zero products are those of x == +-0.
constexpr float kNoUnderflowScale = 0x1p-16f;

// x * out_scale for 8 elements, with a zero product made +0 (see nv_codes):
// the product is formed as fma(x, out_scale, zero) with `zero` = +0.0 passed
// in as a kernel argument (an operand the compiler cannot treat as a
// constant), so an exact -0 product becomes -0 + +0 = +0 under RN while every
// other product is rounded exactly once, as by a plain multiply.
__device__ __forceinline__ void nv_scale8(const uint32_t (&w)[4], float out_scale, float zero, float (&sv)[8],
                                          bool fp16) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = fp16 ? f16lo(w[j]) : bf16lo(w[j]);
    const float b = fp16 ? f16hi(w[j]) : bf16hi(w[j]);
    const float2 t = fma_f32x2(make_float2(a, b), make_float2(out_scale, out_scale), make_float2(zero, zero));
    sv[2 * j] = t.x;
    sv[2 * j + 1] = t.y;
  }
}

// NVFP4 codes of one 16-element group (two 16-byte chunks of bf16/fp16, in
// order) with the per-tensor global scale gs (rgs = its zero-safe
// reciprocal): the codes and E4M3 scale byte of vLLM's NVFP4 quantisation,
// as nvfp4_vec_kernel computes them.  code[c] holds chunk c's eight codes.
template <int kDtype>
__device__ __forceinline__ uint32_t nv_group_codes(const uint4 (&v)[2], float gs, float rgs, float zero,
                                                   uint32_t (&code)[2]) {
  using F = Fmt<kDtype>;
  const uint32_t amax = max(absmax8(v[0]), absmax8(v[1]));
  const NvGroup g = nv_group(F::amax_value(amax), gs, rgs);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    if (g.out_scale >= kNoUnderflowScale) {
      float sv[8];
      nv_scale8(w, g.out_scale, zero, sv, kDtype == QDQ_DTYPE_FP16);
      code[c] = cvt_e2m1x8(sv[0], sv[1], sv[2], sv[3], sv[4], sv[5], sv[6], sv[7]);
    } else {
      uint32_t cw = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) cw |= nv_codes(F::lo(w[j]), F::hi(w[j]), g.out_scale) << (8 * j);
      code[c] = cw;
    }
  }
  return g.sbyte;
}

}  // namespace
}  // namespace qdqb200
