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

}  // namespace
}  // namespace qdqb200
