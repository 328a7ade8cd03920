// Shared helpers for the sm_100a kernels behind include/qdq_b200.h.
//
// Everything here is device-side bit manipulation or thin inline-PTX wrappers
// around conversion instructions that exist on sm_100a:
//   cvt.rn.satfinite.e2m1x2.f32   (two fp32 -> packed E2M1 pair, RNE, saturate at 6)
//   cvt.rn.f16x2.e2m1x2           (packed E2M1 pair -> two exact fp16)
//   cvt.rn.satfinite.e4m3x2.f32   (two fp32 -> packed E4M3 pair, RNE)
//   cvt.rn.f16x2.e4m3x2           (packed E4M3 pair -> two exact fp16)
// No math-library routine is re-implemented here.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qdq_b200.h"

namespace qdqb200 {

// ---------------------------------------------------------------------------
// host-side error plumbing (one message per calling thread)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);
int device_sm_count();  // SM count of the current device (cached)
// Fused small-M MXFP4 linear (gemm_decode.cu): activation quantisation inside
// the GEMM producer, one launch; M in [1, 64], 16-byte aligned activation rows.
// MXFP4 codes + E8M0 scales in the GEMM's tiled layout in one pass (K % 256 == 0).
int qdq_mxfp4_codes_tiled(const void* x, void* codes, void* sf_tiled, int64_t M, int64_t K, int64_t ldx,
                          int dtype, void* stream);
// NVFP4 codes + E4M3 scales in the block16 GEMM's tiled layout in one pass
// against the device scalar *global_scale (K % 256 == 0).
int qdq_nvfp4_codes_tiled(const void* x, const float* global_scale, void* codes, void* sf_tiled, int64_t M,
                          int64_t K, int64_t ldx, int dtype, void* stream);
int fp4_linear_decode(const void* a, int64_t lda, int dtype, const void* w_codes, const void* w_sf_tiled,
                      const void* bias, void* c, int64_t M, int64_t N, int64_t K, int64_t ldw_bytes,
                      int64_t ldc, void* stream);
// The same for NVFP4 weights (E4M3 scales per 16 in the block-16 tiled layout,
// tensor scale w_gs) with the activation quantised to NVFP4 against the device
// scalar *a_gs (a_gs == nullptr: 2688 / max |a|, computed in the kernel); the
// output is scaled by w_gs / gs_a.
int fp4_linear_decode_nvf4(const void* a, int64_t lda, int dtype, const float* a_gs, const void* w_codes,
                           const void* w_sf_tiled, float w_gs, const void* bias, void* c, int64_t M, int64_t N,
                           int64_t K, int64_t ldw_bytes, int64_t ldc, void* stream);
// gs = 2688 / max |x| of a small activation (the decode linear's rows) by one
// cluster of CTAs, writing *gs_out; lets the next kernel launch early
// (programmatic dependent launch).  16-byte aligned rows, K % 8 == 0.
int launch_global_scale_small(const void* x, float* gs_out, int64_t M, int64_t K, int64_t ldx, int dtype,
                              cudaStream_t s);
// Device address of the library's status word on the current device (kernels
// record bounded-wait timeouts there); nullptr + error message on failure.
int* device_status_ptr();

// ---------------------------------------------------------------------------
// device-side conversion helpers
// ---------------------------------------------------------------------------

// Packs RNE-to-E2M1 codes of (lo, hi) into one byte: lo -> bits 0..3, hi -> bits 4..7.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t out;
  asm(
      "{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// Expands one packed E2M1 byte into an fp16x2 word (bits 0..3 -> low half).
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm(
      "{\n\t.reg .b8 t;\n\t"
      "cvt.u8.u32 t, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(out)
      : "r"(byte));
  return out;
}

// Eight values (pairs v[2i], v[2i+1]) -> RNE E2M1 codes packed into one word
// (element 2i in the low nibble of byte i), without widening each byte.
__device__ __forceinline__ uint32_t cvt_e2m1x8(float v0, float v1, float v2, float v3, float v4, float v5,
                                               float v6, float v7) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v0), "f"(v1), "f"(v2), "f"(v3), "f"(v4), "f"(v5), "f"(v6), "f"(v7));
  return out;
}

// Eight values -> RNE E2M1 codes (returned packed) and the same codes decoded
// back to four exact fp16x2 words h[0..3] (pair i in h[i]).
__device__ __forceinline__ uint32_t e2m1_roundtrip8(const float (&v)[8], uint32_t (&h)[4]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %8, %7;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %10, %9;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %12, %11;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %4, b3;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out), "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

// RNE fp32 -> E4M3 (saturating) -> back to fp32, exactly.
__device__ __forceinline__ float round_e4m3(float v) {
  uint32_t h2;
  asm(
      "{\n\t.reg .b16 t;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 t, %1, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, t;\n\t}"
      : "=r"(h2)
      : "f"(v));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

// Four fp32 -> four E4M3 bytes, v0 in the low byte (RNE, saturating to
// +-448).  cvt's first source goes to the high byte of each pair.
__device__ __forceinline__ uint32_t cvt_e4m3x4(float v0, float v1, float v2, float v3) {
  uint32_t r;
  asm(
      "{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(r)
      : "f"(v0), "f"(v1), "f"(v2), "f"(v3));
  return r;
}

// RNE fp32 -> E4M3 byte (saturating).
__device__ __forceinline__ uint32_t e4m3_byte(float v) {
  uint32_t out;
  asm(
      "{\n\t.reg .b16 t;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 t, %1, %1;\n\t"
      "cvt.u32.u16 %0, t;\n\t}"
      : "=r"(out)
      : "f"(v));
  return out & 0xFFu;
}

__device__ __forceinline__ float f16lo(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
__device__ __forceinline__ float f16hi(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Two fp32 -> packed bf16x2 / f16x2 with round-to-nearest-even (subnormals kept).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t out;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
  return out;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t out;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
  return out;
}

// Packed fp32 pair arithmetic (sm_100 f32x2 instructions): each lane is an
// ordinary IEEE round-to-nearest-even operation, subnormals kept.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 unpack_f32x2(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ float2 mul_f32x2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f32x2(a.x, a.y)), "l"(pack_f32x2(b.x, b.y)));
  return unpack_f32x2(d);
}
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f32x2(a.x, a.y)), "l"(pack_f32x2(b.x, b.y)));
  return unpack_f32x2(d);
}
__device__ __forceinline__ float2 fma_f32x2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(pack_f32x2(a.x, a.y)), "l"(pack_f32x2(b.x, b.y)), "l"(pack_f32x2(c.x, c.y)));
  return unpack_f32x2(d);
}

// Streaming 16-byte global load / store (data is touched exactly once).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace qdqb200
