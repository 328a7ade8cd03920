// Shared declarations of the Sage3 FP4 attention (pre-pass + flash kernel).
#pragma once

#include "sm100.cuh"

namespace qdqb200 {
namespace attn {

// Operand formats of the two products.
enum Fmt : int {
  F_MX4 = 0,  // E2M1 + E8M0 per 32 (kind::mxf4), 64-byte code rows
  F_NV4 = 1,  // E2M1 + E4M3 per 16 (kind::mxf4nvf4 block16), 64-byte code rows
  F_MX8 = 2,  // E4M3 + E8M0 per 32 (kind::mxf8f6f4), 128-byte code rows
  F_NV4B32 = 3,  // E2M1 + E4M3 per 32: run as block16 (kind::mxf4nvf4) with each
                 // scale in both of its 16-element slots, 64-byte code rows
  // The reference's emulated E8M0 QuantConfigs, quantised with its own steps
  // (scale arithmetic in the input dtype, quantize.py:21-141) and stored as
  // E4M3 codes + E8M0 per 32, run like F_MX8 (kind::mxf8f6f4, 128-byte rows):
  F_G9 = 4,  // E2M1 configs: the 9 magnitudes {0, .5, .75, 1, 1.5, 2, 3, 4, 6}
             // (quant_primitives.py:52-71; 0.75 is not E2M1, every one is E4M3)
  F_E8 = 5,  // E4M3 configs (mxfp8_s1): E4M3 codes, round to nearest even
};

// Formats whose MMA is kind::mxf4nvf4.block16 (two 512-byte scale chunks per 128 K).
__host__ __device__ constexpr bool fmt_block16(int f) { return f == F_NV4 || f == F_NV4B32; }
// Formats held as E4M3 codes (128-byte rows, kind::mxf8f6f4).
__host__ __device__ constexpr bool fmt_e4m3(int f) { return f == F_MX8 || f == F_G9 || f == F_E8; }

// The 9-level grid of the reference's emulated E2M1 (quant_primitives.py:52-71)
// for a >= 0: 0 below 0.25, 0.5 below 0.5, and from 0.5 up the value rounded
// to one mantissa bit with ties upward (adding half of that bit to the fp32
// pattern), capped at 6.  The midpoints 0.625, 0.875, 1.25, 1.75, 2.5, 3.5
// and 5 are exactly the one-bit ties, so every threshold `a < t` of the
// reference's compare chain is reproduced.  Every result is an E4M3 value.
// Used by the pre-pass (Q / K / V codes) and the flash kernel (P codes).
__device__ __forceinline__ float grid9_mag(float a) {
  const float r = __uint_as_float((__float_as_uint(a) + 0x00200000u) & 0xFFC00000u);
  return a < 0.5f ? (a < 0.25f ? 0.0f : 0.5f) : fminf(r, 6.0f);
}

// One attention problem: Q, K, V, O in the NHD layout [B, L, H, D] (D = 128,
// element stride 1) with arbitrary batch / token / head strides (elements).
struct Problem {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  int B, H, L, Lp, D;
  int64_t q_sb, q_sn, q_sh;
  int64_t k_sb, k_sn, k_sh;
  int64_t v_sb, v_sn, v_sh;
  int64_t o_sb, o_sn, o_sh;
  float sm_scale;
  int causal;
  int smoothing;    // per-128-token Q mean / K mean smoothing with the delta_s correction
  int vsmooth;      // V mean subtracted before quantisation, added back to the output
  int qk_fmt;       // Fmt of Q and K
  int pv_fmt;       // Fmt of P and V
  int emulated;     // 1: the reference's emulated-config P handling (P times p_prescale before
                    //    block scaling, l = sum of quantised P); 0: its hardware kernels'
  float p_prescale; // 448*6 (two-level emulated configs) or 1
  int f16;          // q, k, v, o (and the smoothing intermediates) are fp16, else bf16
};

// Device buffers of the pre-pass (carved out of the caller's workspace).
struct Workspace {
  float* ksum;            // [BH, 128]
  __nv_bfloat16* qmean;   // [BH, G, 128]
  uint8_t* qc;            // [BH * Lp, 64] (E2M1) or [BH * Lp, 128] (E4M3 formats)
  uint8_t* qsf;           // [BH * Lp / 128, 1024]
  uint8_t* kc;            // as qc
  uint8_t* ksf;           // [BH * Lp / 128, 1024]
  uint8_t* vt;            // [BH * 128, Lp / 2] (E2M1) or [BH * 128, Lp] (E4M3)
  uint8_t* vsf;           // [BH * Lp / 128, 1024]
  __nv_bfloat16* ds;      // [BH, G, Lp]
  float* vsum;            // [BH, 128] per-channel sums of v (V smoothing)
  float* vmean;           // [BH, 128] bf16(vsum / L), stored as fp32
};

inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

// Carve the workspace; returns total bytes needed (ws may be null to query).
// The code buffers are sized for 8-bit codes, so one size serves every format.
inline int64_t carve(int B, int H, int L, uint8_t* base, Workspace* w) {
  const int64_t BH = static_cast<int64_t>(B) * H;
  const int64_t Lp = (static_cast<int64_t>(L) + 127) / 128 * 128;
  const int64_t G = Lp / 128;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  uint8_t* ksum = take(BH * 128 * 4);
  uint8_t* qmean = take(BH * G * 128 * 2);
  uint8_t* qc = take(BH * Lp * 128);
  uint8_t* qsf = take(BH * G * 1024);
  uint8_t* kc = take(BH * Lp * 128);
  uint8_t* ksf = take(BH * G * 1024);
  uint8_t* vt = take(BH * 128 * Lp);
  uint8_t* vsf = take(BH * G * 1024);
  uint8_t* ds = take(BH * G * Lp * 2);
  uint8_t* vsum = take(BH * 128 * 4);
  uint8_t* vmean = take(BH * 128 * 4);
  if (w) {
    w->ksum = reinterpret_cast<float*>(ksum);
    w->qmean = reinterpret_cast<__nv_bfloat16*>(qmean);
    w->qc = qc;
    w->qsf = qsf;
    w->kc = kc;
    w->ksf = ksf;
    w->vt = vt;
    w->vsf = vsf;
    w->ds = reinterpret_cast<__nv_bfloat16*>(ds);
    w->vsum = reinterpret_cast<float*>(vsum);
    w->vmean = reinterpret_cast<float*>(vmean);
  }
  return off;
}

int launch_prepass(const Problem& p, const Workspace& w, cudaStream_t s);
int launch_flash(const Problem& p, const Workspace& w, cudaStream_t s);

}  // namespace attn
}  // namespace qdqb200
